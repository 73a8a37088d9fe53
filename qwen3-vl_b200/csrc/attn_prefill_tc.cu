// a6/a7: causal GQA prefill attention on the 5th-generation tensor cores
// (tcgen05 + TMEM), flash-style with an online softmax in fp32.
//
// Semantics are those of q3_attn_prefill (attn_prefill.cu): the S > 1 eager
// attention of forward_layer (model_fused.py:248-262) and
// prefill_gqa_flash_attention (kernels/prefill_attention.py:28-149);
// out = softmax(q k^T * scale + causal) v, query row s at absolute position
// start_pos + s, head h reading KV head h / (Hq/Hkv).
//
// One CTA = one 128-row query block of one head, 256 threads:
//   warp 0      TMA producer: Q once (two 128x64 SW128 boxes), then K and V
//               tiles of 64 keys (two 64x64 boxes each) into a 2-deep ring;
//   warp 1      MMA issuer (one thread): S_j = Q K_j^T (M=128, N=64, K=128)
//               into TMEM, O_j = P_j V_j (M=128, N=128, K=64) into TMEM; S of
//               tile j+1 is issued before O of tile j so QK^T overlaps softmax;
//   warps 2-3   V transposers: V_j [keys, d] -> V_j^T [d, keys] in the 128-byte
//               swizzled K-major layout the MMA reads (every operand is
//               K-major: the descriptors are the GEMM's); rows of keys past
//               the cache end are written as zeros;
//   warps 4-7   softmax: thread t owns query row t (TMEM lane t); reads S_j,
//               masks, updates the running max and sum, writes P_j (bf16,
//               swizzled K-major), then folds O_j into fp32 registers with the
//               running-max correction; finally O / l to global memory.
// TMEM: S double-buffered (2 x 64 columns), O_j double-buffered (2 x 128).
// Every wait is bounded; on a timeout the kernel records the error word, stops
// issuing, waits (bounded) for its own copies and MMAs, frees TMEM, returns.
#include <math.h>

#include "common.cuh"

namespace q3 {
namespace {

constexpr int kFM = 128;      // query rows per CTA
constexpr int kFN = 64;       // keys per tile
constexpr int kFD = 128;      // head dim
constexpr int kFThreads = 256;
constexpr int kQBytes = kFM * kFD * 2;    // 32 KB (two 16 KB boxes)
constexpr int kKVBytes = kFN * kFD * 2;   // 16 KB (two 8 KB boxes)
constexpr int kPBytes = kFM * kFN * 2;    // 16 KB
constexpr int kVTBytes = kFD * kFN * 2;   // 16 KB
// smem: Q | K[2] | V[2] | VT[2] | P[2]
constexpr int kOffK = kQBytes;
constexpr int kOffV = kOffK + 2 * kKVBytes;
constexpr int kOffVT = kOffV + 2 * kKVBytes;
constexpr int kOffP = kOffVT + 2 * kVTBytes;
constexpr int kOffBar = kOffP + 2 * kPBytes;   // 163840
constexpr int kFSmem = kOffBar + 256 + 1024;   // + barriers + alignment slack
constexpr uint32_t kTmemCols = 512;            // S: 0 / 64; O: 128 / 256

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void sts128v(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                        uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
// byte offset of element (row, col) in a 128-byte-swizzled tile whose rows
// hold 64 bf16 (8 rows x 128 B = one 1024-byte swizzle atom)
__device__ __forceinline__ uint32_t sw128(int row, int col) {
  return row * 128 + ((((col >> 3) ^ (row & 7)) & 7) << 4) + (col & 7) * 2;
}

// a bounded wait whose outcome every lane of the warp shares, so the
// warp-collective instructions that follow (tcgen05 loads and stores,
// __syncwarp) stay converged
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, code));
}

struct FlashParams {
  __nv_bfloat16* out;
  int64_t os_b, os_h, os_s;
  int Hq, Hkv, S, B;
  int64_t q_rows_per_head;   // rows of one (b, h) in the Q map (= S)
  int64_t kv_rows_per_head;  // rows of one (b, kv head) in the K/V maps (= cache length)
  int64_t start;
  int causal;
  float scale_log2;
  int* err;
  // variant 1's V descriptor strides: the byte stride between the two 64-dim
  // blocks (MN, the descriptor's leading offset) and between 8-key groups (K,
  // its stride offset)
  uint32_t v_mn_stride, v_k_stride;
  // variant 2 over a page pool (q3_attn_prefill_tc_paged): K/V maps are 2-D
  // over [num_pages * Hkv * page_tokens, 128]; key position t of sequence b
  // lives in page pages[b * pages_stride + t / page_tokens]
  const int32_t* pages;
  int64_t pages_stride;
  int page_tokens, num_pages;
};

__global__ void __launch_bounds__(kFThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                           const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, FlashParams p) {
  pdl_wait();
  pdl_launch();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t s_base = smem_u32(smem);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* kv_full = bar + 1;    // [2]
  uint64_t* kv_empty = bar + 3;   // [2] MMA commit (K done) + one per transposer warp (V done)
  uint64_t* s_full = bar + 5;     // [2]
  uint64_t* s_free = bar + 7;     // [2] 128 softmax threads
  uint64_t* p_full = bar + 9;     // [2] 128 softmax threads
  uint64_t* vt_full = bar + 11;   // [2] 64 transposer threads
  uint64_t* o_full = bar + 13;    // [2]
  uint64_t* o_free = bar + 15;    // [2] 128 softmax threads
  uint64_t* mma_done = bar + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.Hq / p.Hkv);
  const int q0 = qb * kFM;
  const int q_valid = min(kFM, p.S - q0);
  const int64_t kv_total = p.start + p.S;
  const int64_t kv_need = p.causal ? min64(p.start + q0 + kFM, kv_total) : kv_total;
  const int n_kb = (int)((kv_need + kFN - 1) / kFN);
  const int q_row0 = (int)(((int64_t)b * p.Hq + h) * p.q_rows_per_head + q0);
  const int kv_row0 = (int)(((int64_t)b * p.Hkv + kvh) * p.kv_rows_per_head);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 3);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&vt_full[i], 64);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 128);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kQBytes);
      tma_load_2d(smem, &tmQ, q_full, 0, q_row0, kCacheEvictNormal);
      tma_load_2d(smem + kQBytes / 2, &tmQ, q_full, 64, q_row0, kCacheEvictNormal);
      int issued = 0;
      for (int j = 0; j < n_kb && !*abort_flag; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1, p.err, 0x601)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* dk = smem + kOffK + s * kKVBytes;
        uint8_t* dv = smem + kOffV + s * kKVBytes;
        const int y = kv_row0 + j * kFN;
        mbar_arrive_expect_tx(&kv_full[s], 2 * kKVBytes);
        tma_load_2d(dk, &tmK, &kv_full[s], 0, y, kCacheEvictNormal);
        tma_load_2d(dk + kKVBytes / 2, &tmK, &kv_full[s], 64, y, kCacheEvictNormal);
        tma_load_2d(dv, &tmV, &kv_full[s], 0, y, kCacheEvictNormal);
        tma_load_2d(dv + kKVBytes / 2, &tmV, &kv_full[s], 64, y, kCacheEvictNormal);
        issued = j + 1;
      }
      // on an abort, let the copies this thread issued land before the CTA exits
      mbar_wait(q_full, 0, nullptr, 0);
      for (int j = max(0, issued - 2); j < issued; ++j)
        mbar_wait(&kv_full[j & 1], (j >> 1) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kFM, kFN);
      constexpr uint32_t idesc_o = umma_idesc_bf16(kFM, kFD);
      bool ok = mbar_wait(q_full, 0, p.err, 0x602);
      tc_fence_after();
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&kv_full[s], (j >> 1) & 1, p.err, 0x603)) return false;
        if (j >= 2 && !mbar_wait(&s_free[s], ((j >> 1) - 1) & 1, p.err, 0x604)) return false;
        tc_fence_after();
        const uint32_t d = tmem + s * kFN;
#pragma unroll
        for (int ks = 0; ks < kFD / 16; ++ks) {
          const uint32_t qa = s_base + (ks >> 2) * (kQBytes / 2);
          const uint32_t kb = s_base + kOffK + s * kKVBytes + (ks >> 2) * (kKVBytes / 2);
          tc_mma_bf16(d, umma_desc_k_sw128(qa) + 2 * (ks & 3),
                      umma_desc_k_sw128(kb) + 2 * (ks & 3), idesc_s, ks != 0);
        }
        tc_commit(&s_full[s]);
        tc_commit(&kv_empty[s]);  // K of this stage consumed
        return true;
      };
      if (ok && n_kb > 0) ok = issue_s(0);
      for (int j = 0; ok && j < n_kb && !*abort_flag; ++j) {
        if (j + 1 < n_kb && !issue_s(j + 1)) { ok = false; break; }
        const int s = j & 1;
        if (!mbar_wait(&p_full[s], (j >> 1) & 1, p.err, 0x605) ||
            !mbar_wait(&vt_full[s], (j >> 1) & 1, p.err, 0x606) ||
            (j >= 2 && !mbar_wait(&o_free[s], ((j >> 1) - 1) & 1, p.err, 0x607))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + 2 * kFN + s * kFD;
        const uint32_t pa = s_base + kOffP + s * kPBytes;
        const uint32_t vb = s_base + kOffVT + s * kVTBytes;
#pragma unroll
        for (int ks = 0; ks < kFN / 16; ++ks)
          tc_mma_bf16(d, umma_desc_k_sw128(pa) + 2 * ks, umma_desc_k_sw128(vb) + 2 * ks, idesc_o,
                      ks != 0);
        tc_commit(&o_full[s]);
      }
      if (!ok) *abort_flag = 1;
      // every MMA issued above has completed before TMEM is released
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, 0);
    }
  } else if (warp < 4) {
    // ----------------------------- V transposers ------------------------------
    const int t = threadIdx.x - 64;  // 0..63
    for (int j = 0; j < n_kb; ++j) {
      if (__any_sync(0xffffffffu, *abort_flag != 0)) break;  // as a warp
      const int s = j & 1;
      if (!warp_wait(&kv_full[s], (j >> 1) & 1, p.err, 0x608)) { *abort_flag = 1; break; }
      // VT[s] was last read by the MMA of tile j - 2
      if (j >= 2 && !warp_wait(&o_full[s], ((j >> 1) - 1) & 1, p.err, 0x609)) {
        *abort_flag = 1;
        break;
      }
      const uint32_t v = s_base + kOffV + s * kKVBytes;
      const uint32_t vt = s_base + kOffVT + s * kVTBytes;
      // thread t: key pair kp = t & 31 (keys 2kp, 2kp+1), dims d in [ (t>>5)*64, +64 ).
      // Keys at or past the end of the cache get zero rows: their P is 0, and
      // whatever bytes the copy brought (the next head's rows, stale cache)
      // must not turn 0 * V into NaN.
      const int kp = t & 31, dh = t >> 5;
      const int64_t key0 = (int64_t)j * kFN + 2 * kp;
      const uint32_t keep0 = key0 < kv_total ? 0xffffffffu : 0u;
      const uint32_t keep1 = key0 + 1 < kv_total ? 0xffffffffu : 0u;
#pragma unroll 4
      for (int dd = 0; dd < 64; dd += 2) {
        const int d = dh * 64 + dd;
        const int box = d >> 6, dc = d & 63;
        const uint32_t r0 = lds32(v + box * (kKVBytes / 2) + sw128(2 * kp, dc)) & keep0;
        const uint32_t r1 = lds32(v + box * (kKVBytes / 2) + sw128(2 * kp + 1, dc)) & keep1;
        // (key 2kp, dims d, d+1) and (key 2kp+1, dims d, d+1) -> rows d, d+1 of VT
        sts32(vt + sw128(d, 2 * kp), __byte_perm(r0, r1, 0x5410));
        sts32(vt + sw128(d + 1, 2 * kp), __byte_perm(r0, r1, 0x7632));
      }
      fence_async_smem();
      mbar_arrive(&vt_full[s]);
      // V of this stage consumed by this warp.  Each warp releases its own
      // share (no named barrier across the two warps: one that left the loop
      // on a timeout would hold the other at that barrier for good).
      __syncwarp();
      if (lane == 0) mbar_arrive(&kv_empty[s]);
    }
  } else {
    // -------------------------------- softmax ---------------------------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int64_t qpos = p.start + q0 + row;
    float m = -INFINITY, l = 0.f;
    float o[kFD];
#pragma unroll
    for (int i = 0; i < kFD; ++i) o[i] = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kb; ++j) {
      const int s = j & 1;
      if (!warp_wait(&s_full[s], (j >> 1) & 1, p.err, 0x60a)) { ok = false; break; }
      tc_fence_after();
      float sc[kFN];
      {
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_ld_32cols(tmem + lane_off + s * kFN + c * 32, r);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) sc[c * 32 + i] = __uint_as_float(r[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_free[s]);
      const int64_t kbase = (int64_t)j * kFN;
      float mx = m;
#pragma unroll
      for (int c = 0; c < kFN; ++c) {
        const int64_t key = kbase + c;
        float x = sc[c] * p.scale_log2;
        if (key >= kv_total || (p.causal && key > qpos)) x = -INFINITY;
        sc[c] = x;
        mx = fmaxf(mx, x);
      }
      const float base = (mx == -INFINITY) ? 0.f : mx;
      const float corr = exp2f(m - base);  // m = -inf -> 0
      float rs = 0.f;
      const uint32_t prow = s_base + kOffP + s * kPBytes;
#pragma unroll
      for (int c = 0; c < kFN; c += 8) {
        uint32_t w4[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const float p0 = exp2f(sc[c + e] - base), p1 = exp2f(sc[c + e + 1] - base);
          rs += p0 + p1;
          w4[e / 2] = pack_bf16x2(p0, p1);
        }
        sts128v(prow + sw128(row, c), w4[0], w4[1], w4[2], w4[3]);
      }
      fence_async_smem();
      mbar_arrive(&p_full[s]);
      l = l * corr + rs;
      m = mx;
      // fold O_j in, after rescaling the running sum to the new maximum
      if (!warp_wait(&o_full[s], (j >> 1) & 1, p.err, 0x60b)) { ok = false; break; }
      tc_fence_after();
      {
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < kFD / 32; ++c) {
          tmem_ld_32cols(tmem + lane_off + 2 * kFN + s * kFD + c * 32, r);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c * 32 + i] = fmaf(o[c * 32 + i], corr, __uint_as_float(r[i]));
        }
      }
      tc_fence_before();
      mbar_arrive(&o_free[s]);
    }
    if (!ok) *abort_flag = 1;
    if (ok && row < q_valid) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = p.out + b * p.os_b + h * p.os_h + (int64_t)(q0 + row) * p.os_s;
#pragma unroll
      for (int d = 0; d < kFD; d += 8) {
        uint4 u;
        u.x = pack_bf16x2(o[d] * inv, o[d + 1] * inv);
        u.y = pack_bf16x2(o[d + 2] * inv, o[d + 3] * inv);
        u.z = pack_bf16x2(o[d + 4] * inv, o[d + 5] * inv);
        u.w = pack_bf16x2(o[d + 6] * inv, o[d + 7] * inv);
        *reinterpret_cast<uint4*>(dst + d) = u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Variant 1: V read in place as an MN-major operand, O accumulated in TMEM.
//   warp 0      TMA producer, as in variant 0;
//   warp 1      MMA issuer: S_j = Q K_j^T into TMEM S[j&1]; O += P_j V_j into
//               one TMEM accumulator across all tiles, with V_j taken straight
//               from its TMA tile through an MN-major descriptor (rows of 64
//               head dims per key, 1024-byte atoms of 8 keys; the two 64-dim
//               boxes are the two MN blocks), so nothing is transposed;
//   warps 2-5   softmax, row (warp % 4) * 32 + lane (TMEM lane quarter warp % 4).
//               P_j is taken relative to a base that moves only when a row's
//               maximum grows by more than 2^8 (P stays <= 256 between moves);
//               when it moves, the warp rescales its rows of O in TMEM, after
//               O_{j-1} has completed and before it releases P_j.
// P[s] is reused two tiles later, after O of that tile completes: o_full[s]
// counts the O MMAs of tiles with parity s, so each softmax wait is for the
// next phase of one barrier (never two phases ahead).
// TMEM: S at columns 0 / 64, O at 128..255 (256 allocated).
constexpr int kMnThreads = 192;
constexpr int kMnOffK = kQBytes;
constexpr int kMnOffV = kMnOffK + 2 * kKVBytes;
constexpr int kMnOffP = kMnOffV + 2 * kKVBytes;
constexpr int kMnOffBar = kMnOffP + 2 * kPBytes;    // 131072
constexpr int kMnSmem = kMnOffBar + 256 + 1024;
constexpr uint32_t kMnTmemCols = 256;
constexpr uint32_t kMnTmemO = 128;
constexpr float kRescaleLog2 = 8.0f;


__global__ void __launch_bounds__(kMnThreads, 1)
    attn_prefill_tc_mn_kernel(const __grid_constant__ CUtensorMap tmQ,
                              const __grid_constant__ CUtensorMap tmK,
                              const __grid_constant__ CUtensorMap tmV, FlashParams p) {
  pdl_wait();
  pdl_launch();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t s_base = smem_u32(smem);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kMnOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* kv_full = bar + 1;    // [2]
  uint64_t* kv_empty = bar + 3;   // [2] MMA commit after O_j (S_j and O_j done)
  uint64_t* s_full = bar + 5;     // [2]
  uint64_t* p_full = bar + 7;     // [2] 128 softmax threads
  uint64_t* o_full = bar + 9;     // [2] O MMAs of even / odd tiles
  uint64_t* mma_done = bar + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.Hq / p.Hkv);
  const int q0 = qb * kFM;
  const int q_valid = min(kFM, p.S - q0);
  const int64_t kv_total = p.start + p.S;
  const int64_t kv_need = p.causal ? min64(p.start + q0 + kFM, kv_total) : kv_total;
  const int n_kb = (int)((kv_need + kFN - 1) / kFN);
  const int q_row0 = (int)(((int64_t)b * p.Hq + h) * p.q_rows_per_head + q0);
  const int kv_row0 = (int)(((int64_t)b * p.Hkv + kvh) * p.kv_rows_per_head);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kMnTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kQBytes);
      tma_load_2d(smem, &tmQ, q_full, 0, q_row0, kCacheEvictNormal);
      tma_load_2d(smem + kQBytes / 2, &tmQ, q_full, 64, q_row0, kCacheEvictNormal);
      int issued = 0;
      for (int j = 0; j < n_kb && !*abort_flag; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[s], ((j >> 1) - 1) & 1, p.err, 0x611)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* dk = smem + kMnOffK + s * kKVBytes;
        uint8_t* dv = smem + kMnOffV + s * kKVBytes;
        const int y = kv_row0 + j * kFN;
        mbar_arrive_expect_tx(&kv_full[s], 2 * kKVBytes);
        tma_load_2d(dk, &tmK, &kv_full[s], 0, y, kCacheEvictNormal);
        tma_load_2d(dk + kKVBytes / 2, &tmK, &kv_full[s], 64, y, kCacheEvictNormal);
        tma_load_2d(dv, &tmV, &kv_full[s], 0, y, kCacheEvictNormal);
        tma_load_2d(dv + kKVBytes / 2, &tmV, &kv_full[s], 64, y, kCacheEvictNormal);
        issued = j + 1;
      }
      // let the copies this thread issued land before the CTA exits
      mbar_wait(q_full, 0, nullptr, 0);
      for (int j = max(0, issued - 2); j < issued; ++j)
        mbar_wait(&kv_full[j & 1], (j >> 1) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kFM, kFN);
      constexpr uint32_t idesc_o = umma_idesc_bf16_bmn(kFM, kFD);
      bool ok = mbar_wait(q_full, 0, p.err, 0x612);
      tc_fence_after();
      // S[(j)&1] is free: the softmax released P_{j-2} (read S_{j-2} first),
      // which this thread waited for before issuing O_{j-2}
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&kv_full[s], (j >> 1) & 1, p.err, 0x613)) return false;
        tc_fence_after();
        const uint32_t d = tmem + s * kFN;
#pragma unroll
        for (int ks = 0; ks < kFD / 16; ++ks) {
          const uint32_t qa = s_base + (ks >> 2) * (kQBytes / 2);
          const uint32_t kb = s_base + kMnOffK + s * kKVBytes + (ks >> 2) * (kKVBytes / 2);
          tc_mma_bf16(d, umma_desc_k_sw128(qa) + 2 * (ks & 3),
                      umma_desc_k_sw128(kb) + 2 * (ks & 3), idesc_s, ks != 0);
        }
        tc_commit(&s_full[s]);
        return true;
      };
      if (ok && n_kb > 0) ok = issue_s(0);
      for (int j = 0; ok && j < n_kb && !*abort_flag; ++j) {
        if (j + 1 < n_kb && !issue_s(j + 1)) { ok = false; break; }
        const int s = j & 1;
        if (!mbar_wait(&p_full[s], (j >> 1) & 1, p.err, 0x614)) { ok = false; break; }
        tc_fence_after();
        const uint32_t pa = s_base + kMnOffP + s * kPBytes;
        const uint32_t vb = s_base + kMnOffV + s * kKVBytes;
#pragma unroll
        for (int ks = 0; ks < kFN / 16; ++ks)
          tc_mma_bf16(tmem + kMnTmemO, umma_desc_k_sw128(pa) + 2 * ks,
                      umma_desc_mn_sw128(vb + ks * 2048, p.v_mn_stride, p.v_k_stride), idesc_o,
                      j > 0 || ks > 0);
        tc_commit(&o_full[s]);
        tc_commit(&kv_empty[s]);  // K_j and V_j consumed
      }
      if (!ok) *abort_flag = 1;
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, 0);
    }
  } else {
    // -------------------------------- softmax ---------------------------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int64_t qpos = p.start + q0 + row;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kb; ++j) {
      // the abort flag is read once per lane: leave the loop as a warp
      if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
      const int s = j & 1;
      if (!warp_wait(&s_full[s], (j >> 1) & 1, p.err, 0x615)) { ok = false; break; }
      tc_fence_after();
      float sc[kFN];
      {
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_ld_32cols(tmem + lane_off + s * kFN + c * 32, r);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) sc[c * 32 + i] = __uint_as_float(r[i]);
        }
      }
      const int64_t kbase = (int64_t)j * kFN;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kFN; ++c) {
        const int64_t key = kbase + c;
        float x = sc[c] * p.scale_log2;
        if (key >= kv_total || (p.causal && key > qpos)) x = -INFINITY;
        sc[c] = x;
        mx = fmaxf(mx, x);
      }
      // P[s] was read by O_{j-2}
      if (j >= 2 && !warp_wait(&o_full[s], ((j >> 1) - 1) & 1, p.err, 0x616)) {
        ok = false;
        break;
      }
      const float m_new = fmaxf(m_used, mx);
      const bool move = m_new > m_used + kRescaleLog2;   // -inf + 8 = -inf
      const bool rescale = move && j > 0 && m_used != -INFINITY;
      if (__any_sync(0xffffffffu, rescale)) {
        // O holds tiles 0..j-1 at the old base: wait for O_{j-1}, then scale
        if (!warp_wait(&o_full[(j - 1) & 1], ((j - 1) >> 1) & 1, p.err, 0x617)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float corr = rescale ? exp2f(m_used - m_new) : 1.f;
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < kFD / 32; ++c) {
          const uint32_t a = tmem + lane_off + kMnTmemO + c * 32;
          tmem_ld_32cols(a, r);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
          tmem_st_32cols(a, r);
        }
        tc_wait_st();
      }
      if (move) {
        l *= exp2f(m_used - m_new);  // m_used = -inf: l is 0 and stays 0
        m_used = m_new;
      }
      const float base = (m_used == -INFINITY) ? 0.f : m_used;
      float rs = 0.f;
      const uint32_t prow = s_base + kMnOffP + s * kPBytes;
#pragma unroll
      for (int c = 0; c < kFN; c += 8) {
        uint32_t w4[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const float p0 = exp2f(sc[c + e] - base), p1 = exp2f(sc[c + e + 1] - base);
          rs += p0 + p1;
          w4[e / 2] = pack_bf16x2(p0, p1);
        }
        sts128v(prow + sw128(row, c), w4[0], w4[1], w4[2], w4[3]);
      }
      l += rs;
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[s]);
    }
    if (!ok) *abort_flag = 1;
    // the last O MMA, then O / l to global memory
    if (__all_sync(0xffffffffu, ok && *abort_flag == 0) &&
        warp_wait(&o_full[(n_kb - 1) & 1], ((n_kb - 1) >> 1) & 1, p.err, 0x618)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = p.out + b * p.os_b + h * p.os_h + (int64_t)(q0 + row) * p.os_s;
      uint32_t r[32];
#pragma unroll
      for (int c = 0; c < kFD / 32; ++c) {
        tmem_ld_32cols(tmem + lane_off + kMnTmemO + c * 32, r);
        tc_wait_ld();
        if (row < q_valid) {
#pragma unroll
          for (int d = 0; d < 32; d += 8) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(r[d]) * inv, __uint_as_float(r[d + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(r[d + 2]) * inv, __uint_as_float(r[d + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(r[d + 4]) * inv, __uint_as_float(r[d + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(r[d + 6]) * inv, __uint_as_float(r[d + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c * 32 + d) = u;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kMnTmemCols);
  }
}


// ---------------------------------------------------------------------------
// Variant 2: two query tiles per CTA, 128-key tiles, P kept in TMEM.
//   One CTA holds the same 128 query rows of two heads that share a KV head
//   (G = Hq / Hkv even), so both tiles read the same K/V tiles and masks.
//   warp 0      TMA producer: Q (two heads x two 128x64 boxes), then K_j and
//               V_j (128 keys x two 64-dim boxes each) into 2-deep K and V
//               rings.  The K/V maps are 3-D (dim, key, head) and end at the
//               last valid key, so keys past it arrive as zeros;
//   warp 1      MMA issuer (one thread), alternating between the tiles:
//               S_0(0), S_0(1), then for each j: PV_j(0), S_{j+1}(0), PV_j(1),
//               S_{j+1}(1), where S_j(t) = Q_t K_j^T (M=128, N=128, K=128)
//               goes to TMEM S[t] and PV_j(t) accumulates P_j(t) V_j into
//               TMEM O[t], with P read from TMEM (it overwrites the first 64
//               columns of S[t], two bf16 per column) and V as an MN-major
//               shared-memory operand.  While one tile's softmax runs, the
//               tensor core works on the other tile;
//   warps 2-5   softmax of tile 0, warps 6-9 of tile 1; row 32 (warp % 4) +
//               lane, the warp's TMEM lane quarter.  P_j = 2^(s - m) against a
//               base m that moves only when a row's maximum grows by more
//               than 2^8; when it moves, the row of O[t] is rescaled in TMEM.
//               The commit of S_j(t) also covers PV_{j-1}(t), issued before
//               it, so O[t] is complete when S_j(t) is.  Finally O / l.
// TMEM (512 columns): S[0] 0..127, S[1] 128..255, O[0] 256..383, O[1] 384..511.
constexpr int kPpThreads = 320;           // 10 warps
constexpr int kPpN = 128;                 // keys per tile
constexpr int kPpQBytes = kFM * kFD * 2;  // 32 KB per query tile
constexpr int kPpKVBytes = kPpN * kFD * 2;  // 32 KB per K or V tile
constexpr int kPpHalf = kPpKVBytes / 2;   // one 64-dim box of 128 keys
constexpr int kPpOffK = 2 * kPpQBytes;
constexpr int kPpOffV = kPpOffK + 2 * kPpKVBytes;
constexpr int kPpOffBar = kPpOffV + 2 * kPpKVBytes;  // 196608
constexpr int kPpSmem = kPpOffBar + 256 + 1024;
constexpr uint32_t kPpTmemCols = 512;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// max of three (one instruction on sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// Packed fp32 pairs (one instruction per pair on sm_100).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
// 2^x for a pair on the FMA pipe, so that part of the softmax's exponentials
// leave the MUFU pipe (the MUFU pipe bounds the softmax of a 128-key tile).
// Cody-Waite range reduction, 2^x = 2^j * 2^f with j = round(x) (the 1.5 *
// 2^23 shifter) and f in [-0.5, 0.5], then a degree-5 polynomial for 2^f whose
// coefficients were fitted here by iteratively reweighted least squares for
// the smallest maximum relative error on [-0.5, 0.5] with p(0) = 1: 1.9e-7
// through the fp32 evaluation, the size of ex2.approx's own error, so the bf16
// P of nearly every key (all but about 2 in 10^6) rounds as it does from the
// exact exponential.  (A cubic, 1.0e-4, changed the bf16 rounding of 5 % of
// its keys, enough to flip near-tie greedy tokens downstream.)  2^j is added
// to the exponent field:
// the shifter's low mantissa bits hold j, and shifting its bits left by 23
// leaves exactly j << 23.  x is clamped to -127, where the result is exactly
// 0 (masked keys, x = -inf); results below 2^-126 are flushed towards zero
// as with ex2.approx.ftz.  Inputs above 0 stay exact up to 2^127 (the lazy
// rescale lets x reach +8).
constexpr int kExpPolyLane = 3;  // i % 4 of the key pairs that take the polynomial
constexpr float kExp2C1 = 0.6931470036506653f;
constexpr float kExp2C2 = 0.24022242426872253f;
constexpr float kExp2C3 = 0.05550733581185341f;
constexpr float kExp2C4 = 0.00967150554060936f;
constexpr float kExp2C5 = 0.0013264697045087814f;
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -127.f);
  x.y = fmaxf(x.y, -127.f);
  const float2 t = fadd2(x, make_float2(kShift, kShift));
  const float2 r = fadd2(t, make_float2(-kShift, -kShift));  // round(x), exact
  const float2 f = ffma2(r, make_float2(-1.f, -1.f), x);     // x - round(x), exact
  float2 q = ffma2(f, make_float2(kExp2C5, kExp2C5), make_float2(kExp2C4, kExp2C4));
  q = ffma2(q, f, make_float2(kExp2C3, kExp2C3));
  q = ffma2(q, f, make_float2(kExp2C2, kExp2C2));
  q = ffma2(q, f, make_float2(kExp2C1, kExp2C1));
  q = ffma2(q, f, make_float2(1.f, 1.f));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// The kernel is persistent: min(items, SMs) CTAs, where an item is one
// (query row block, head pair, sequence).  Items run longest first (the
// causal work of a row block grows with its index), dealt to the CTAs in a
// snake order (round r gives item r * grid + c, or r * grid + grid - 1 - c on
// odd rounds) so each CTA's total work is nearly the same.  Barrier phases run
// on across items: the producer loads an item's Q once the previous item's S
// MMAs are done (q_empty), and the first PV of an item overwrites O[t] only
// after the softmax warps have read out the previous item's O[t] (o_empty).
struct PpItem {
  int qb, h0, b;
};
__device__ __forceinline__ int pp_items(const FlashParams& p) {
  return ((p.S + kFM - 1) / kFM) * (p.Hq / 2) * p.B;
}
__device__ __forceinline__ bool pp_item(const FlashParams& p, int round, PpItem& it) {
  const int n = pp_items(p), G = gridDim.x, c = blockIdx.x;
  const int idx = round * G + ((round & 1) ? (G - 1 - c) : c);
  if (idx >= n) return false;
  const int pairs = p.Hq / 2, per = pairs * p.B, nqb = (p.S + kFM - 1) / kFM;
  it.qb = nqb - 1 - idx / per;
  const int rem = idx % per;
  it.h0 = 2 * (rem % pairs);
  it.b = rem / pairs;
  return true;
}

template <bool PAGED>
__global__ void __launch_bounds__(kPpThreads, 1)
    attn_prefill_tc_pp_kernel(const __grid_constant__ CUtensorMap tmQ,
                              const __grid_constant__ CUtensorMap tmK,
                              const __grid_constant__ CUtensorMap tmV, FlashParams p) {
  pdl_wait();
  pdl_launch();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t s_base = smem_u32(smem);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kPpOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;    // [2]
  uint64_t* k_empty = bar + 3;   // [2] MMA commit after S_j of both tiles
  uint64_t* v_full = bar + 5;    // [2]
  uint64_t* v_empty = bar + 7;   // [2] MMA commit after PV_j of both tiles
  uint64_t* s_full = bar + 9;    // [tile] S_j(t) (and PV_{j-1}(t)) complete
  uint64_t* p_full = bar + 11;   // [tile] P_j(t) in TMEM: one arrival per softmax warp
  uint64_t* o_final = bar + 13;  // [tile] the item's last PV of the tile complete
  uint64_t* o_empty = bar + 15;  // [tile] the item's O[t] read out: one arrival per warp
  uint64_t* q_empty = bar + 17;  // the item's S MMAs complete (Q may be replaced)
  uint64_t* mma_done = bar + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t kv_total = p.start + p.S;
  const int G = p.Hq / p.Hkv;
  const int n_items = pp_items(p);
  const int rounds = (n_items + gridDim.x - 1) / gridDim.x;
  auto n_kb_of = [&](int qb) {
    const int64_t kv_need = p.causal ? min64(p.start + qb * kFM + kFM, kv_total) : kv_total;
    return (int)((kv_need + kPpN - 1) / kPpN);
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_final[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kPpTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int T = 0, ic = 0, nk = 0, nv = 0;
      bool ok = true;
      for (int r = 0; ok && r < rounds && !*abort_flag; ++r) {
        PpItem itm;
        if (!pp_item(p, r, itm)) continue;
        const int q0 = itm.qb * kFM, n_kb = n_kb_of(itm.qb);
        const int kvh = itm.h0 / G, kv_plane = itm.b * p.Hkv + kvh;
        if (ic >= 1 && !mbar_wait(q_empty, (ic - 1) & 1, p.err, 0x63b)) { ok = false; break; }
        mbar_arrive_expect_tx(q_full, 2 * kPpQBytes);
        for (int t = 0; t < 2; ++t) {
          const int qrow = (int)(((int64_t)itm.b * p.Hq + itm.h0 + t) * p.q_rows_per_head + q0);
          tma_load_2d(smem + t * kPpQBytes, &tmQ, q_full, 0, qrow, kCacheEvictNormal);
          tma_load_2d(smem + t * kPpQBytes + kPpQBytes / 2, &tmQ, q_full, 64, qrow,
                      kCacheEvictNormal);
        }
        ++ic;
        for (int j = 0; j < n_kb; ++j, ++T) {
          const int s = T & 1;
          const uint32_t ph_prev = ((T >> 1) - 1) & 1;
          const int key0 = j * kPpN;
          if (T >= 2 && !mbar_wait(&k_empty[s], ph_prev, p.err, 0x631)) { ok = false; break; }
          // paged: the tile's rows in the pool (a 128-key tile never straddles
          // pages); an entry outside the pool is recorded and page 0 read
          int prow = 0;
          if constexpr (PAGED) {
            int pg = p.pages[(int64_t)itm.b * p.pages_stride + key0 / p.page_tokens];
            if (pg < 0 || pg >= p.num_pages) {
              report_timeout(p.err, 0x63a);
              pg = 0;
            }
            prow = (int)(((int64_t)pg * p.Hkv + kvh) * p.page_tokens + key0 % p.page_tokens);
          }
          uint8_t* dk = smem + kPpOffK + s * kPpKVBytes;
          mbar_arrive_expect_tx(&k_full[s], kPpKVBytes);
          if constexpr (PAGED) {
            tma_load_2d(dk, &tmK, &k_full[s], 0, prow, kCacheEvictNormal);
            tma_load_2d(dk + kPpHalf, &tmK, &k_full[s], 64, prow, kCacheEvictNormal);
          } else {
            tma_load_3d(dk, &tmK, &k_full[s], 0, key0, kv_plane, kCacheEvictNormal);
            tma_load_3d(dk + kPpHalf, &tmK, &k_full[s], 64, key0, kv_plane, kCacheEvictNormal);
          }
          nk = T + 1;
          if (T >= 2 && !mbar_wait(&v_empty[s], ph_prev, p.err, 0x632)) { ok = false; break; }
          uint8_t* dv = smem + kPpOffV + s * kPpKVBytes;
          mbar_arrive_expect_tx(&v_full[s], kPpKVBytes);
          if constexpr (PAGED) {
            tma_load_2d(dv, &tmV, &v_full[s], 0, prow, kCacheEvictNormal);
            tma_load_2d(dv + kPpHalf, &tmV, &v_full[s], 64, prow, kCacheEvictNormal);
          } else {
            tma_load_3d(dv, &tmV, &v_full[s], 0, key0, kv_plane, kCacheEvictNormal);
            tma_load_3d(dv + kPpHalf, &tmV, &v_full[s], 64, key0, kv_plane, kCacheEvictNormal);
          }
          nv = T + 1;
        }
      }
      if (!ok) *abort_flag = 1;
      // let the copies this thread issued land before the CTA exits
      if (ic > 0) mbar_wait(q_full, (ic - 1) & 1, nullptr, 0);
      for (int j = max(0, nk - 2); j < nk; ++j) mbar_wait(&k_full[j & 1], (j >> 1) & 1, nullptr, 0);
      for (int j = max(0, nv - 2); j < nv; ++j) mbar_wait(&v_full[j & 1], (j >> 1) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kFM, kPpN);
      constexpr uint32_t idesc_o = umma_idesc_bf16_bmn(kFM, kFD);
      // The MMA loops are unrolled with every descriptor a base plus a
      // constant: a tcgen05.mma of 128 x 128 x 16 takes 64 cycles, and an
      // issue loop that recomputes descriptors per step measured 75-140
      // cycles per MMA on B200, which left the tensor pipe idle half the time.
      // Descriptor start addresses are in 16-byte units (14 bits cover the
      // 256 KB of shared memory), so adding byte offset / 16 to a descriptor
      // is exact.
      auto issue_s = [&](int T, int t) {
        const uint64_t dq = umma_desc_k_sw128(s_base + t * kPpQBytes);
        const uint64_t dk = umma_desc_k_sw128(s_base + kPpOffK + (T & 1) * kPpKVBytes);
        const uint32_t ds = tmem + t * kPpN;
#pragma unroll
        for (int ks = 0; ks < kFD / 16; ++ks)
          tc_mma_bf16(ds, dq + (uint64_t)(((ks >> 2) * (kPpQBytes / 2)) >> 4) + 2 * (ks & 3),
                      dk + (uint64_t)(((ks >> 2) * kPpHalf) >> 4) + 2 * (ks & 3), idesc_s, ks != 0);
        tc_commit(&s_full[t]);
      };
      auto issue_pv = [&](int T, int t, bool first) {
        const uint64_t dv =
            umma_desc_mn_sw128(s_base + kPpOffV + (T & 1) * kPpKVBytes, kPpHalf, 1024u);
        const uint32_t dO = tmem + 2 * kPpN + t * kFD, dp = tmem + t * kPpN;
        tc_mma_bf16_ts(dO, dp, dv, idesc_o, first ? 0u : 1u);
#pragma unroll
        for (int ks = 1; ks < kPpN / 16; ++ks)
          tc_mma_bf16_ts(dO, dp + ks * 8, dv + (uint64_t)((ks * 2048) >> 4), idesc_o, 1u);
      };
      bool ok = true;
      int T = 0, ic = 0;
      for (int r = 0; ok && r < rounds && !*abort_flag; ++r) {
        PpItem itm;
        if (!pp_item(p, r, itm)) continue;
        const int n_kb = n_kb_of(itm.qb);
        if (!mbar_wait(q_full, ic & 1, p.err, 0x633) ||
            !mbar_wait(&k_full[T & 1], (T >> 1) & 1, p.err, 0x634)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_s(T, 0);
        issue_s(T, 1);
        tc_commit(&k_empty[T & 1]);
        if (n_kb == 1) tc_commit(q_empty);
        for (int j = 0; ok && j < n_kb; ++j) {
          const int Tj = T + j;
          if (!mbar_wait(&v_full[Tj & 1], (Tj >> 1) & 1, p.err, 0x635)) { ok = false; break; }
          for (int t = 0; t < 2 && ok; ++t) {
            if (!mbar_wait(&p_full[t], Tj & 1, p.err, 0x636) ||
                (j == 0 && ic >= 1 && !mbar_wait(&o_empty[t], (ic - 1) & 1, p.err, 0x63c))) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(Tj, t, j == 0);
            if (t == 1) tc_commit(&v_empty[Tj & 1]);
            if (j + 1 < n_kb) {
              if (t == 0 && !mbar_wait(&k_full[(Tj + 1) & 1], ((Tj + 1) >> 1) & 1, p.err, 0x637)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_s(Tj + 1, t);
              if (t == 1) {
                tc_commit(&k_empty[(Tj + 1) & 1]);
                if (j + 2 == n_kb) tc_commit(q_empty);  // the item's last S MMAs
              }
            } else {
              tc_commit(&o_final[t]);
            }
          }
        }
        T += n_kb;
        ++ic;
      }
      if (!ok) *abort_flag = 1;
      // every MMA issued above has completed before TMEM is released
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, nullptr, 0);
    }
  } else {
    // -------------------------------- softmax ---------------------------------
    const int t = (warp - 2) >> 2;         // query tile (head h0 + t)
    const int quarter = warp & 3;          // TMEM lane quarter of this warp
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = tmem + lane_off + t * kPpN;
    const uint32_t o_col = tmem + lane_off + 2 * kPpN + t * kFD;
    bool ok = true;
    int T = 0, ic = 0;
    for (int r = 0; ok && r < rounds; ++r) {
      PpItem itm;
      if (!pp_item(p, r, itm)) continue;
      const int q0 = itm.qb * kFM, n_kb = n_kb_of(itm.qb);
      const int q_valid = min(kFM, p.S - q0);
      const int64_t qpos = p.start + q0 + row;
      const int64_t qpos_min = p.start + q0;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < n_kb; ++j) {
        const int Tj = T + j;
        if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
        if (!warp_wait(&s_full[t], Tj & 1, p.err, 0x638)) { ok = false; break; }
        tc_fence_after();
        // raw scores S (fp32); the softmax works on S * scale_log2, and as the
        // scale is positive the row max of the raw scores scales to the max of
        // the scaled ones (rounding is monotonic), so the scaling is folded into
        // one packed FMA with the subtraction of the base: p = 2^(s * scale - m)
        uint32_t rr[kPpN];
#pragma unroll
        for (int c = 0; c < kPpN / 32; ++c) {
          uint32_t(&r32)[32] = *reinterpret_cast<uint32_t(*)[32]>(&rr[c * 32]);
          tmem_ld_32cols(s_col + c * 32, r32);
        }
        tc_wait_ld();
        const int kbase = j * kPpN;
        // masks only where a key can lie past a row's position or past the end
        if (kbase + kPpN - 1 > qpos_min || kbase + kPpN > kv_total) {
          const int lim = (int)min64(kv_total - 1, p.causal ? qpos : kv_total - 1) - kbase;
#pragma unroll
          for (int c = 0; c < kPpN; ++c)
            if (c > lim) rr[c] = __float_as_uint(-INFINITY);
        }
        // four independent max chains (a single chain would serialise 64 maxes)
        float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < kPpN; c += 8)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            mq[q] = max3f(mq[q], __uint_as_float(rr[c + 2 * q]), __uint_as_float(rr[c + 2 * q + 1]));
        const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
        const float m_new = fmaxf(m_used, mx * p.scale_log2);
        const bool move = m_new > m_used + kRescaleLog2;   // -inf + 8 = -inf
        const bool rescale = move && j > 0 && m_used != -INFINITY;
        const float corr = rescale ? ex2_approx(m_used - m_new) : 1.f;
        if (move) {
          l *= ex2_approx(m_used - m_new);  // m_used = -inf: l is 0 and stays 0
          m_used = m_new;
        }
        const float base = (m_used == -INFINITY) ? 0.f : m_used;
        const float nbase = -base;
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
        const float2 nb2 = make_float2(nbase, nbase);
        float2 rsq[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // sum chains
#pragma unroll
        for (int c = 0; c < kPpN / 32; ++c) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 x = ffma2(make_float2(__uint_as_float(rr[c * 32 + 2 * i]),
                                               __uint_as_float(rr[c * 32 + 2 * i + 1])),
                                   sc2, nb2);
            // one key pair in four on the FMA pipe, the rest on MUFU
            const float2 e = (i & 3) == kExpPolyLane
                                 ? exp2_poly2(x)
                                 : make_float2(ex2_approx(x.x), ex2_approx(x.y));
            rsq[i & 1] = fadd2(rsq[i & 1], e);
            w[i] = pack_bf16x2(e.x, e.y);
          }
          tmem_st_16cols(s_col + c * 16, w);  // P: 32 keys per 16 columns
        }
        const float rs = (rsq[0].x + rsq[1].x) + (rsq[0].y + rsq[1].y);
        if (__any_sync(0xffffffffu, rescale)) {
          // O[t] holds tiles 0..j-1 of this item, complete (covered by the
          // commit of S_j(t)): rescale it to the new base before PV_j adds to it
#pragma unroll 1
          for (int c = 0; c < kFD / 32; ++c) {
            uint32_t r32[32];
            tmem_ld_32cols(o_col + c * 32, r32);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r32[i] = __float_as_uint(__uint_as_float(r32[i]) * corr);
            tmem_st_32cols(o_col + c * 32, r32);
          }
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
        l += rs;
      }
      if (!ok) break;
      // the item's last PV of this tile, then O / l to global memory, then O[t]
      // is free for the next item
      if (!warp_wait(&o_final[t], ic & 1, p.err, 0x639)) { ok = false; break; }
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = p.out + itm.b * p.os_b + (int64_t)(itm.h0 + t) * p.os_h +
                           (int64_t)(q0 + row) * p.os_s;
#pragma unroll
      for (int c = 0; c < kFD / 32; ++c) {
        uint32_t r32[32];
        tmem_ld_32cols(o_col + c * 32, r32);
        tc_wait_ld();
        if (row < q_valid) {
#pragma unroll
          for (int d = 0; d < 32; d += 8) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(r32[d]) * inv, __uint_as_float(r32[d + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(r32[d + 2]) * inv, __uint_as_float(r32[d + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(r32[d + 4]) * inv, __uint_as_float(r32[d + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(r32[d + 6]) * inv, __uint_as_float(r32[d + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c * 32 + d) = u;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[t]);
      T += n_kb;
      ++ic;
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kPpTmemCols);
  }
}

}  // namespace
}  // namespace q3

extern "C" int q3_attn_prefill_tc(const void* q, const void* k, const void* v, void* out, int B,
                                  int Hq, int Hkv, int S, int head_dim, int64_t start_pos,
                                  int causal, float scale, int64_t kv_rows_per_head,
                                  const int64_t* o_strides, int variant, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(q && k && v && out && o_strides, "q3_attn_prefill_tc: null pointer");
  Q3_REQUIRE(head_dim == kFD, "q3_attn_prefill_tc: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(variant >= 0 && variant <= 2, "q3_attn_prefill_tc: unknown variant %d", variant);
  Q3_REQUIRE(variant != 2 || (Hkv > 0 && Hq % Hkv == 0 && (Hq / Hkv) % 2 == 0),
             "q3_attn_prefill_tc: variant 2 pairs query heads of one KV head (Hq/Hkv even)");
  Q3_REQUIRE(B > 0 && S > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && start_pos >= 0,
             "q3_attn_prefill_tc: bad shape B=%d S=%d Hq=%d Hkv=%d", B, S, Hq, Hkv);
  Q3_REQUIRE(kv_rows_per_head >= start_pos + S,
             "q3_attn_prefill_tc: the cache holds %lld rows per head, need %lld",
             (long long)kv_rows_per_head, (long long)(start_pos + S));
  Q3_REQUIRE((int64_t)B * Hq * S < (1ll << 31) && (int64_t)B * Hkv * kv_rows_per_head < (1ll << 31),
             "q3_attn_prefill_tc: tensors too large for 32-bit TMA rows");
  Q3_REQUIRE(o_strides[2] % 8 == 0 && o_strides[1] % 8 == 0 && o_strides[0] % 8 == 0,
             "q3_attn_prefill_tc: output rows must stay 16-byte aligned");
  Q3_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(out, 16),
             "q3_attn_prefill_tc: pointers must be 16-byte aligned");
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_2d(&tq, q, (int64_t)B * Hq * S, kFD, kFM, 64);
  if (rc) return rc;
  rc = make_tmap_2d(&tk, k, (int64_t)B * Hkv * kv_rows_per_head, kFD, kFN, 64);
  if (rc) return rc;
  rc = make_tmap_2d(&tv, v, (int64_t)B * Hkv * kv_rows_per_head, kFD, kFN, 64);
  if (rc) return rc;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    Q3_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_tc_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kFSmem));
    Q3_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_tc_mn_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kMnSmem));
    Q3_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_tc_pp_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kPpSmem));
    Q3_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_tc_pp_kernel<true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kPpSmem));
    attr_set[dev] = true;
  }
  FlashParams p{};
  p.out = (__nv_bfloat16*)out;
  p.os_b = o_strides[0]; p.os_h = o_strides[1]; p.os_s = o_strides[2];
  p.Hq = Hq; p.Hkv = Hkv; p.S = S; p.B = B;
  p.q_rows_per_head = S;
  p.kv_rows_per_head = kv_rows_per_head;
  p.start = start_pos;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = device_error_word();
  // V of one stage: two 64-dim boxes 8 KB apart (MN), 8-key groups 1 KB apart (K)
  p.v_mn_stride = (uint32_t)(kKVBytes / 2);
  p.v_k_stride = 1024u;
  if (variant == 2) {
    // K/V as (dim, key, head) maps that end at the last valid key
    rc = make_tmap_3d_rows128(&tk, k, start_pos + S, (int64_t)B * Hkv, kv_rows_per_head * kFD,
                              kPpN);
    if (rc) return rc;
    rc = make_tmap_3d_rows128(&tv, v, start_pos + S, (int64_t)B * Hkv, kv_rows_per_head * kFD,
                              kPpN);
    if (rc) return rc;
    const int64_t items = (int64_t)((S + kFM - 1) / kFM) * (Hq / 2) * B;
    dim3 grid2((unsigned)min64(items, (int64_t)num_sms()));
    return launch_ex(attn_prefill_tc_pp_kernel<false>, grid2, dim3(kPpThreads), kPpSmem,
                     (cudaStream_t)stream, 1, tq, tk, tv, p);
  }
  dim3 grid((S + kFM - 1) / kFM, Hq, B);
  if (variant == 1)
    return launch_ex(attn_prefill_tc_mn_kernel, grid, dim3(kMnThreads), kMnSmem,
                     (cudaStream_t)stream, 1, tq, tk, tv, p);
  return launch_ex(attn_prefill_tc_kernel, grid, dim3(kFThreads), kFSmem, (cudaStream_t)stream,
                   1, tq, tk, tv, p);
}

extern "C" int q3_attn_prefill_tc_paged(const void* q, const void* k_pages, const void* v_pages,
                                        void* out, int B, int Hq, int Hkv, int S, int head_dim,
                                        int64_t start_pos, int causal, float scale,
                                        const int64_t* o_strides, const int32_t* block_table,
                                        int64_t table_stride, int page_tokens, int num_pages,
                                        q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(q && k_pages && v_pages && out && o_strides && block_table,
             "q3_attn_prefill_tc_paged: null pointer");
  Q3_REQUIRE(head_dim == kFD, "q3_attn_prefill_tc_paged: head_dim must be 128 (got %d)",
             head_dim);
  Q3_REQUIRE(B > 0 && S > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && (Hq / Hkv) % 2 == 0 &&
                 start_pos >= 0,
             "q3_attn_prefill_tc_paged: bad shape B=%d S=%d Hq=%d Hkv=%d (Hq/Hkv must be even)",
             B, S, Hq, Hkv);
  Q3_REQUIRE(page_tokens > 0 && page_tokens % kPpN == 0 && num_pages > 0,
             "q3_attn_prefill_tc_paged: page_tokens=%d must be a positive multiple of %d",
             page_tokens, kPpN);
  Q3_REQUIRE(table_stride > 0 && start_pos + S <= table_stride * page_tokens,
             "q3_attn_prefill_tc_paged: positions up to %lld beyond the table width",
             (long long)(start_pos + S - 1));
  Q3_REQUIRE((int64_t)B * Hq * S < (1ll << 31) &&
                 (int64_t)num_pages * Hkv * page_tokens < (1ll << 31),
             "q3_attn_prefill_tc_paged: tensors too large for 32-bit TMA rows");
  Q3_REQUIRE(o_strides[2] % 8 == 0 && o_strides[1] % 8 == 0 && o_strides[0] % 8 == 0,
             "q3_attn_prefill_tc_paged: output rows must stay 16-byte aligned");
  Q3_REQUIRE(aligned(q, 16) && aligned(k_pages, 16) && aligned(v_pages, 16) && aligned(out, 16) &&
                 aligned(block_table, 4),
             "q3_attn_prefill_tc_paged: misaligned pointer");
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_2d(&tq, q, (int64_t)B * Hq * S, kFD, kFM, 64);
  if (rc) return rc;
  rc = make_tmap_2d(&tk, k_pages, (int64_t)num_pages * Hkv * page_tokens, kFD, kPpN, 64);
  if (rc) return rc;
  rc = make_tmap_2d(&tv, v_pages, (int64_t)num_pages * Hkv * page_tokens, kFD, kPpN, 64);
  if (rc) return rc;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    Q3_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_tc_pp_kernel<true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kPpSmem));
    attr_set[dev] = true;
  }
  FlashParams p{};
  p.out = (__nv_bfloat16*)out;
  p.os_b = o_strides[0]; p.os_h = o_strides[1]; p.os_s = o_strides[2];
  p.Hq = Hq; p.Hkv = Hkv; p.S = S; p.B = B;
  p.q_rows_per_head = S;
  p.kv_rows_per_head = 0;
  p.start = start_pos;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = device_error_word();
  p.pages = block_table;
  p.pages_stride = table_stride;
  p.page_tokens = page_tokens;
  p.num_pages = num_pages;
  const int64_t items = (int64_t)((S + kFM - 1) / kFM) * (Hq / 2) * B;
  dim3 grid((unsigned)min64(items, (int64_t)num_sms()));
  return launch_ex(attn_prefill_tc_pp_kernel<true>, grid, dim3(kPpThreads), kPpSmem,
                   (cudaStream_t)stream, 1, tq, tk, tv, p);
}
