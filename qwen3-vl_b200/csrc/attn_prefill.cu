// a6/a7: causal GQA prefill attention (flash-style, online softmax in fp32).
//
// Semantics: the S>1 eager attention of forward_layer (model_fused.py:248-262)
// and prefill_gqa_flash_attention (kernels/prefill_attention.py:28-149):
// out = softmax(q k^T * scale + causal) v, query row s at absolute position
// start_pos + s, GQA head h reading KV head h / (Hq/Hkv).
//
// Tiling: one CTA = 8 warps = 128 query rows of one head; keys stream through
// shared memory in 64-row K/V tiles, double-buffered with cp.async; the tiles
// are XOR-swizzled (16-byte chunk ^ row%8) so ldmatrix is bank-conflict free.
// S = Q K^T and O += P V run on bf16 mma.sync m16n8k16 with fp32 accumulators;
// P is re-packed from the S accumulators into A fragments in registers.  Query
// blocks are launched longest-first, and heads that share a KV head are
// adjacent in the grid so their K/V tiles are served from L2.
#include <math.h>

#include "common.cuh"

namespace q3 {

constexpr int kPBM = 128;  // query rows per CTA
constexpr int kPBN = 64;   // keys per tile
constexpr int kPD = 128;   // head dim
constexpr int kPWarps = 8;
constexpr int kPThreads = kPWarps * 32;
constexpr int kPSmem = (kPBM + 4 * kPBN) * kPD * 2;  // Q + 2x(K,V) = 96 KB

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // src-size 0 => zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// byte offset of 16-byte chunk c of row r in a swizzled [rows][128] bf16 tile
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * 256 + ((c ^ (r & 7)) << 4); }

struct PrefillParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* out;
  int64_t qs_b, qs_h, qs_s;
  int64_t ks_b, ks_h, ks_s;
  int64_t os_b, os_h, os_s;
  int B, Hq, Hkv, S;
  int64_t start;
  int causal;
  float scale_log2;  // scale * log2(e)
  // paged K/V (q3_attn_prefill_paged): k/v are page pools [num_pages, Hkv,
  // page_tokens, 128]; key position t of row b lives in page
  // pages[b * pages_stride + t / page_tokens] at offset t % page_tokens
  const int32_t* pages;
  int64_t pages_stride;
  int page_tokens, num_pages;
  int* err;
};

// Paged caches: first row of the 64-key tile starting at key position k0 (a
// multiple of 64; a tile never straddles pages since page_tokens % 64 == 0).
// A table entry outside the pool is recorded and page 0 read instead.
__device__ __forceinline__ const __nv_bfloat16* paged_tile(const PrefillParams& p,
                                                           const __nv_bfloat16* base, int b,
                                                           int kvh, int64_t k0) {
  int pg = p.pages[(int64_t)b * p.pages_stride + k0 / p.page_tokens];
  if (pg < 0 || pg >= p.num_pages) {
    if (threadIdx.x == 0) report_timeout(p.err, 0x404);
    pg = 0;
  }
  return base + (((int64_t)pg * p.Hkv + kvh) * p.page_tokens + k0 % p.page_tokens) * kPD;
}

// Copy `rows` rows (global row stride `gstride` elements) of a [rows][128]
// tile into swizzled smem; rows >= valid are zero-filled.
__device__ __forceinline__ void load_tile(uint32_t smem, const __nv_bfloat16* g, int64_t gstride,
                                          int rows, int valid) {
  for (int i = threadIdx.x; i < rows * 16; i += kPThreads) {
    const int r = i >> 4, c = i & 15;
    const bool ok = r < valid;
    const __nv_bfloat16* src = ok ? g + r * gstride + c * 8 : g;
    cp_async_16(smem + swz(r, c), src, ok);
  }
}

template <bool PAGED>
__global__ void __launch_bounds__(kPThreads, 1) attn_prefill_kernel(PrefillParams p) {
  pdl_wait();
  pdl_launch();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t sQ = smem_u32(smem_raw);
  const uint32_t sK0 = sQ + kPBM * kPD * 2;
  const uint32_t sV0 = sK0 + 2 * kPBN * kPD * 2;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;

  const int qb = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.Hq / p.Hkv);
  const int q0 = qb * kPBM;
  const int q_valid = min(kPBM, p.S - q0);
  const int64_t kv_total = p.start + p.S;
  const int64_t kv_need = p.causal ? min64(p.start + q0 + kPBM, kv_total) : kv_total;
  const int n_kb = (int)((kv_need + kPBN - 1) / kPBN);

  const __nv_bfloat16* qg = p.q + b * p.qs_b + h * p.qs_h + (int64_t)q0 * p.qs_s;
  const __nv_bfloat16* kg = p.k + b * p.ks_b + kvh * p.ks_h;
  const __nv_bfloat16* vg = p.v + b * p.ks_b + kvh * p.ks_h;

  load_tile(sQ, qg, p.qs_s, kPBM, q_valid);
  {
    const int valid = (int)min64(kPBN, kv_total);
    if constexpr (PAGED) {
      load_tile(sK0, paged_tile(p, p.k, b, kvh, 0), kPD, kPBN, valid);
      load_tile(sV0, paged_tile(p, p.v, b, kvh, 0), kPD, kPBN, valid);
    } else {
      load_tile(sK0, kg, p.ks_s, kPBN, valid);
      load_tile(sV0, vg, p.ks_s, kPBN, valid);
    }
  }
  cp_async_commit();

  uint32_t qf[8][4];  // Q fragments: 8 k-steps of 16 dims
  float o[16][4];     // O accumulators: 16 dim tiles of 8
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  // absolute positions of this lane's two query rows
  const int64_t pos0 = p.start + q0 + warp * 16 + g8;
  const int64_t pos1 = pos0 + 8;

  for (int kb = 0; kb < n_kb; ++kb) {
    const int st = kb & 1;
    if (kb + 1 < n_kb) {
      const int64_t k0 = (int64_t)(kb + 1) * kPBN;
      const int valid = (int)min64(kPBN, kv_total - k0);
      const uint32_t sKn = sK0 + (st ^ 1) * kPBN * kPD * 2;
      const uint32_t sVn = sV0 + (st ^ 1) * kPBN * kPD * 2;
      if constexpr (PAGED) {
        load_tile(sKn, paged_tile(p, p.k, b, kvh, k0), kPD, kPBN, valid);
        load_tile(sVn, paged_tile(p, p.v, b, kvh, k0), kPD, kPBN, valid);
      } else {
        load_tile(sKn, kg + k0 * p.ks_s, p.ks_s, kPBN, valid);
        load_tile(sVn, vg + k0 * p.ks_s, p.ks_s, kPBN, valid);
      }
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int r = warp * 16 + (lane & 15);
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(qf[ks], sQ + swz(r, c));
      }
    }
    const uint32_t sK = sK0 + st * kPBN * kPD * 2;
    const uint32_t sV = sV0 + st * kPBN * kPD * 2;

    // ---- S = Q K^T for 16 rows x 64 keys ----
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {  // pairs of key tiles
        uint32_t kf[4];
        const int r = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(kf, sK + swz(r, c));
        mma_16816(s[2 * jp], qf[ks], kf[0], kf[1]);
        mma_16816(s[2 * jp + 1], qf[ks], kf[2], kf[3]);
      }
    }
    // ---- scale + mask ----
    const int64_t kbase = (int64_t)kb * kPBN;
    const bool need_mask =
        (p.causal && kbase + kPBN - 1 > p.start + q0 + warp * 16) || (kbase + kPBN > kv_total);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[j][e] * p.scale_log2;
        if (need_mask) {
          const int64_t key = kbase + j * 8 + 2 * t4 + (e & 1);
          const int64_t qp = (e < 2) ? pos0 : pos1;
          if (key >= kv_total || (p.causal && key > qp)) x = -INFINITY;
        }
        s[j][e] = x;
      }
    }
    // ---- online softmax (rows g8 and g8+8) ----
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx[0] = fmaxf(mx[0], fmaxf(s[j][0], s[j][1]));
      mx[1] = fmaxf(mx[1], fmaxf(s[j][2], s[j][3]));
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float corr[2], base_m[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      base_m[r] = (mx[r] == -INFINITY) ? 0.f : mx[r];
      corr[r] = exp2f(m_r[r] - base_m[r]);  // m_r=-inf -> 0
      m_r[r] = mx[r];
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pf[4][4];  // P as A fragments: 4 k-steps of 16 keys
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = exp2f(s[j][0] - base_m[0]);
      const float p1 = exp2f(s[j][1] - base_m[0]);
      const float p2 = exp2f(s[j][2] - base_m[1]);
      const float p3 = exp2f(s[j][3] - base_m[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int ks = j >> 1, hi = j & 1;
      pf[ks][hi * 2 + 0] = pack_bf16x2(p0, p1);
      pf[ks][hi * 2 + 1] = pack_bf16x2(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_r[r] = l_r[r] * corr[r] + rs[r];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= corr[0]; o[i][1] *= corr[0];
      o[i][2] *= corr[1]; o[i][3] *= corr[1];
    }
    // ---- O += P V ----
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int ip = 0; ip < 8; ++ip) {  // pairs of dim tiles
        uint32_t vf[4];
        const int r = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = ip * 2 + (lane >> 4);
        ldsm_x4_t(vf, sV + swz(r, c));
        mma_16816(o[2 * ip], pf[ks], vf[0], vf[1]);
        mma_16816(o[2 * ip + 1], pf[ks], vf[2], vf[3]);
      }
    }
    __syncthreads();  // stage st is overwritten by the next prefetch
  }

  // ---- finalize: O / l, bf16 store ----
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
  const float inv0 = l_r[0] > 0.f ? 1.f / l_r[0] : 0.f;
  const float inv1 = l_r[1] > 0.f ? 1.f / l_r[1] : 0.f;
  const int row0 = warp * 16 + g8;
  __nv_bfloat16* ob = p.out + b * p.os_b + h * p.os_h;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int d = i * 8 + 2 * t4;
    if (row0 < q_valid)
      *reinterpret_cast<uint32_t*>(ob + (int64_t)(q0 + row0) * p.os_s + d) =
          pack_bf16x2(o[i][0] * inv0, o[i][1] * inv0);
    if (row0 + 8 < q_valid)
      *reinterpret_cast<uint32_t*>(ob + (int64_t)(q0 + row0 + 8) * p.os_s + d) =
          pack_bf16x2(o[i][2] * inv1, o[i][3] * inv1);
  }
}

}  // namespace q3

extern "C" int q3_attn_prefill(const void* q, const void* k, const void* v, void* out, int B,
                               int Hq, int Hkv, int S, int head_dim, int64_t start_pos,
                               int causal, float scale, const int64_t* q_strides,
                               const int64_t* kv_strides, const int64_t* o_strides,
                               q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(q && k && v && out && q_strides && kv_strides && o_strides,
             "q3_attn_prefill: null pointer");
  Q3_REQUIRE(head_dim == kPD, "q3_attn_prefill: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(B > 0 && S > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && start_pos >= 0,
             "q3_attn_prefill: bad shape B=%d S=%d Hq=%d Hkv=%d", B, S, Hq, Hkv);
  for (int i = 0; i < 3; ++i)
    Q3_REQUIRE(q_strides[i] % 8 == 0 && kv_strides[i] % 8 == 0 && o_strides[i] % 2 == 0,
               "q3_attn_prefill: strides must keep 16-byte rows aligned");
  Q3_REQUIRE(aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(out, 4),
             "q3_attn_prefill: misaligned pointer");
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    Q3_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem));
    attr_set[dev] = true;
  }
  PrefillParams p;
  p.q = (const __nv_bfloat16*)q;
  p.k = (const __nv_bfloat16*)k;
  p.v = (const __nv_bfloat16*)v;
  p.out = (__nv_bfloat16*)out;
  p.qs_b = q_strides[0]; p.qs_h = q_strides[1]; p.qs_s = q_strides[2];
  p.ks_b = kv_strides[0]; p.ks_h = kv_strides[1]; p.ks_s = kv_strides[2];
  p.os_b = o_strides[0]; p.os_h = o_strides[1]; p.os_s = o_strides[2];
  p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.S = S;
  p.start = start_pos;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  dim3 grid((S + kPBM - 1) / kPBM, Hq, B);
  return launch_ex(attn_prefill_kernel<false>, grid, dim3(kPThreads), kPSmem,
                   (cudaStream_t)stream, 1, p);
}

extern "C" int q3_attn_prefill_paged(const void* q, const void* k_pages, const void* v_pages,
                                     void* out, int B, int Hq, int Hkv, int S, int head_dim,
                                     int64_t start_pos, int causal, float scale,
                                     const int64_t* q_strides, const int64_t* o_strides,
                                     const int32_t* block_table, int64_t table_stride,
                                     int page_tokens, int num_pages, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(q && k_pages && v_pages && out && q_strides && o_strides && block_table,
             "q3_attn_prefill_paged: null pointer");
  Q3_REQUIRE(head_dim == kPD, "q3_attn_prefill_paged: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(B > 0 && S > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && start_pos >= 0,
             "q3_attn_prefill_paged: bad shape B=%d S=%d Hq=%d Hkv=%d", B, S, Hq, Hkv);
  Q3_REQUIRE(page_tokens > 0 && page_tokens % kPBN == 0 && num_pages > 0,
             "q3_attn_prefill_paged: page_tokens=%d must be a positive multiple of %d",
             page_tokens, kPBN);
  Q3_REQUIRE(table_stride > 0 && start_pos + S <= table_stride * page_tokens,
             "q3_attn_prefill_paged: positions up to %lld beyond the table width",
             (long long)(start_pos + S - 1));
  for (int i = 0; i < 3; ++i)
    Q3_REQUIRE(q_strides[i] % 8 == 0 && o_strides[i] % 2 == 0,
               "q3_attn_prefill_paged: strides must keep 16-byte rows aligned");
  Q3_REQUIRE(aligned(q, 16) && aligned(k_pages, 16) && aligned(v_pages, 16) && aligned(out, 4) &&
                 aligned(block_table, 4),
             "q3_attn_prefill_paged: misaligned pointer");
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    Q3_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_kernel<true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem));
    attr_set[dev] = true;
  }
  PrefillParams p{};
  p.q = (const __nv_bfloat16*)q;
  p.k = (const __nv_bfloat16*)k_pages;
  p.v = (const __nv_bfloat16*)v_pages;
  p.out = (__nv_bfloat16*)out;
  p.qs_b = q_strides[0]; p.qs_h = q_strides[1]; p.qs_s = q_strides[2];
  p.os_b = o_strides[0]; p.os_h = o_strides[1]; p.os_s = o_strides[2];
  p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.S = S;
  p.start = start_pos;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.pages = block_table;
  p.pages_stride = table_stride;
  p.page_tokens = page_tokens;
  p.num_pages = num_pages;
  p.err = device_error_word();
  dim3 grid((S + kPBM - 1) / kPBM, Hq, B);
  return launch_ex(attn_prefill_kernel<true>, grid, dim3(kPThreads), kPSmem,
                   (cudaStream_t)stream, 1, p);
}
