// a3/a10/a11/a13: bf16 projections C = A W^T with fused epilogues.
//
// Reference: the compiled matmuls h @ Wqkv (model_fused.py:103), x @ Wo (:141),
// h @ Wgate_up -> silu(gate)*up (:165-169), h @ Wdown (:172), lm_head (:183),
// with the residual add of forward_layer (:269, :275) folded in.  Weights are
// stored [N, K] (K-major).  Epilogues reproduce the reference's bf16 rounding
// points: every torch op on bf16 tensors rounds its result to bf16.
//
// Dispatch: M <= 16 (decode) goes to the TMA-ring GEMV of gemv.cu (tensor
// cores idle at this M; the design goal is bytes in flight).  M > 16
// (prefill) runs the persistent warp-specialised tcgen05 kernel below: warp 0
// issues TMA loads (128-byte swizzle, no multicast) into a 4-6 stage smem
// ring, warp 1 issues tcgen05.mma (M=128, N=BN, K=16 per instruction) into a
// double-buffered TMEM accumulator, warps 2-5 drain TMEM with tcgen05.ld and
// run the epilogue while the next tile accumulates.  Epilogues: plain,
// residual add, SwiGLU on interleaved gate/up rows, and (q3_gemm_qkv_rope) the
// per-head QK-RMSNorm + RoPE + KV-cache write of the QKV projection.
#include <math.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace q3 {

// ===========================================================================
// ===========================================================================
// tcgen05 kernel (M > 16)
// ===========================================================================
constexpr int kBM = 128;
constexpr int kBK = 64;  // one 128-byte swizzle row of bf16
constexpr int kTcThreads = 192;

template <int BN>
struct TcCfg {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kSmem = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int kTmemCols = 2 * BN;
};

// Internal epilogue id of the fused QKV projection: per-head QK-RMSNorm,
// rotate-half RoPE and the KV-cache write (AttentionBlock.forward after the
// matmul, model_fused.py:107-129, and the cache write, :244-246).
constexpr int kEpiQkvRope = 16;
// The same with the K/V rows written into a page pool through a block table.
constexpr int kEpiQkvRopePaged = 17;

// Internal epilogue id of the prefill all-reduce's first half: the bf16
// partial tile goes over NVLink into the receive stripe of the rank that owns
// its rows, and each epilogue warp then publishes a flag for its 32 rows.
constexpr int kEpiPushStripe = 18;
constexpr int kPushMaxRanks = 8;

// Bias epilogues of nn.Linear (the vision tower's linears): v = bf16(acc + b)
// -- one rounding, as a linear with bias computes -- then Q3_EPI_BIAS_GELU_TANH
// bf16(gelu_tanh(v)), Q3_EPI_BIAS_GELU bf16(gelu_erf(v)), or
// Q3_EPI_BIAS_RESIDUAL bf16(R + v).
__device__ __forceinline__ bool epi_has_bias(int e) {
  return e == Q3_EPI_BIAS || e == Q3_EPI_BIAS_GELU_TANH || e == Q3_EPI_BIAS_GELU ||
         e == Q3_EPI_BIAS_RESIDUAL;
}
// torch's tanh-approximated GELU: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
__device__ __forceinline__ float gelu_tanh(float x) {
  const float kBeta = 0.7978845608028654f, kKappa = 0.044715f;
  const float inner = kBeta * (x + kKappa * x * x * x);
  return 0.5f * x * (1.0f + tanhf(inner));
}
// exact GELU: 0.5 x (1 + erf(x / sqrt(2)))
__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f));
}
template <int EPI>
__device__ __forceinline__ float bias_epilogue(float acc, float bias, float res) {
  float v = rbf(acc + bias);
  if constexpr (EPI == Q3_EPI_BIAS_GELU_TANH) v = rbf(gelu_tanh(v));
  if constexpr (EPI == Q3_EPI_BIAS_GELU) v = rbf(gelu_erf(v));
  if constexpr (EPI == Q3_EPI_BIAS_RESIDUAL) v = rbf(res + v);
  return v;
}

struct TcQkv {
  const __nv_bfloat16* q_norm;  // [128]
  const __nv_bfloat16* k_norm;  // [128]
  const void* cos;              // [rows, 64] bf16 or f32
  const void* sin;
  int cs_f32, cs_use_pos;
  int64_t cs_offset, cs_stride_b;
  __nv_bfloat16* q_out;    // [B, Hq, S, 128]
  __nv_bfloat16* k_cache;  // [B, Hkv, max_seq, 128], rows start_pos .. start_pos + S - 1
  __nv_bfloat16* v_cache;
  int S, Hq, Hkv;
  int64_t start_pos, max_seq;
  float eps;
  // kEpiQkvRopePaged: k_cache / v_cache are page pools [num_pages, Hkv,
  // page_tokens, 128]; position t of sequence b lives in page
  // pages[b * pages_stride + t / page_tokens] at offset t % page_tokens
  const int32_t* pages;
  int64_t pages_stride;
  int page_tokens, num_pages;
};

// Element offset of cache row (b, kv head hkv, position pos), or -1 when a
// paged table entry lies outside the pool (the row is then not written).
template <int EPI>
__device__ __forceinline__ int64_t kv_row(const TcQkv& q, int b, int hkv, int64_t pos) {
  if constexpr (EPI == kEpiQkvRopePaged) {
    const int pg = q.pages[(int64_t)b * q.pages_stride + pos / q.page_tokens];
    if (pg < 0 || pg >= q.num_pages) return -1;
    return (((int64_t)pg * q.Hkv + hkv) * q.page_tokens + pos % q.page_tokens) * 128;
  } else {
    return (((int64_t)b * q.Hkv + hkv) * q.max_seq + pos) * 128;
  }
}

// kEpiPushStripe: rows [o * stripe, (o + 1) * stripe) belong to rank o; this
// rank's partial of row r lands at recv[o] + (r - o * stripe) * N and the
// flag of (m-tile mt, n-tile nt, epilogue warp w) at flags[o] + (mt * n_tiles +
// nt) * 4 + w, set to `call`
// once the warp's rows are stored (the owner's receive region and flag array
// for this source rank and this call's parity).
struct TcPush {
  __nv_bfloat16* recv[kPushMaxRanks];
  uint32_t* flags[kPushMaxRanks];
  int stripe;
  uint32_t call;
};

struct TcParams {
  __nv_bfloat16* C;
  const __nv_bfloat16* R;
  const __nv_bfloat16* bias;  // [N], bias epilogues only
  int M, N, K, ldc;
  int m_tiles, n_tiles;
  int group_m;  // 0: tiles in column order (M fastest); g > 0: grouped raster, g M-tiles per group
  int* err;
  TcQkv qkv;  // kEpiQkvRope only
  TcPush push;  // kEpiPushStripe only
};

// 8 consecutive RoPE table entries (bf16 tables as RotaryEmbedding builds them;
// f32 M-RoPE rows are rounded to bf16 as the reference casts them to x.dtype)
__device__ __forceinline__ void load8_cs(const TcQkv& q, const void* tab, int64_t row, int j,
                                         float (&v)[8]) {
  if (q.cs_f32) {
    const float4* f = reinterpret_cast<const float4*>(static_cast<const float*>(tab) + row * 64 + j);
    const float4 a = f[0], b = f[1];
    v[0] = rbf(a.x); v[1] = rbf(a.y); v[2] = rbf(a.z); v[3] = rbf(a.w);
    v[4] = rbf(b.x); v[5] = rbf(b.y); v[6] = rbf(b.z); v[7] = rbf(b.w);
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(
        static_cast<const __nv_bfloat16*>(tab) + row * 64 + j);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}
__device__ __forceinline__ void unpack8(uint4 u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Output tile of linear tile index `tile`.  group_m == 0: column order (M
// fastest).  group_m = g: tiles run over g M-tiles x every N-tile per group,
// so one wave of CTAs shares fewer A rows and B columns in L2.  Both orders
// are bijections of [0, m_tiles * n_tiles).
__device__ __forceinline__ void tile_coords(const TcParams& p, int tile, int& mt, int& nt) {
  if (p.group_m <= 0) {
    mt = tile % p.m_tiles;
    nt = tile / p.m_tiles;
    return;
  }
  const int per_group = p.group_m * p.n_tiles;
  const int first_m = (tile / per_group) * p.group_m;
  const int gm = min(p.m_tiles - first_m, p.group_m);
  const int in = tile % per_group;
  mt = first_m + in % gm;
  nt = in / gm;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   TcParams p) {
  pdl_wait();
  pdl_launch();
  using Cfg = TcCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.m_tiles * p.n_tiles;
  const int nk = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------- TMA producer -------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        int mt, nt;
        tile_coords(p, tile, mt, nt);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, 0x101)) { *abort_flag = 1; break; }
          uint8_t* sa = smem + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kABytes;
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          tma_load_2d(sa, &tmA, &full[stage], kb * kBK, mt * kBM, kCacheEvictNormal);
          tma_load_2d(sb, &tmW, &full[stage], kb * kBK, nt * BN, kCacheEvictNormal);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------- MMA issuer ---------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err, 0x102)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, 0x103)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::kStageBytes);
          const uint32_t sb = sa + Cfg::kABytes;
          const uint64_t da = umma_desc_k_sw128(sa);
          const uint64_t db = umma_desc_k_sw128(sb);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // advance 16 bf16 = 32 bytes (>>4 = 2) inside the swizzle row
            tc_mma_bf16(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
          }
          tc_commit(&empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) { *abort_flag = 1; break; }
        tc_commit(&tfull[acc]);
      }
    }
  } else {
    // ------------------------- epilogue (warps 2..5) -----------------------
    const int sub = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = sub * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int mt, nt;
      tile_coords(p, tile, mt, nt);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      bool got;
      if constexpr (EPI == kEpiPushStripe)  // the warp stays converged for its flag
        got = __all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, p.err, 0x104));
      else
        got = mbar_wait(&tfull[acc], acc_phase, p.err, 0x104);
      if (!got) { *abort_flag = 1; break; }
      tc_fence_after();
      const int row = mt * kBM + row_in_tile;
      const uint32_t t_row = tmem_base + acc * BN + ((uint32_t)(sub * 32) << 16);
      if constexpr (EPI == kEpiQkvRope || EPI == kEpiQkvRopePaged) {
        // The tile's columns are whole heads (BN = 2 x 128; rows of W are
        // [q heads | k heads | v heads] x 128); this thread owns token `row`.
        const TcQkv& q = p.qkv;
        const int b = row / q.S, s = row - (row / q.S) * q.S;
        const int64_t pos = q.start_pos + s;  // cache row of this token
        // RoPE row, as q3_qkv_norm_rope: base position + offset + b * stride + s
        const int64_t crow =
            q.cs_use_pos * q.start_pos + q.cs_offset + (int64_t)b * q.cs_stride_b + s;
#pragma unroll 1
        for (int hh = 0; hh < BN / 128; ++hh) {
          const int head = nt * (BN / 128) + hh;
          if (head * 128 >= p.N) break;
          const uint32_t t_head = t_row + hh * 128;
          if (head >= q.Hq + q.Hkv) {
            // value head: the bf16 projection output goes to the cache
            const int hv = head - q.Hq - q.Hkv;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              uint32_t r[32];
              tmem_ld_32cols(t_head + c * 32, r);
              tc_wait_ld();
              int64_t vrow = 0;
              if constexpr (EPI == kEpiQkvRopePaged) {
                vrow = row < p.M ? kv_row<EPI>(q, b, hv, pos) : 0;
                if (vrow < 0 && c == 0) report_timeout(p.err, 0x405);
              }
              if (row < p.M && vrow >= 0) {
                uint4* dst = reinterpret_cast<uint4*>(
                    EPI == kEpiQkvRopePaged
                        ? q.v_cache + vrow + c * 32
                        : q.v_cache + (((int64_t)b * q.Hkv + hv) * q.max_seq + pos) * 128 + c * 32);
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                  uint32_t o[4];
#pragma unroll
                  for (int i = 0; i < 4; ++i)
                    o[i] = pack_bf16x2(__uint_as_float(r[v * 8 + 2 * i]),
                                       __uint_as_float(r[v * 8 + 2 * i + 1]));
                  dst[v] = make_uint4(o[0], o[1], o[2], o[3]);
                }
              }
            }
            continue;
          }
          // q or k head: RMSNorm over the head's 128 bf16 values, then RoPE
          float ss = 0.f;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld_32cols(t_head + c * 32, r);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float v = rbf(__uint_as_float(r[i]));
              ss = fmaf(v, v, ss);
            }
          }
          const float rr = 1.0f / sqrtf(ss * (1.0f / 128) + q.eps);  // IEEE, as torch.rsqrt on CPU
          const bool is_q = head < q.Hq;
          const __nv_bfloat16* nw = is_q ? q.q_norm : q.k_norm;
          __nv_bfloat16* dst_row;
          if constexpr (EPI == kEpiQkvRopePaged) {
            const int64_t krow = (is_q || row >= p.M) ? 0 : kv_row<EPI>(q, b, head - q.Hq, pos);
            if (krow < 0) report_timeout(p.err, 0x405);
            dst_row = is_q ? q.q_out + (((int64_t)b * q.Hq + head) * q.S + s) * 128
                           : (krow >= 0 ? q.k_cache + krow : nullptr);
          } else {
            dst_row =
                is_q ? q.q_out + (((int64_t)b * q.Hq + head) * q.S + s) * 128
                     : q.k_cache + (((int64_t)b * q.Hkv + (head - q.Hq)) * q.max_seq + pos) * 128;
          }
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            // dims c*32 .. +31 (lo) pair with dims 64 + c*32 .. +31 (hi)
            uint32_t lo[32], hi[32];
            tmem_ld_32cols(t_head + c * 32, lo);
            tmem_ld_32cols(t_head + 64 + c * 32, hi);
            tc_wait_ld();
            if (row >= p.M || (EPI == kEpiQkvRopePaged && dst_row == nullptr)) continue;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const int j = c * 32 + g * 8;  // table column of both halves
              float co[8], si[8], wl[8], wh[8];
              load8_cs(q, q.cos, crow, j, co);
              load8_cs(q, q.sin, crow, j, si);
              unpack8(*reinterpret_cast<const uint4*>(nw + j), wl);
              unpack8(*reinterpret_cast<const uint4*>(nw + 64 + j), wh);
              uint32_t olo[4], ohi[4];
#pragma unroll
              for (int i = 0; i < 8; i += 2) {
                float a[2], bb[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const float nl = rbf(rbf(rbf(__uint_as_float(lo[g * 8 + i + e])) * rr) * wl[i + e]);
                  const float nh = rbf(rbf(rbf(__uint_as_float(hi[g * 8 + i + e])) * rr) * wh[i + e]);
                  a[e] = rbf(nl * co[i + e]) + rbf(-nh * si[i + e]);
                  bb[e] = rbf(nh * co[i + e]) + rbf(nl * si[i + e]);
                }
                olo[i / 2] = pack_bf16x2(a[0], a[1]);
                ohi[i / 2] = pack_bf16x2(bb[0], bb[1]);
              }
              *reinterpret_cast<uint4*>(dst_row + j) = make_uint4(olo[0], olo[1], olo[2], olo[3]);
              *reinterpret_cast<uint4*>(dst_row + 64 + j) =
                  make_uint4(ohi[0], ohi[1], ohi[2], ohi[3]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        continue;
      }
      if constexpr (EPI == kEpiPushStripe) {
        const TcPush& q = p.push;
        const int owner = (mt * kBM) / q.stripe;
        __nv_bfloat16* dst_row =
            q.recv[owner] + (int64_t)(row - owner * q.stripe) * p.N + nt * BN;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32cols(t_row + c * 32, r);
          tc_wait_ld();
          if (row < p.M && nt * BN + c * 32 + 32 <= p.N) {
            uint4* dst = reinterpret_cast<uint4*>(dst_row + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              dst[v] = make_uint4(
                  pack_bf16x2(__uint_as_float(r[8 * v]), __uint_as_float(r[8 * v + 1])),
                  pack_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3])),
                  pack_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5])),
                  pack_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7])));
          }
        }
        // the warp's 32 rows are out: publish them to the owner
        __syncwarp();
        if (lane == 0) {
          __threadfence_system();
          // keyed by (m-tile, n-tile), whatever order the tiles ran in
          st_release_sys(q.flags[owner] + ((int64_t)mt * p.n_tiles + nt) * 4 + sub, q.call);
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32cols(t_row + c * 32, r);
        tc_wait_ld();
        if (row < p.M) {
          if (EPI == Q3_EPI_SWIGLU) {
            // 32 columns = [gate 8 | up 8 | gate 8 | up 8] -> 16 outputs
            const int f0 = (nt * BN + c * 32) / 2;
            uint32_t o[8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
#pragma unroll
              for (int i = 0; i < 8; i += 2) {
                const float g0 = rbf(__uint_as_float(r[h * 16 + i]));
                const float g1 = rbf(__uint_as_float(r[h * 16 + i + 1]));
                const float u0 = rbf(__uint_as_float(r[h * 16 + 8 + i]));
                const float u1 = rbf(__uint_as_float(r[h * 16 + 8 + i + 1]));
                o[h * 4 + i / 2] = pack_bf16x2(silu_ref(g0) * u0, silu_ref(g1) * u1);
              }
            }
            // N is a multiple of 16, so the last chunk may hold one [gate 8 | up 8]
            // pair (8 outputs) instead of two
            uint4* dst = reinterpret_cast<uint4*>(p.C + (int64_t)row * p.ldc + f0);
            if (f0 + 8 <= p.ldc) dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
            if (f0 + 16 <= p.ldc) dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
          } else if constexpr (EPI == Q3_EPI_BIAS || EPI == Q3_EPI_BIAS_GELU_TANH ||
                               EPI == Q3_EPI_BIAS_GELU || EPI == Q3_EPI_BIAS_RESIDUAL) {
            const int col0 = nt * BN + c * 32;
            __nv_bfloat16* dst = p.C + (int64_t)row * p.ldc + col0;
            const __nv_bfloat16* rrow = p.R + (int64_t)row * p.ldc + col0;
            if (col0 + 32 <= p.N) {
              uint32_t o[16];
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const uint4 bv = *reinterpret_cast<const uint4*>(p.bias + col0 + v * 8);
                const uint4 rv = EPI == Q3_EPI_BIAS_RESIDUAL
                                     ? *reinterpret_cast<const uint4*>(rrow + v * 8)
                                     : make_uint4(0, 0, 0, 0);
                const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
                const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const float2 bb = unpack_bf16x2(bw[i]);
                  const float2 res = unpack_bf16x2(rw[i]);
                  o[v * 4 + i] = pack_bf16x2(
                      bias_epilogue<EPI>(__uint_as_float(r[v * 8 + 2 * i]), bb.x, res.x),
                      bias_epilogue<EPI>(__uint_as_float(r[v * 8 + 2 * i + 1]), bb.y, res.y));
                }
              }
              uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
              for (int v = 0; v < 4; ++v)
                d4[v] = make_uint4(o[v * 4], o[v * 4 + 1], o[v * 4 + 2], o[v * 4 + 3]);
            } else {
              for (int i = 0; i < 32 && col0 + i < p.N; ++i) {
                const float res = EPI == Q3_EPI_BIAS_RESIDUAL ? bf2f(rrow[i]) : 0.f;
                dst[i] = f2bf(bias_epilogue<EPI>(__uint_as_float(r[i]), bf2f(p.bias[col0 + i]), res));
              }
            }
          } else {
            const int col0 = nt * BN + c * 32;
            uint32_t o[16];
            if (EPI == Q3_EPI_RESIDUAL) {
              const uint4* rs = reinterpret_cast<const uint4*>(p.R + (int64_t)row * p.ldc + col0);
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const uint4 rv = (col0 + 32 <= p.N) ? rs[v] : make_uint4(0, 0, 0, 0);
                const uint32_t rr[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const float2 res = unpack_bf16x2(rr[i]);
                  const float a0 = rbf(__uint_as_float(r[v * 8 + 2 * i]));
                  const float a1 = rbf(__uint_as_float(r[v * 8 + 2 * i + 1]));
                  o[v * 4 + i] = pack_bf16x2(res.x + a0, res.y + a1);
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                o[i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
            }
            if (col0 + 32 <= p.N) {
              uint4* dst = reinterpret_cast<uint4*>(p.C + (int64_t)row * p.ldc + col0);
#pragma unroll
              for (int v = 0; v < 4; ++v)
                dst[v] = make_uint4(o[v * 4], o[v * 4 + 1], o[v * 4 + 2], o[v * 4 + 3]);
            } else {
              __nv_bfloat16* dst = p.C + (int64_t)row * p.ldc;
              for (int i = 0; i < 32 && col0 + i < p.N; ++i) {
                float val = __uint_as_float(r[i]);
                if (EPI == Q3_EPI_RESIDUAL)
                  val = bf2f(p.R[(int64_t)row * p.ldc + col0 + i]) + rbf(val);
                dst[col0 + i] = f2bf(val);
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side: launch
// ---------------------------------------------------------------------------
// Tile raster of the tcgen05 GEMM: groups of 32 M-tiles swept across every
// N-tile (measured on B200 for 8192 x 6144 x 4096: 1333 TFLOP/s against 1250
// in column order, whose waves re-read A from DRAM).  Q3VL_GEMM_GROUP_M=g
// sets another group size; 0 selects the column order.
static int gemm_group_m() {
  static const int g = [] {
    const char* e = getenv("Q3VL_GEMM_GROUP_M");
    const int v = e ? atoi(e) : 32;
    return v > 0 ? v : 0;
  }();
  return g;
}

template <int BN, int EPI>
static int launch_tc(const void* A, const void* W, void* C, const void* R, int M, int N, int K,
                     cudaStream_t s, const TcQkv* qkv = nullptr, const void* bias = nullptr,
                     const TcPush* push = nullptr) {
  using Cfg = TcCfg<BN>;
  CUtensorMap ta, tw;
  int rc = make_tmap_2d(&ta, A, M, K, kBM, kBK);
  if (rc) return rc;
  rc = cached_tmap_2d(&tw, W, N, K, BN, kBK);
  if (rc) return rc;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    Q3_CUDA_CHECK(cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem));
    attr_set[dev] = true;
  }
  TcParams p;
  p.C = (__nv_bfloat16*)C;
  p.R = (const __nv_bfloat16*)R;
  p.bias = (const __nv_bfloat16*)bias;
  p.M = M; p.N = N; p.K = K;
  p.ldc = EPI == Q3_EPI_SWIGLU ? N / 2 : N;
  p.m_tiles = (M + kBM - 1) / kBM;
  p.n_tiles = (N + BN - 1) / BN;
  p.group_m = gemm_group_m();
  p.err = device_error_word();
  p.qkv = qkv ? *qkv : TcQkv{};
  p.push = push ? *push : TcPush{};
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  return launch_ex(gemm_tc_kernel<BN, EPI>, dim3(grid), dim3(kTcThreads), Cfg::kSmem, s, 1, ta,
                   tw, p);
}

// The partial-product GEMM of the prefill all-reduce (comm_prefill.cu): bf16
// tiles pushed into the owners' receive stripes with per-warp flags.
int launch_gemm_push(const void* A, const void* W, int M, int N, int K,
                     __nv_bfloat16* const* recv, uint32_t* const* flags, int world, int stripe,
                     uint32_t call, cudaStream_t s) {
  TcPush push{};
  for (int r = 0; r < world && r < kPushMaxRanks; ++r) {
    push.recv[r] = recv[r];
    push.flags[r] = flags[r];
  }
  push.stripe = stripe;
  push.call = call;
  return launch_tc<256, kEpiPushStripe>(A, W, nullptr, nullptr, M, N, K, s, nullptr, nullptr,
                                        &push);
}

}  // namespace q3

extern "C" int q3_gemm(const void* A, const void* W, void* C, int64_t M, int64_t N, int64_t K,
                       int epilogue, const void* aux, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(A && W && C, "q3_gemm: null pointer");
  Q3_REQUIRE(M >= 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31),
             "q3_gemm: bad shape M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  Q3_REQUIRE(K % 32 == 0, "q3_gemm: K=%lld must be a multiple of 32", (long long)K);
  Q3_REQUIRE(N % 16 == 0, "q3_gemm: N=%lld must be a multiple of 16", (long long)N);
  Q3_REQUIRE(epilogue == Q3_EPI_NONE || epilogue == Q3_EPI_RESIDUAL || epilogue == Q3_EPI_SWIGLU,
             "q3_gemm: unknown epilogue %d", epilogue);
  Q3_REQUIRE(epilogue != Q3_EPI_RESIDUAL || aux, "q3_gemm: residual epilogue needs aux");
  Q3_REQUIRE(aligned(A, 16) && aligned(W, 16) && aligned(C, 16) && (!aux || aligned(aux, 16)),
             "q3_gemm: pointers must be 16-byte aligned");
  if (M == 0) return Q3_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int m = (int)M, n = (int)N, k = (int)K;
  if (M <= 16) return launch_gemv(A, W, C, aux, m, n, k, epilogue, s);
  switch (epilogue) {
    case Q3_EPI_NONE: return launch_tc<256, Q3_EPI_NONE>(A, W, C, aux, m, n, k, s);
    case Q3_EPI_RESIDUAL: return launch_tc<256, Q3_EPI_RESIDUAL>(A, W, C, aux, m, n, k, s);
    default: return launch_tc<256, Q3_EPI_SWIGLU>(A, W, C, aux, m, n, k, s);
  }
}

extern "C" int q3_gemm_norm(const void* A, const void* norm_w, float eps, const void* W, void* C,
                            int64_t M, int64_t N, int64_t K, int epilogue, const void* aux,
                            q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(A && norm_w && W && C, "q3_gemm_norm: null pointer");
  Q3_REQUIRE(M >= 1 && M <= 16, "q3_gemm_norm: M=%lld outside [1, 16] (decode shapes)",
             (long long)M);
  Q3_REQUIRE(N > 0 && N % 16 == 0 && K > 0 && K % 32 == 0 && N < (1ll << 31) && K < (1ll << 31),
             "q3_gemm_norm: bad shape N=%lld K=%lld", (long long)N, (long long)K);
  Q3_REQUIRE(epilogue == Q3_EPI_NONE || epilogue == Q3_EPI_RESIDUAL || epilogue == Q3_EPI_SWIGLU,
             "q3_gemm_norm: unknown epilogue %d", epilogue);
  Q3_REQUIRE(epilogue != Q3_EPI_RESIDUAL || aux, "q3_gemm_norm: residual epilogue needs aux");
  Q3_REQUIRE(aligned(A, 16) && aligned(W, 16) && aligned(C, 16) && aligned(norm_w, 16) &&
                 (!aux || aligned(aux, 16)),
             "q3_gemm_norm: pointers must be 16-byte aligned");
  GemvOpts o;
  o.norm_w = norm_w;
  o.eps = eps;
  return launch_gemv(A, W, C, aux, (int)M, (int)N, (int)K, epilogue, (cudaStream_t)stream, o);
}

extern "C" int q3_gate_up_swiglu(const void* A, const void* W_gate_up, void* C, int64_t M,
                                 int64_t inter, int64_t K, const void* norm_w, float eps,
                                 q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(A && W_gate_up && C, "q3_gate_up_swiglu: null pointer");
  Q3_REQUIRE(M >= 0 && inter > 0 && inter % 8 == 0 && inter < (1ll << 30),
             "q3_gate_up_swiglu: bad shape M=%lld inter=%lld (inter %% 8 == 0)", (long long)M,
             (long long)inter);
  Q3_REQUIRE(!norm_w || M <= 16,
             "q3_gate_up_swiglu: the fused norm is for M <= 16 (got %lld); normalise first",
             (long long)M);
  if (norm_w) {
    if (M == 0) return Q3_OK;
    return q3_gemm_norm(A, norm_w, eps, W_gate_up, C, M, 2 * inter, K, Q3_EPI_SWIGLU, nullptr,
                        stream);
  }
  return q3_gemm(A, W_gate_up, C, M, 2 * inter, K, Q3_EPI_SWIGLU, nullptr, stream);
}

extern "C" int q3_gemm_decode(const void* A, const void* W, void* C, int64_t M, int64_t N,
                              int64_t K, int epilogue, const void* aux, const void* norm_w,
                              float eps, const float* ss_in, int ss_tiles, float* ss_out,
                              q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(A && W && C, "q3_gemm_decode: null pointer");
  Q3_REQUIRE(M >= 1 && M <= 16, "q3_gemm_decode: M=%lld outside [1, 16]", (long long)M);
  Q3_REQUIRE(N > 0 && N % 16 == 0 && K > 0 && K % 32 == 0 && N < (1ll << 31) && K < (1ll << 31),
             "q3_gemm_decode: bad shape N=%lld K=%lld", (long long)N, (long long)K);
  Q3_REQUIRE(epilogue == Q3_EPI_NONE || epilogue == Q3_EPI_RESIDUAL || epilogue == Q3_EPI_SWIGLU,
             "q3_gemm_decode: unknown epilogue %d", epilogue);
  Q3_REQUIRE(epilogue != Q3_EPI_RESIDUAL || aux, "q3_gemm_decode: residual epilogue needs aux");
  Q3_REQUIRE(!ss_in || (norm_w && ss_tiles > 0), "q3_gemm_decode: ss_in needs norm_w, ss_tiles");
  Q3_REQUIRE(!ss_out || epilogue == Q3_EPI_RESIDUAL,
             "q3_gemm_decode: ss_out is produced by the residual epilogue only");
  Q3_REQUIRE(aligned(A, 16) && aligned(W, 16) && aligned(C, 16) &&
                 (!norm_w || aligned(norm_w, 16)) && (!aux || aligned(aux, 16)),
             "q3_gemm_decode: pointers must be 16-byte aligned");
  GemvOpts o;
  o.norm_w = norm_w;
  o.eps = eps;
  o.ss_in = ss_in;
  o.ss_tiles = ss_tiles;
  o.ss_out = ss_out;
  return launch_gemv(A, W, C, aux, (int)M, (int)N, (int)K, epilogue, (cudaStream_t)stream, o);
}

extern "C" int q3_gemm_qkv_rope(const void* A, const void* W, int64_t hidden, const void* q_norm_w,
                                const void* k_norm_w, const void* cos, const void* sin,
                                int cs_dtype, int cs_use_pos, int64_t cs_offset,
                                int64_t cs_stride_b, void* q_out, void* k_cache, void* v_cache,
                                int B, int S, int Hq, int Hkv, int head_dim, int64_t start_pos,
                                int64_t max_seq, float eps, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(A && W && q_norm_w && k_norm_w && cos && sin && q_out && k_cache && v_cache,
             "q3_gemm_qkv_rope: null pointer");
  Q3_REQUIRE(head_dim == 128, "q3_gemm_qkv_rope: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(B > 0 && S > 0 && Hq > 0 && Hkv > 0 && (int64_t)B * S > 16 &&
                 (int64_t)B * S < (1ll << 31),
             "q3_gemm_qkv_rope: needs B*S > 16 tokens (prefill); B=%d S=%d", B, S);
  Q3_REQUIRE(hidden > 0 && hidden % 32 == 0 && hidden < (1ll << 31),
             "q3_gemm_qkv_rope: hidden=%lld must be a multiple of 32", (long long)hidden);
  Q3_REQUIRE(cs_dtype == Q3_F32 || cs_dtype == Q3_BF16, "q3_gemm_qkv_rope: bad cs_dtype");
  Q3_REQUIRE(start_pos >= 0 && start_pos + S <= max_seq,
             "q3_gemm_qkv_rope: positions %lld..%lld outside the cache (%lld rows)",
             (long long)start_pos, (long long)(start_pos + S - 1), (long long)max_seq);
  Q3_REQUIRE(aligned(A, 16) && aligned(W, 16) && aligned(q_norm_w, 16) && aligned(k_norm_w, 16) &&
                 aligned(cos, 16) && aligned(sin, 16) && aligned(q_out, 16) &&
                 aligned(k_cache, 16) && aligned(v_cache, 16),
             "q3_gemm_qkv_rope: pointers must be 16-byte aligned");
  TcQkv q;
  q.q_norm = (const __nv_bfloat16*)q_norm_w;
  q.k_norm = (const __nv_bfloat16*)k_norm_w;
  q.cos = cos;
  q.sin = sin;
  q.cs_f32 = cs_dtype == Q3_F32;
  q.cs_use_pos = cs_use_pos ? 1 : 0;
  q.cs_offset = cs_offset;
  q.cs_stride_b = cs_stride_b;
  q.q_out = (__nv_bfloat16*)q_out;
  q.k_cache = (__nv_bfloat16*)k_cache;
  q.v_cache = (__nv_bfloat16*)v_cache;
  q.S = S; q.Hq = Hq; q.Hkv = Hkv;
  q.start_pos = start_pos;
  q.max_seq = max_seq;
  q.eps = eps;
  const int M = B * S, N = (Hq + 2 * Hkv) * 128;
  return launch_tc<256, kEpiQkvRope>(A, W, nullptr, nullptr, M, N, (int)hidden,
                                     (cudaStream_t)stream, &q);
}

extern "C" int q3_gemm_bias(const void* A, const void* W, const void* bias, void* C, int64_t M,
                            int64_t N, int64_t K, int epilogue, const void* aux,
                            q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(A && W && bias && C, "q3_gemm_bias: null pointer");
  Q3_REQUIRE(M >= 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31),
             "q3_gemm_bias: bad shape M=%lld N=%lld K=%lld", (long long)M, (long long)N,
             (long long)K);
  Q3_REQUIRE(K % 8 == 0, "q3_gemm_bias: K=%lld must be a multiple of 8 (16-byte rows)",
             (long long)K);
  Q3_REQUIRE(N % 8 == 0, "q3_gemm_bias: N=%lld must be a multiple of 8", (long long)N);
  Q3_REQUIRE(epilogue == Q3_EPI_BIAS || epilogue == Q3_EPI_BIAS_GELU_TANH ||
                 epilogue == Q3_EPI_BIAS_GELU || epilogue == Q3_EPI_BIAS_RESIDUAL,
             "q3_gemm_bias: epilogue %d is not a bias epilogue", epilogue);
  Q3_REQUIRE(epilogue != Q3_EPI_BIAS_RESIDUAL || aux, "q3_gemm_bias: residual epilogue needs aux");
  Q3_REQUIRE(aligned(A, 16) && aligned(W, 16) && aligned(C, 16) && aligned(bias, 16) &&
                 (!aux || aligned(aux, 16)),
             "q3_gemm_bias: pointers must be 16-byte aligned");
  if (M == 0) return Q3_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int m = (int)M, n = (int)N, k = (int)K;
  switch (epilogue) {
    case Q3_EPI_BIAS: return launch_tc<256, Q3_EPI_BIAS>(A, W, C, aux, m, n, k, s, nullptr, bias);
    case Q3_EPI_BIAS_GELU_TANH:
      return launch_tc<256, Q3_EPI_BIAS_GELU_TANH>(A, W, C, aux, m, n, k, s, nullptr, bias);
    case Q3_EPI_BIAS_GELU:
      return launch_tc<256, Q3_EPI_BIAS_GELU>(A, W, C, aux, m, n, k, s, nullptr, bias);
    default:
      return launch_tc<256, Q3_EPI_BIAS_RESIDUAL>(A, W, C, aux, m, n, k, s, nullptr, bias);
  }
}

extern "C" int q3_gemm_qkv_rope_paged(const void* A, const void* W, int64_t hidden,
                                      const void* q_norm_w, const void* k_norm_w, const void* cos,
                                      const void* sin, int cs_dtype, int cs_use_pos,
                                      int64_t cs_offset, int64_t cs_stride_b, void* q_out,
                                      void* k_pages, void* v_pages, int B, int S, int Hq, int Hkv,
                                      int head_dim, int64_t start_pos, const int32_t* block_table,
                                      int64_t table_stride, int page_tokens, int num_pages,
                                      float eps, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(A && W && q_norm_w && k_norm_w && cos && sin && q_out && k_pages && v_pages &&
                 block_table,
             "q3_gemm_qkv_rope_paged: null pointer");
  Q3_REQUIRE(head_dim == 128, "q3_gemm_qkv_rope_paged: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(B > 0 && S > 0 && Hq > 0 && Hkv > 0 && (int64_t)B * S > 16 &&
                 (int64_t)B * S < (1ll << 31),
             "q3_gemm_qkv_rope_paged: needs B*S > 16 tokens (prefill); B=%d S=%d", B, S);
  Q3_REQUIRE(hidden > 0 && hidden % 32 == 0 && hidden < (1ll << 31),
             "q3_gemm_qkv_rope_paged: hidden=%lld must be a multiple of 32", (long long)hidden);
  Q3_REQUIRE(cs_dtype == Q3_F32 || cs_dtype == Q3_BF16, "q3_gemm_qkv_rope_paged: bad cs_dtype");
  Q3_REQUIRE(page_tokens > 0 && num_pages > 0 && table_stride > 0 && start_pos >= 0 &&
                 start_pos + S <= table_stride * page_tokens,
             "q3_gemm_qkv_rope_paged: positions %lld..%lld beyond the table width",
             (long long)start_pos, (long long)(start_pos + S - 1));
  Q3_REQUIRE(aligned(A, 16) && aligned(W, 16) && aligned(q_norm_w, 16) && aligned(k_norm_w, 16) &&
                 aligned(cos, 16) && aligned(sin, 16) && aligned(q_out, 16) &&
                 aligned(k_pages, 16) && aligned(v_pages, 16) && aligned(block_table, 4),
             "q3_gemm_qkv_rope_paged: pointers must be 16-byte aligned");
  TcQkv q{};
  q.q_norm = (const __nv_bfloat16*)q_norm_w;
  q.k_norm = (const __nv_bfloat16*)k_norm_w;
  q.cos = cos;
  q.sin = sin;
  q.cs_f32 = cs_dtype == Q3_F32;
  q.cs_use_pos = cs_use_pos ? 1 : 0;
  q.cs_offset = cs_offset;
  q.cs_stride_b = cs_stride_b;
  q.q_out = (__nv_bfloat16*)q_out;
  q.k_cache = (__nv_bfloat16*)k_pages;
  q.v_cache = (__nv_bfloat16*)v_pages;
  q.S = S; q.Hq = Hq; q.Hkv = Hkv;
  q.start_pos = start_pos;
  q.max_seq = table_stride * page_tokens;
  q.eps = eps;
  q.pages = block_table;
  q.pages_stride = table_stride;
  q.page_tokens = page_tokens;
  q.num_pages = num_pages;
  const int M = B * S, N = (Hq + 2 * Hkv) * 128;
  return launch_tc<256, kEpiQkvRopePaged>(A, W, nullptr, nullptr, M, N, (int)hidden,
                                          (cudaStream_t)stream, &q);
}
