// a6/a8: GQA decode attention for one query token per sequence.
//
// Semantics follow the eager path of forward_layer (model_fused.py:248-262)
// with S=1: out_h = softmax(q_h . K_g^T * scale) V_g over cache positions
// [0, kv_len), g = h / (Hq/Hkv).  The reference reads the whole max_seq buffer
// and masks the tail (model_fused.py:259-260); this kernel reads only the valid
// prefix, which gives the same result because masked scores contribute exp(-inf)=0.
//
// Layout/work split (HBM-bound: every K/V byte of the valid prefix is read once):
//   grid = (splits, Hkv, B); one CTA = 4 warps owns a contiguous chunk of cache
//   positions for one KV head and ALL Hq/Hkv query heads that share it, so K/V
//   are read once per KV head, not once per query head.  Each warp handles 4
//   positions per step with 8-byte (bf16) / 16-byte (fp32) coalesced loads, lane
//   l holding dims 4l..4l+3.  The G per-head dot products are reduced with a
//   transposed butterfly (log2 G halving steps, then full reduction) so a lane
//   ends with one head's score.  Online softmax runs in fp32 per warp; warps
//   merge in shared memory; splits merge in a second small kernel through the
//   fp32 workspace.
// That CUDA-core kernel serves the fp32 case (config 1); bf16 caches use the
// tensor-core kernel further down (TMA-fed K/V ring, mma.sync), which also has
// a variant that starts from the raw QKV row (q3_attn_decode_qkv): it applies
// the head norms and RoPE itself and writes the new token's K/V row.
#include <math.h>

#include "common.cuh"

namespace q3 {

constexpr int kDecWarps = 4;
constexpr int kDecUnroll = 4;                       // positions per warp step
constexpr int kDecStep = kDecWarps * kDecUnroll;    // positions per CTA step
constexpr int kHD = 128;

template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
  using raw = float4;
  __device__ static void load(const float* p, float (&v)[4]) {
    float4 f = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  }
  __device__ static void store(float* p, const float (&v)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <>
struct Vec4<__nv_bfloat16> {
  __device__ static void load(const __nv_bfloat16* p, float (&v)[4]) {
    uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  }
  __device__ static void store(__nv_bfloat16* p, const float (&v)[4]) {
    uint2 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    *reinterpret_cast<uint2*>(p) = u;
  }
};

// Butterfly that reduces G per-lane partial sums across the warp; afterwards
// the lane holds the full sum for head index head_of_lane<G>(lane) in d[0].
template <int G>
__device__ __forceinline__ void transpose_reduce(float (&d)[G], int lane) {
  int n = G;
  int bit = 16;
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    if (n > 1) {
      const int half = n >> 1;
      const bool hi = (lane & bit) != 0;
#pragma unroll
      for (int i = 0; i < G / 2; ++i) {
        if (i < half) {
          const float send = hi ? d[i] : d[i + half];
          const float recv = __shfl_xor_sync(0xffffffffu, send, bit);
          d[i] = (hi ? d[i + half] : d[i]) + recv;
        }
      }
      n = half;
    } else {
      d[0] += __shfl_xor_sync(0xffffffffu, d[0], bit);
    }
    bit >>= 1;
  }
}
template <int G>
__device__ __forceinline__ int head_of_lane(int lane) {
  if (G == 1) return 0;
  if (G == 2) return (lane >> 4) & 1;
  if (G == 4) return ((lane >> 4) & 1) * 2 + ((lane >> 3) & 1);
  return ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
}
// A lane that holds head g's reduced value.
template <int G>
__device__ __forceinline__ int lane_of_head(int g) {
  if (G == 1) return 0;
  if (G == 2) return g << 4;
  if (G == 4) return ((g >> 1) << 4) | ((g & 1) << 3);
  return ((g >> 2) << 4) | (((g >> 1) & 1) << 3) | ((g & 1) << 2);
}

struct DecodeParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  float* ws_acc;  // [B, Hq, splits, D]
  float* ws_ml;   // [B, Hq, splits, 2]  (running max, running sum)
  int B, Hq, Hkv, splits, chunk;
  int64_t kv_len;
  const int32_t* kv_len_dev;
  int64_t max_seq;
  float scale;
  // fused variant (q3_attn_decode_qkv): q and the new K/V row come from the
  // raw qkv row [B, (Hq+2*Hkv)*128]; QK-RMSNorm + RoPE run here
  const __nv_bfloat16* qkv;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const __nv_bfloat16* cos;  // bf16 [rows, 64]; row of the new token = pos + cs_offset
  const __nv_bfloat16* sin;
  int64_t cs_offset;
  float eps;
  __nv_bfloat16* k_cache_w;  // the caches again, for writing the new row
  __nv_bfloat16* v_cache_w;
  // paged variant (q3_attn_decode_paged): k/v are page pools [num_pages, Hkv,
  // page_tokens, 128]; position t of sequence b lives in page
  // pages[b * pages_stride + t / page_tokens] at offset t % page_tokens
  const int32_t* pages;
  int64_t pages_stride;
  int page_tokens, num_pages;
  // tensor-core kernel, splits > 1: the splits of one (sequence, KV head) run
  // as one thread-block cluster and cluster rank 0 merges them through
  // distributed shared memory (no workspace, no combine kernel)
  int cluster_merge;
};

// Positions per split.  The grid's split count is planned on the host from
// an upper bound of the length; when the length is read on the device, the
// chunk is recomputed from it so every split gets an equal share of the
// positions actually present (whole steps of `step`).
__device__ __forceinline__ int64_t split_chunk(const DecodeParams& p, int64_t L, int step) {
  if (!p.kv_len_dev || p.splits <= 1) return p.chunk;
  const int64_t ch = (L + p.splits - 1) / p.splits;
  return (ch + step - 1) / step * step;
}

template <typename T, int G>
__global__ void __launch_bounds__(kDecWarps * 32) attn_decode_kernel(DecodeParams p) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int64_t L = p.kv_len_dev ? (int64_t)(*p.kv_len_dev) : p.kv_len;
  const int64_t chunk = split_chunk(p, L, kDecStep);
  const int64_t start = (int64_t)split * chunk;
  const int64_t end = min64(start + chunk, L);

  const T* qb = reinterpret_cast<const T*>(p.q) + ((int64_t)b * p.Hq + (int64_t)kvh * G) * kHD;
  const T* kb = reinterpret_cast<const T*>(p.k) + ((int64_t)b * p.Hkv + kvh) * p.max_seq * kHD;
  const T* vb = reinterpret_cast<const T*>(p.v) + ((int64_t)b * p.Hkv + kvh) * p.max_seq * kHD;
  const int d0 = lane * 4;

  float q[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) Vec4<T>::load(qb + g * kHD + d0, q[g]);

  const int my_g = head_of_lane<G>(lane);
  float m_run = -INFINITY, l_run = 0.f;  // for head my_g (replicated across its lanes)
  float acc[G][4];
  float m_all[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m_all[g] = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[g][i] = 0.f;
  }

  for (int64_t base = start + warp * kDecUnroll; base < end; base += kDecStep) {
    float kv[kDecUnroll][4], vv[kDecUnroll][4];
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) {
      const int64_t pos = base + u;
      if (pos < end) {
        Vec4<T>::load(kb + pos * kHD + d0, kv[u]);
        Vec4<T>::load(vb + pos * kHD + d0, vv[u]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) kv[u][i] = vv[u][i] = 0.f;
      }
    }
    float s[kDecUnroll];
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) {
      float d[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) a = fmaf(q[g][i], kv[u][i], a);
        d[g] = a;
      }
      transpose_reduce<G>(d, lane);
      s[u] = (base + u < end) ? d[0] * p.scale : -INFINITY;
    }
    float m_new = m_run;
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) m_new = fmaxf(m_new, s[u]);
    const float corr = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
    float pr[kDecUnroll];
    float psum = 0.f;
#pragma unroll
    for (int u = 0; u < kDecUnroll; ++u) {
      pr[u] = (s[u] == -INFINITY) ? 0.f : expf(s[u] - m_new);
      psum += pr[u];
    }
    l_run = l_run * corr + psum;
    m_run = m_new;
    // broadcast each head's correction and probabilities to every lane
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int src = lane_of_head<G>(g);
      const float cg = __shfl_sync(0xffffffffu, corr, src);
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[g][i] *= cg;
#pragma unroll
      for (int u = 0; u < kDecUnroll; ++u) {
        const float pg = __shfl_sync(0xffffffffu, pr[u], src);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[g][i] = fmaf(pg, vv[u][i], acc[g][i]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) m_all[g] = __shfl_sync(0xffffffffu, m_run, lane_of_head<G>(g));
  float l_all[G];
#pragma unroll
  for (int g = 0; g < G; ++g) l_all[g] = __shfl_sync(0xffffffffu, l_run, lane_of_head<G>(g));

  // merge the 4 warps through shared memory
  __shared__ float sm_acc[kDecWarps][G][kHD];
  __shared__ float sm_ml[kDecWarps][G][2];
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int i = 0; i < 4; ++i) sm_acc[warp][g][d0 + i] = acc[g][i];
    if (lane == 0) {
      sm_ml[warp][g][0] = m_all[g];
      sm_ml[warp][g][1] = l_all[g];
    }
  }
  __syncthreads();
  // thread t handles (g = t / 32 ... ) : G*128 outputs over 128 threads
  for (int idx = threadIdx.x; idx < G * kHD; idx += blockDim.x) {
    const int g = idx / kHD, d = idx % kHD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, sm_ml[w][g][0]);
    float a = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
      const float mw = sm_ml[w][g][0];
      const float f = (mw == -INFINITY) ? 0.f : expf(mw - M);
      a = fmaf(f, sm_acc[w][g][d], a);
      l = fmaf(f, sm_ml[w][g][1], l);
    }
    const int h = kvh * G + g;
    if (p.splits == 1) {
      T* o = reinterpret_cast<T*>(p.out) + ((int64_t)b * p.Hq + h) * kHD + d;
      const float val = (l > 0.f) ? a / l : 0.f;
      if constexpr (sizeof(T) == 4) *reinterpret_cast<float*>(o) = val;
      else *reinterpret_cast<__nv_bfloat16*>(o) = f2bf(val);
    } else {
      const int64_t slot = ((int64_t)b * p.Hq + h) * p.splits + split;
      p.ws_acc[slot * kHD + d] = a;
      if (d == 0) {
        p.ws_ml[slot * 2 + 0] = M;
        p.ws_ml[slot * 2 + 1] = l;
      }
    }
  }
}

// One warp per (b, h): merge the split partials.
template <typename T>
__global__ void attn_decode_combine(DecodeParams p) {
  // dependents first: the projection that follows prefetches its weights
  // before its own wait, which covers this kernel's outputs
  pdl_launch();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t bh = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (bh >= (int64_t)p.B * p.Hq) return;
  const float* ml = p.ws_ml + bh * p.splits * 2;
  float M = -INFINITY;
  for (int s = lane; s < p.splits; s += 32) M = fmaxf(M, ml[2 * s]);
  M = warp_max(M);
  float a[4] = {0.f, 0.f, 0.f, 0.f};
  float l = 0.f;
  const int d0 = lane * 4;
  for (int s = 0; s < p.splits; ++s) {
    const float ms = ml[2 * s];
    if (ms == -INFINITY) continue;
    const float f = expf(ms - M);
    l = fmaf(f, ml[2 * s + 1], l);
    const float4 v = *reinterpret_cast<const float4*>(p.ws_acc + (bh * p.splits + s) * kHD + d0);
    a[0] = fmaf(f, v.x, a[0]);
    a[1] = fmaf(f, v.y, a[1]);
    a[2] = fmaf(f, v.z, a[2]);
    a[3] = fmaf(f, v.w, a[3]);
  }
  const float inv = (l > 0.f) ? 1.f / l : 0.f;
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = a[i] * inv;
  Vec4<T>::store(reinterpret_cast<T*>(p.out) + bh * kHD + d0, o);
}

// Split the valid prefix [0, L) into chunks (multiples of `step`) so that the
// grid covers about two CTAs per SM.  A larger step never yields more splits,
// so the plan with the smallest step bounds the workspace of every kernel.
static void decode_split_plan_step(int B, int Hkv, int64_t max_kv_len, int step, int* splits,
                                   int* chunk) {
  const int64_t L = max_kv_len < 1 ? 1 : max_kv_len;
  const int target = 2 * num_sms();
  int64_t sp = (target + (int64_t)B * Hkv - 1) / ((int64_t)B * Hkv);
  const int64_t max_sp = (L + step - 1) / step;
  if (sp > max_sp) sp = max_sp;
  if (sp < 1) sp = 1;
  int64_t ch = (L + sp - 1) / sp;
  ch = (ch + step - 1) / step * step;
  sp = (L + ch - 1) / ch;
  *splits = (int)sp;
  *chunk = (int)ch;
}

static void decode_split_plan(int B, int Hkv, int64_t max_kv_len, int* splits, int* chunk) {
  decode_split_plan_step(B, Hkv, max_kv_len, kDecStep, splits, chunk);
}

// ---------------------------------------------------------------------------
// bf16 tensor-core variant.  The fp32 kernel above keeps the exact fp32
// arithmetic config 1 needs; for bf16 caches the work per position (G query
// heads x 128 dims, twice) moves to mma.sync so the kernel is HBM-bound:
//   * a producer warp streams 64-position K and V tiles of the split's chunk
//     with TMA (two 64-dim boxes each, 128-byte swizzle) into a 3-stage ring
//     (32 KB per stage, full/empty mbarriers);
//   * four consumer warps take 16 positions of each tile: S = Q K^T with the
//     G query heads as rows 0..G-1 of the 16-row A operand (Q fragments stay
//     in registers), online softmax per head row in fp32, then O += P V with
//     V read by ldmatrix.trans; K is read by ldmatrix from the swizzled tile;
//   * the warps merge (m, l, O) in shared memory and write one split-K
//     partial (or the output when there is a single split).
// ---------------------------------------------------------------------------
constexpr int kTcTile = 64;                       // positions per stage
constexpr int kTcStages = 3;
constexpr int kTcHalfBytes = kTcTile * 128;       // one 64x64 bf16 box (8 KB)
constexpr int kTcStageBytes = 4 * kTcHalfBytes;   // K lo/hi + V lo/hi = 32 KB
constexpr int kTcConsumers = 4;
constexpr int kTcThreads = (kTcConsumers + 1) * 32;
constexpr int kTcSmem = kTcStages * kTcStageBytes + 1024 + 256;

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
// Byte offset of 16-byte chunk c (0..15 across the 128 dims) of row r in a
// stage's K or V region (two 64-dim boxes, each with the 128-byte swizzle).
__device__ __forceinline__ uint32_t kv_off(int r, int c) {
  return (c >> 3) * kTcHalfBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

struct DecodeTcParams {
  DecodeParams p;
  int* err;
};

// One head row of the fused variant, computed by one warp as q3_qkv_norm_rope
// computes it (lane owns dims 4*lane .. 4*lane+3, partner dims via lane ^ 16):
// RMSNorm over the head (model_fused.py:113-119) and rotate-half RoPE
// (:122-129) in the reference's bf16 rounding points.
// The lane's norm-weight and RoPE-table entries (static data: loadable before
// the wait on the kernel that produced qkv).
struct HeadTabs {
  uint2 w, c, s;
};
__device__ __forceinline__ HeadTabs head_tabs(const __nv_bfloat16* w, const __nv_bfloat16* cs_cos,
                                              const __nv_bfloat16* cs_sin, int64_t crow,
                                              int lane) {
  const int d0 = lane * 4, j0 = d0 & 63;
  HeadTabs t;
  t.w = *reinterpret_cast<const uint2*>(w + d0);
  t.c = *reinterpret_cast<const uint2*>(cs_cos + crow * 64 + j0);
  t.s = *reinterpret_cast<const uint2*>(cs_sin + crow * 64 + j0);
  return t;
}
__device__ __forceinline__ void head_norm_rope(const __nv_bfloat16* x, const HeadTabs& tb,
                                               float eps, int lane, float (&o)[4]) {
  const int d0 = lane * 4;
  const uint2 u = *reinterpret_cast<const uint2*>(x + d0);
  const float2 a = unpack_bf16x2(u.x), bb = unpack_bf16x2(u.y);
  const float v[4] = {a.x, a.y, bb.x, bb.y};
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss * (1.0f / kHD) + eps);
  const float2 w0 = unpack_bf16x2(tb.w.x), w1 = unpack_bf16x2(tb.w.y);
  const float wv[4] = {w0.x, w0.y, w1.x, w1.y};
  const float2 c0 = unpack_bf16x2(tb.c.x), c1 = unpack_bf16x2(tb.c.y);
  const float2 s0 = unpack_bf16x2(tb.s.x), s1 = unpack_bf16x2(tb.s.y);
  const float cv[4] = {c0.x, c0.y, c1.x, c1.y}, sv[4] = {s0.x, s0.y, s1.x, s1.y};
  float n[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = rbf(rbf(v[i] * r) * wv[i]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float pp = __shfl_xor_sync(0xffffffffu, n[i], 16);
    const float rot = (lane < 16) ? -pp : pp;
    o[i] = rbf(rbf(n[i] * cv[i]) + rbf(rot * sv[i]));
  }
}

template <int G, bool FQ, bool PAGED = false>
__global__ void __launch_bounds__(kTcThreads) attn_decode_tc_kernel(
    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
    DecodeTcParams prm) {
  // No dependency wait yet: cache rows below the newest position were
  // completed before this launch sequence began (the host API contract), so
  // the producer streams them while the kernel that writes q and the newest
  // row finishes.  q, the newest row and the outputs wait for it.
  pdl_launch();
  const DecodeParams& p = prm.p;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kTcStages * kTcStageBytes);
  uint64_t* empty = full + kTcStages;
  __shared__ float sm_o[kTcConsumers][G][kHD];
  __shared__ float sm_ml[kTcConsumers][G][2];
  __shared__ __align__(16) __nv_bfloat16 q_s[FQ ? G : 1][kHD];  // FQ: normed, rotated q
  __shared__ float new_s[FQ ? 2 : 1][kHD];                       // FQ: new k and v rows
  __shared__ float snew_s[FQ ? G : 1];                           // FQ: new row's scores
  __shared__ float cl_ml[G][2];  // cluster merge: this split's (max, sum) per head

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int64_t L = p.kv_len_dev ? (int64_t)(*p.kv_len_dev) : p.kv_len;
  const int64_t chunk = split_chunk(p, L, kTcTile);
  const int64_t start = (int64_t)split * chunk;
  // FQ: the cache rows streamed are the old ones [0, L-1); the new token's
  // row L-1 is computed here and added by the split whose range holds it
  const int64_t end = min64(start + chunk, FQ ? L - 1 : L);
  const bool with_new = FQ && start <= L - 1 && L - 1 < start + chunk;
  const int ntiles = end > start ? (int)((end - start + kTcTile - 1) / kTcTile) : 0;
  const int64_t row_base = ((int64_t)b * p.Hkv + kvh) * p.max_seq + start;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTcConsumers);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  __syncthreads();

  if (warp == kTcConsumers) {
    if (lane == 0) {
      bool waited = false;
      for (int i = 0; i < ntiles; ++i) {
        const int s = i % kTcStages;
        const uint32_t ph = (i / kTcStages) & 1;
        // a tile reaching the newest row (L - 1) waits for its writer (the
        // fused variant never reads that row from the cache)
        if (!FQ && !waited && start + (int64_t)(i + 1) * kTcTile > L - 1) {
          pdl_wait();
          waited = true;
        }
        if (!mbar_wait(&empty[s], ph ^ 1, prm.err, 0x401)) break;
        uint8_t* st = ring + s * kTcStageBytes;
        int y;
        if constexpr (PAGED) {
          // a 64-position tile never straddles pages (page_tokens % 64 == 0)
          const int64_t t = start + (int64_t)i * kTcTile;
          int pg = p.pages[(int64_t)b * p.pages_stride + t / p.page_tokens];
          if (pg < 0 || pg >= p.num_pages) {  // a bad table entry: record it, read page 0
            report_timeout(prm.err, 0x402);
            pg = 0;
          }
          y = (int)(((int64_t)pg * p.Hkv + kvh) * p.page_tokens + t % p.page_tokens);
        } else {
          y = (int)(row_base + (int64_t)i * kTcTile);
        }
        mbar_arrive_expect_tx(&full[s], kTcStageBytes);
        tma_load_2d(st, &tmK, &full[s], 0, y, kCacheEvictFirst);
        tma_load_2d(st + kTcHalfBytes, &tmK, &full[s], 64, y, kCacheEvictFirst);
        tma_load_2d(st + 2 * kTcHalfBytes, &tmV, &full[s], 0, y, kCacheEvictFirst);
        tma_load_2d(st + 3 * kTcHalfBytes, &tmV, &full[s], 64, y, kCacheEvictFirst);
      }
    }
  } else {
    HeadTabs qtab{};
    if constexpr (FQ) qtab = head_tabs(p.q_norm, p.cos, p.sin, (L - 1) + p.cs_offset, lane);
    pdl_wait();  // q and the outputs
    const int g = lane >> 2, t = lane & 3;
    if constexpr (FQ) {
      // this KV head's G query heads, normed and rotated, into shared memory
      const int ld = (p.Hq + 2 * p.Hkv) * kHD;
      for (int gg = warp; gg < G; gg += kTcConsumers) {
        float o4[4];
        head_norm_rope(p.qkv + (int64_t)b * ld + (kvh * G + gg) * kHD, qtab, p.eps, lane, o4);
        *reinterpret_cast<uint2*>(&q_s[gg][lane * 4]) =
            make_uint2(pack_bf16x2(o4[0], o4[1]), pack_bf16x2(o4[2], o4[3]));
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kTcConsumers * 32) : "memory");
    }
    // Q as the A operand: row g = query head kvh*G + g (rows >= G are zero)
    uint32_t qf[8][2];
    {
      const __nv_bfloat16* qh =
          FQ ? &q_s[g < G ? g : 0][0]
             : reinterpret_cast<const __nv_bfloat16*>(p.q) + ((int64_t)b * p.Hq + kvh * G + g) * kHD;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        if (g < G) {
          qf[ks][0] = *reinterpret_cast<const uint32_t*>(qh + ks * 16 + 2 * t);
          qf[ks][1] = *reinterpret_cast<const uint32_t*>(qh + ks * 16 + 8 + 2 * t);
        } else {
          qf[ks][0] = qf[ks][1] = 0u;
        }
      }
    }
    const float sl2 = p.scale * 1.4426950408889634f;
    float o[16][2];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = 0.f;
    float m_r = -INFINITY, l_r = 0.f;
    const uint32_t ring_base = smem_u32(ring);

    for (int i = 0; i < ntiles; ++i) {
      const int s = i % kTcStages;
      const uint32_t ph = (i / kTcStages) & 1;
      if (!mbar_wait(&full[s], ph, prm.err, 0x402)) break;
      const uint32_t sK = ring_base + s * kTcStageBytes;
      const uint32_t sV = sK + 2 * kTcHalfBytes;
      // ---- S = Q K^T: 16 rows x 16 positions (two n-tiles of 8) ----
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t kf[4];
        const int r = warp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks * 2 + ((lane >> 3) & 1);
        ldsm_x4(kf, sK + kv_off(r, c));
        mma_bf16_16816(sc[0], qf[ks][0], 0u, qf[ks][1], 0u, kf[0], kf[1]);
        mma_bf16_16816(sc[1], qf[ks][0], 0u, qf[ks][1], 0u, kf[2], kf[3]);
      }
      // ---- mask + online softmax for row g (c0, c1 of each n-tile) ----
      const int64_t pos0 = start + (int64_t)i * kTcTile + warp * 16;
      float x[4];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int64_t pos = pos0 + j * 8 + 2 * t + e;
          x[j * 2 + e] = (pos < end) ? sc[j][e] * sl2 : -INFINITY;
        }
      float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_r, mx);
      const float base = (m_new == -INFINITY) ? 0.f : m_new;
      const float corr = exp2f(m_r - base);
      float pr[4], rs = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        pr[e] = exp2f(x[e] - base);
        rs += pr[e];
      }
      l_r = l_r * corr + rs;
      m_r = m_new;
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        o[d][0] *= corr;
        o[d][1] *= corr;
      }
      // P as A (rows g; rows g+8 are zero): k = 16 positions of this warp
      const uint32_t pa0 = pack_bf16x2(pr[0], pr[1]);
      const uint32_t pa2 = pack_bf16x2(pr[2], pr[3]);
      // ---- O += P V ----
#pragma unroll
      for (int ip = 0; ip < 8; ++ip) {
        uint32_t vf[4];
        const int r = warp * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = ip * 2 + (lane >> 4);
        ldsm_x4_t(vf, sV + kv_off(r, c));
        float d0[4] = {o[2 * ip][0], o[2 * ip][1], 0.f, 0.f};
        float d1[4] = {o[2 * ip + 1][0], o[2 * ip + 1][1], 0.f, 0.f};
        mma_bf16_16816(d0, pa0, 0u, pa2, 0u, vf[0], vf[1]);
        mma_bf16_16816(d1, pa0, 0u, pa2, 0u, vf[2], vf[3]);
        o[2 * ip][0] = d0[0]; o[2 * ip][1] = d0[1];
        o[2 * ip + 1][0] = d1[0]; o[2 * ip + 1][1] = d1[1];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // row sums across the 4 lanes of a row
    l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
    l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);
    if (g < G) {
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        sm_o[warp][g][d * 8 + 2 * t] = o[d][0];
        sm_o[warp][g][d * 8 + 2 * t + 1] = o[d][1];
      }
      if (t == 0) {
        sm_ml[warp][g][0] = m_r;  // in log2 units
        sm_ml[warp][g][1] = l_r;
      }
    }
  }
  __syncthreads();
  if constexpr (FQ) {
    if (with_new) {
      // the new token's k (normed, rotated) and v rows: into the caches and
      // into this split's merge (warps 0 and 1; the producer warp idles)
      const int ld = (p.Hq + 2 * p.Hkv) * kHD;
      const int64_t pos = L - 1;
      const int64_t crow = pos + p.cs_offset;
      int64_t crow_off;
      bool row_ok = true;
      if constexpr (PAGED) {
        // the new row's page (the caller grew the table to hold it)
        const int pg = p.pages[(int64_t)b * p.pages_stride + pos / p.page_tokens];
        row_ok = pg >= 0 && pg < p.num_pages;
        if (!row_ok && threadIdx.x == 0) report_timeout(prm.err, 0x402);
        crow_off = ((row_ok ? (int64_t)pg * p.Hkv + kvh : 0) * p.page_tokens +
                    pos % p.page_tokens) * kHD;
      } else {
        crow_off = (((int64_t)b * p.Hkv + kvh) * p.max_seq + pos) * kHD;
      }
      if (warp == 0) {
        float o4[4];
        head_norm_rope(p.qkv + (int64_t)b * ld + (p.Hq + kvh) * kHD,
                       head_tabs(p.k_norm, p.cos, p.sin, crow, lane), p.eps, lane, o4);
        const uint2 pk = make_uint2(pack_bf16x2(o4[0], o4[1]), pack_bf16x2(o4[2], o4[3]));
        if (row_ok) *reinterpret_cast<uint2*>(p.k_cache_w + crow_off + lane * 4) = pk;
        const float2 a0 = unpack_bf16x2(pk.x), a1 = unpack_bf16x2(pk.y);
        new_s[0][lane * 4 + 0] = a0.x; new_s[0][lane * 4 + 1] = a0.y;
        new_s[0][lane * 4 + 2] = a1.x; new_s[0][lane * 4 + 3] = a1.y;
      } else if (warp == 1) {
        const uint2 pv = *reinterpret_cast<const uint2*>(
            p.qkv + (int64_t)b * ld + (p.Hq + p.Hkv + kvh) * kHD + lane * 4);
        if (row_ok) *reinterpret_cast<uint2*>(p.v_cache_w + crow_off + lane * 4) = pv;
        const float2 a0 = unpack_bf16x2(pv.x), a1 = unpack_bf16x2(pv.y);
        new_s[1][lane * 4 + 0] = a0.x; new_s[1][lane * 4 + 1] = a0.y;
        new_s[1][lane * 4 + 2] = a1.x; new_s[1][lane * 4 + 3] = a1.y;
      }
      __syncthreads();
      const float sl2 = p.scale * 1.4426950408889634f;
      for (int gg = warp; gg < G; gg += kTcConsumers + 1) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          acc = fmaf(bf2f(q_s[gg][lane * 4 + i]), new_s[0][lane * 4 + i], acc);
        acc = warp_sum(acc);
        if (lane == 0) snew_s[gg] = acc * sl2;
      }
      __syncthreads();
    }
  }
  // ---- merge the consumer warps; write the partial or the output ----
  for (int idx = threadIdx.x; idx < G * kHD; idx += blockDim.x) {
    const int gg = idx / kHD, d = idx % kHD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kTcConsumers; ++w) M = fmaxf(M, sm_ml[w][gg][0]);
    if (FQ && with_new) M = fmaxf(M, snew_s[FQ ? gg : 0]);
    float a = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kTcConsumers; ++w) {
      const float mw = sm_ml[w][gg][0];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      a = fmaf(f, sm_o[w][gg][d], a);
      l = fmaf(f, sm_ml[w][gg][1], l);
    }
    if (FQ && with_new) {
      const float f = exp2f(snew_s[FQ ? gg : 0] - M);
      a = fmaf(f, new_s[FQ ? 1 : 0][d], a);
      l += f;
    }
    const int h = kvh * G + gg;
    if (p.splits == 1) {
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out) + ((int64_t)b * p.Hq + h) * kHD;
      out[d] = f2bf(l > 0.f ? a / l : 0.f);
    } else if (p.cluster_merge) {
      // only this thread reads sm_o[*][gg][d]: its warp-0 slot takes the
      // split's sum; (max, sum) go to cl_ml, which no thread reads yet
      sm_o[0][gg][d] = a;
      if (d == 0) {
        cl_ml[gg][0] = M;  // log2 units
        cl_ml[gg][1] = l;
      }
    } else {
      const int64_t slot = ((int64_t)b * p.Hq + h) * p.splits + split;
      p.ws_acc[slot * kHD + d] = a;
      if (d == 0) {
        // the combine kernel works in natural-log units
        p.ws_ml[slot * 2 + 0] = (M == -INFINITY) ? -INFINITY : M * 0.6931471805599453f;
        p.ws_ml[slot * 2 + 1] = l;
      }
    }
  }
  if (p.splits > 1 && p.cluster_merge) {
    // every split of this (sequence, KV head) left (max, sum, O) in its own
    // shared memory; rank 0 reads them in rank order and writes the output,
    // and the second barrier keeps the peers resident until it has read
    cluster_sync_all();
    if (cluster_ctarank() == 0) {
      const uint32_t nr = cluster_nctarank();
      for (int idx = threadIdx.x; idx < G * kHD; idx += blockDim.x) {
        const int gg = idx / kHD, d = idx % kHD;
        const uint32_t a_loc = smem_u32(&sm_o[0][gg][d]);
        const uint32_t m_loc = smem_u32(&cl_ml[gg][0]);
        float M = -INFINITY;
        for (uint32_t r = 0; r < nr; ++r)
          M = fmaxf(M, ld_shared_cluster_f32(map_shared_rank(m_loc, r)));
        float a = 0.f, l = 0.f;
        for (uint32_t r = 0; r < nr; ++r) {
          const uint32_t mr = map_shared_rank(m_loc, r);
          const float mw = ld_shared_cluster_f32(mr);
          if (mw == -INFINITY) continue;
          const float f = exp2f(mw - M);
          a = fmaf(f, ld_shared_cluster_f32(map_shared_rank(a_loc, r)), a);
          l = fmaf(f, ld_shared_cluster_f32(mr + 4), l);
        }
        __nv_bfloat16* out =
            reinterpret_cast<__nv_bfloat16*>(p.out) + ((int64_t)b * p.Hq + kvh * G + gg) * kHD;
        out[d] = f2bf(l > 0.f ? a / l : 0.f);
      }
    }
    cluster_sync_all();
  }
}

static void decode_split_plan_step(int B, int Hkv, int64_t max_kv_len, int step, int* splits,
                                   int* chunk);

// Decode attention CTAs per SM the split plan may use (Q3VL_DECODE_SLOTS_PER_SM
// = 1 or 2; unset: as many as are resident, at most 2), for sweeping the
// split on a GPU without a rebuild.
static int decode_slots_per_sm() {
  static const int v = [] {
    const char* e = getenv("Q3VL_DECODE_SLOTS_PER_SM");
    const int x = e ? atoi(e) : 0;
    return (x == 1 || x == 2) ? x : 0;
  }();
  return v;
}

// Whether the tensor-core kernel merges 2-8 splits inside a thread-block
// cluster (Q3VL_DECODE_CLUSTER_MERGE=1) instead of through the workspace and
// the combine kernel (the default).  Measured on B200, B = 8, L = 1152 in a
// CUDA graph: 11.7 us per call with the cluster merge against 10.1 us with
// the combine kernel, whose launch overlaps the next kernel's start; clusters
// must be co-scheduled in one GPC, and the next launch's CTAs lose their
// early start.  Read per call so a process can compare both.
static bool decode_cluster_merge() {
  const char* e = getenv("Q3VL_DECODE_CLUSTER_MERGE");
  return e && e[0] == '1';
}

static int launch_decode_tc(DecodeParams& p, int G, cudaStream_t s, bool fused_qkv = false,
                            bool paged = false) {
  void (*kern)(const CUtensorMap, const CUtensorMap, DecodeTcParams) = nullptr;
  int gi = 0;
  if (paged) {
    switch (G) {
      case 1: kern = fused_qkv ? attn_decode_tc_kernel<1, true, true> : attn_decode_tc_kernel<1, false, true>; gi = 8; break;
      case 2: kern = fused_qkv ? attn_decode_tc_kernel<2, true, true> : attn_decode_tc_kernel<2, false, true>; gi = 9; break;
      case 4: kern = fused_qkv ? attn_decode_tc_kernel<4, true, true> : attn_decode_tc_kernel<4, false, true>; gi = 10; break;
      case 8: kern = fused_qkv ? attn_decode_tc_kernel<8, true, true> : attn_decode_tc_kernel<8, false, true>; gi = 11; break;
      default: return fail(Q3_ERR_UNSUPPORTED, "q3_attn_decode: Hq/Hkv=%d not in {1,2,4,8}", G);
    }
    if (fused_qkv) gi += 4;
  } else {
    switch (G) {
      case 1: kern = fused_qkv ? attn_decode_tc_kernel<1, true> : attn_decode_tc_kernel<1, false>; gi = 0; break;
      case 2: kern = fused_qkv ? attn_decode_tc_kernel<2, true> : attn_decode_tc_kernel<2, false>; gi = 1; break;
      case 4: kern = fused_qkv ? attn_decode_tc_kernel<4, true> : attn_decode_tc_kernel<4, false>; gi = 2; break;
      case 8: kern = fused_qkv ? attn_decode_tc_kernel<8, true> : attn_decode_tc_kernel<8, false>; gi = 3; break;
      default: return fail(Q3_ERR_UNSUPPORTED, "q3_attn_decode: Hq/Hkv=%d not in {1,2,4,8}", G);
    }
    if (fused_qkv) gi += 4;
  }
  static int per_sm_cache[64][16] = {{0}};
  int dev = 0;
  cudaGetDevice(&dev);
  const bool cacheable = dev >= 0 && dev < 64;
  if (!cacheable || per_sm_cache[dev][gi] == 0) {
    Q3_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kTcSmem));
    int per_sm = 0;
    Q3_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTcThreads,
                                                                kTcSmem));
    if (cacheable) per_sm_cache[dev][gi] = per_sm > 0 ? per_sm : 1;
  }
  const int per_sm = cacheable ? per_sm_cache[dev][gi] : 1;
  // One wave: at most (resident CTAs per SM x SMs) CTAs, and never more splits
  // than the workspace was sized for (two CTAs per SM, 16-position chunks).
  int64_t slots = (int64_t)per_sm * num_sms();
  if (slots > 2 * (int64_t)num_sms()) slots = 2 * (int64_t)num_sms();
  const int64_t pairs = (int64_t)p.B * p.Hkv;
  // one CTA per SM: its ring keeps the SM's stream at full rate, and the
  // splits come out more even and leave fewer partials to merge (B200, L =
  // 1152: 8 pairs 7.6 us against 11.6 us at two CTAs per SM; 64 pairs 17.4
  // against 19.5 us per call)
  slots = num_sms();
  if (decode_slots_per_sm() > 0 && decode_slots_per_sm() <= per_sm)
    slots = (int64_t)decode_slots_per_sm() * num_sms();
  const int64_t L = p.kv_len < 1 ? 1 : p.kv_len;
  int64_t sp = slots / pairs;
  const int64_t max_sp = (L + kTcTile - 1) / kTcTile;
  if (sp > max_sp) sp = max_sp;
  if (sp < 1) sp = 1;
  int64_t ch = (L + sp - 1) / sp;
  ch = (ch + kTcTile - 1) / kTcTile * kTcTile;
  sp = (L + ch - 1) / ch;
  if (sp > 1 && (p.splits <= 1 || sp > p.splits))
    return fail(Q3_ERR_INVALID, "q3_attn_decode: internal split plan mismatch");
  p.splits = (int)sp;
  p.chunk = (int)ch;
  if (sp > 1) p.ws_ml = p.ws_acc + (size_t)p.B * p.Hq * sp * kHD;
  // 2-8 splits: one cluster per (sequence, KV head), merged in shared memory
  const bool cl = sp > 1 && sp <= 8 && decode_cluster_merge();
  p.cluster_merge = cl ? 1 : 0;
  CUtensorMap tk, tv;
  const int64_t rows = paged ? (int64_t)p.num_pages * p.Hkv * p.page_tokens
                             : (int64_t)p.B * p.Hkv * p.max_seq;
  int rc = cached_tmap_2d(&tk, p.k, rows, kHD, kTcTile, 64);
  if (rc) return rc;
  rc = cached_tmap_2d(&tv, p.v, rows, kHD, kTcTile, 64);
  if (rc) return rc;
  DecodeTcParams prm{p, device_error_word()};
  rc = launch_ex_cluster(kern, dim3(p.splits, p.Hkv, p.B), dim3(kTcThreads), kTcSmem, s,
                         dim3(cl ? p.splits : 1, 1, 1), tk, tv, prm);
  if (rc) return rc;
  if (p.splits > 1 && !cl) {
    const int warps = 4;
    const int64_t n = (int64_t)p.B * p.Hq;
    rc = launch_ex(attn_decode_combine<__nv_bfloat16>, dim3((unsigned)((n + warps - 1) / warps)),
                   dim3(warps * 32), 0, s, 1, p);
    if (rc) return rc;
  }
  return Q3_OK;
}

template <typename T>
static int launch_decode(DecodeParams& p, int G, cudaStream_t s) {
  if constexpr (sizeof(T) == 2) return launch_decode_tc(p, G, s);
  dim3 grid(p.splits, p.Hkv, p.B), block(kDecWarps * 32);
  int rc = Q3_OK;
  switch (G) {
    case 1: rc = launch_ex(attn_decode_kernel<T, 1>, grid, block, 0, s, 1, p); break;
    case 2: rc = launch_ex(attn_decode_kernel<T, 2>, grid, block, 0, s, 1, p); break;
    case 4: rc = launch_ex(attn_decode_kernel<T, 4>, grid, block, 0, s, 1, p); break;
    case 8: rc = launch_ex(attn_decode_kernel<T, 8>, grid, block, 0, s, 1, p); break;
    default: return fail(Q3_ERR_UNSUPPORTED, "q3_attn_decode: Hq/Hkv=%d not in {1,2,4,8}", G);
  }
  if (rc) return rc;
  if (p.splits > 1) {
    const int warps = 4;
    const int64_t n = (int64_t)p.B * p.Hq;
    rc = launch_ex(attn_decode_combine<T>, dim3((unsigned)((n + warps - 1) / warps)),
                   dim3(warps * 32), 0, s, 1, p);
    if (rc) return rc;
  }
  return Q3_OK;
}

}  // namespace q3

extern "C" size_t q3_attn_decode_workspace_bytes(int B, int Hq, int Hkv, int head_dim,
                                                 int64_t max_kv_len) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || head_dim <= 0) return 0;
  int splits = 1, chunk = 0;
  q3::decode_split_plan(B, Hkv, max_kv_len, &splits, &chunk);
  if (splits == 1) return 0;
  return (size_t)B * Hq * splits * (head_dim + 2) * sizeof(float);
}

extern "C" int q3_attn_decode(const void* q, const void* k_cache, const void* v_cache, void* out,
                              int B, int Hq, int Hkv, int head_dim, int64_t kv_len,
                              const int32_t* kv_len_dev, int64_t max_seq, float scale, int dtype,
                              void* workspace, size_t workspace_bytes, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(q && k_cache && v_cache && out, "q3_attn_decode: null pointer");
  Q3_REQUIRE(head_dim == kHD, "q3_attn_decode: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0,
             "q3_attn_decode: bad heads Hq=%d Hkv=%d", Hq, Hkv);
  Q3_REQUIRE(kv_len >= 1 && kv_len <= max_seq,
             "q3_attn_decode: kv_len=%lld outside [1, max_seq=%lld]", (long long)kv_len,
             (long long)max_seq);
  Q3_REQUIRE(dtype == Q3_F32 || dtype == Q3_BF16, "q3_attn_decode: dtype must be f32 or bf16");
  const size_t align = dtype == Q3_F32 ? 16 : 8;
  Q3_REQUIRE(aligned(q, align) && aligned(k_cache, align) && aligned(v_cache, align) &&
                 aligned(out, align),
             "q3_attn_decode: misaligned pointer");
  DecodeParams p{};
  p.q = q; p.k = k_cache; p.v = v_cache; p.out = out;
  p.B = B; p.Hq = Hq; p.Hkv = Hkv;
  p.kv_len = kv_len; p.kv_len_dev = kv_len_dev; p.max_seq = max_seq; p.scale = scale;
  decode_split_plan(B, Hkv, kv_len, &p.splits, &p.chunk);
  if (p.splits > 1) {
    const size_t need = (size_t)B * Hq * p.splits * (kHD + 2) * sizeof(float);
    Q3_REQUIRE(workspace && workspace_bytes >= need && aligned(workspace, 16),
               "q3_attn_decode: workspace of %zu bytes needed (got %zu)", need, workspace_bytes);
    p.ws_acc = reinterpret_cast<float*>(workspace);
    p.ws_ml = p.ws_acc + (size_t)B * Hq * p.splits * kHD;
  }
  const int G = Hq / Hkv;
  cudaStream_t s = (cudaStream_t)stream;
  return dtype == Q3_F32 ? launch_decode<float>(p, G, s) : launch_decode<__nv_bfloat16>(p, G, s);
}

extern "C" int q3_attn_decode_qkv(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                                  const void* cos, const void* sin, int64_t cs_offset,
                                  void* k_cache, void* v_cache, void* out, int B, int Hq, int Hkv,
                                  int head_dim, int64_t kv_len, const int32_t* kv_len_dev,
                                  int64_t max_seq, float scale, float eps, void* workspace,
                                  size_t workspace_bytes, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(qkv && q_norm_w && k_norm_w && cos && sin && k_cache && v_cache && out,
             "q3_attn_decode_qkv: null pointer");
  Q3_REQUIRE(head_dim == kHD, "q3_attn_decode_qkv: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0,
             "q3_attn_decode_qkv: bad heads Hq=%d Hkv=%d", Hq, Hkv);
  Q3_REQUIRE(kv_len >= 1 && kv_len <= max_seq,
             "q3_attn_decode_qkv: kv_len=%lld outside [1, max_seq=%lld]", (long long)kv_len,
             (long long)max_seq);
  Q3_REQUIRE(aligned(qkv, 8) && aligned(q_norm_w, 8) && aligned(k_norm_w, 8) && aligned(cos, 8) &&
                 aligned(sin, 8) && aligned(k_cache, 16) && aligned(v_cache, 16) &&
                 aligned(out, 8),
             "q3_attn_decode_qkv: misaligned pointer");
  DecodeParams p{};
  p.q = nullptr; p.k = k_cache; p.v = v_cache; p.out = out;
  p.B = B; p.Hq = Hq; p.Hkv = Hkv;
  p.kv_len = kv_len; p.kv_len_dev = kv_len_dev; p.max_seq = max_seq; p.scale = scale;
  p.qkv = (const __nv_bfloat16*)qkv;
  p.q_norm = (const __nv_bfloat16*)q_norm_w;
  p.k_norm = (const __nv_bfloat16*)k_norm_w;
  p.cos = (const __nv_bfloat16*)cos;
  p.sin = (const __nv_bfloat16*)sin;
  p.cs_offset = cs_offset;
  p.eps = eps;
  p.k_cache_w = (__nv_bfloat16*)k_cache;
  p.v_cache_w = (__nv_bfloat16*)v_cache;
  decode_split_plan(B, Hkv, kv_len, &p.splits, &p.chunk);
  if (p.splits > 1) {
    const size_t need = (size_t)B * Hq * p.splits * (kHD + 2) * sizeof(float);
    Q3_REQUIRE(workspace && workspace_bytes >= need && aligned(workspace, 16),
               "q3_attn_decode_qkv: workspace of %zu bytes needed (got %zu)", need,
               workspace_bytes);
    p.ws_acc = reinterpret_cast<float*>(workspace);
    p.ws_ml = p.ws_acc + (size_t)B * Hq * p.splits * kHD;
  }
  return launch_decode_tc(p, Hq / Hkv, (cudaStream_t)stream, true);
}

// The fused variant over a page pool: the new token's K/V row goes to its page
// (block_table[b, (kv_len - 1) / page_tokens]), the older rows are read
// through the table.
extern "C" int q3_attn_decode_qkv_paged(const void* qkv, const void* q_norm_w,
                                        const void* k_norm_w, const void* cos, const void* sin,
                                        int64_t cs_offset, void* k_pages, void* v_pages, void* out,
                                        int B, int Hq, int Hkv, int head_dim, int64_t kv_len,
                                        const int32_t* kv_len_dev, const int32_t* block_table,
                                        int64_t table_stride, int page_tokens, int num_pages,
                                        float scale, float eps, void* workspace,
                                        size_t workspace_bytes, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(qkv && q_norm_w && k_norm_w && cos && sin && k_pages && v_pages && out && block_table,
             "q3_attn_decode_qkv_paged: null pointer");
  Q3_REQUIRE(head_dim == kHD, "q3_attn_decode_qkv_paged: head_dim must be 128 (got %d)",
             head_dim);
  Q3_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0,
             "q3_attn_decode_qkv_paged: bad heads Hq=%d Hkv=%d", Hq, Hkv);
  Q3_REQUIRE(page_tokens > 0 && page_tokens % kTcTile == 0 && num_pages > 0,
             "q3_attn_decode_qkv_paged: page_tokens=%d must be a positive multiple of %d",
             page_tokens, kTcTile);
  Q3_REQUIRE((int64_t)num_pages * Hkv * page_tokens < (1ll << 31),
             "q3_attn_decode_qkv_paged: pool of %d pages too large for 32-bit rows", num_pages);
  Q3_REQUIRE(table_stride > 0 && kv_len >= 1 && kv_len <= table_stride * page_tokens,
             "q3_attn_decode_qkv_paged: kv_len=%lld beyond the table width (%lld pages of %d)",
             (long long)kv_len, (long long)table_stride, page_tokens);
  Q3_REQUIRE(aligned(qkv, 8) && aligned(q_norm_w, 8) && aligned(k_norm_w, 8) && aligned(cos, 8) &&
                 aligned(sin, 8) && aligned(k_pages, 16) && aligned(v_pages, 16) &&
                 aligned(out, 8) && aligned(block_table, 4),
             "q3_attn_decode_qkv_paged: misaligned pointer");
  DecodeParams p{};
  p.q = nullptr; p.k = k_pages; p.v = v_pages; p.out = out;
  p.B = B; p.Hq = Hq; p.Hkv = Hkv;
  p.kv_len = kv_len; p.kv_len_dev = kv_len_dev; p.max_seq = table_stride * page_tokens;
  p.scale = scale;
  p.qkv = (const __nv_bfloat16*)qkv;
  p.q_norm = (const __nv_bfloat16*)q_norm_w;
  p.k_norm = (const __nv_bfloat16*)k_norm_w;
  p.cos = (const __nv_bfloat16*)cos;
  p.sin = (const __nv_bfloat16*)sin;
  p.cs_offset = cs_offset;
  p.eps = eps;
  p.k_cache_w = (__nv_bfloat16*)k_pages;
  p.v_cache_w = (__nv_bfloat16*)v_pages;
  p.pages = block_table;
  p.pages_stride = table_stride;
  p.page_tokens = page_tokens;
  p.num_pages = num_pages;
  decode_split_plan(B, Hkv, kv_len, &p.splits, &p.chunk);
  if (p.splits > 1) {
    const size_t need = (size_t)B * Hq * p.splits * (kHD + 2) * sizeof(float);
    Q3_REQUIRE(workspace && workspace_bytes >= need && aligned(workspace, 16),
               "q3_attn_decode_qkv_paged: workspace of %zu bytes needed (got %zu)", need,
               workspace_bytes);
    p.ws_acc = reinterpret_cast<float*>(workspace);
    p.ws_ml = p.ws_acc + (size_t)B * Hq * p.splits * kHD;
  }
  return launch_decode_tc(p, Hq / Hkv, (cudaStream_t)stream, true, true);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of q3_attn_decode.
//
// Some callers cannot allocate device memory when they call this kernel: a
// serving runtime that has already handed all free HBM to its own KV-cache
// pool, or a foreign-language binding that only owns the q/cache/out buffers
// and has no allocator to create a split-K workspace with.  This entry point
// takes no workspace.  Its split-K partial sums live in the fixed array below,
// which every GPU that loads this library keeps for the life of the process.
//
// Limits and sharing rules:
//  * the array holds kNoAllocScratchBytes (4 MiB); a request whose split-K
//    partials would need more is rejected with Q3_ERR_INVALID before launch;
//  * all calls on a device share the one array, and it keeps whatever the
//    last call wrote.  Each call writes every partial slot it later reads, so
//    nothing needs clearing between calls, but two calls that run at the same
//    time on the GPU (different streams, or different host threads) overwrite
//    each other's partials: order them on one stream;
//  * the first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current).  Make that first call
//    before any stream capture on the device.  The address is kept for the
//    life of the process: after cudaDeviceReset the module may load elsewhere,
//    so reload the library before calling this entry point again;
//  * the split plan launches at most 2 x SMs + B x Hkv CTAs, so the partials
//    need at most (4 x SMs) x G x 520 bytes (G = Hq / Hkv <= 8): about 2.5 MB
//    on a 148-SM B200.  The limit binds only on larger GPUs or for head ratios
//    the kernels do not support.
// ---------------------------------------------------------------------------
#include <mutex>

namespace q3 {
constexpr size_t kNoAllocScratchBytes = 4u << 20;
static __device__ __align__(256) float g_decode_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of g_decode_scratch on the current device (looked up once per
// device); nullptr with the error recorded if the lookup fails.
static float* decode_scratch_address() {
  static float* addr[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("q3_attn_decode_noalloc: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) {
      set_error("q3_attn_decode_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = static_cast<float*>(p);
  }
  return addr[dev];
}
}  // namespace q3

extern "C" int q3_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                      void* out, int B, int Hq, int Hkv, int head_dim,
                                      int64_t kv_len, const int32_t* kv_len_dev, int64_t max_seq,
                                      float scale, int dtype, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(q && k_cache && v_cache && out, "q3_attn_decode_noalloc: null pointer");
  Q3_REQUIRE(head_dim == kHD, "q3_attn_decode_noalloc: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0,
             "q3_attn_decode_noalloc: bad heads Hq=%d Hkv=%d", Hq, Hkv);
  Q3_REQUIRE(kv_len >= 1 && kv_len <= max_seq,
             "q3_attn_decode_noalloc: kv_len=%lld outside [1, max_seq=%lld]",
             (long long)kv_len, (long long)max_seq);
  Q3_REQUIRE(dtype == Q3_F32 || dtype == Q3_BF16,
             "q3_attn_decode_noalloc: dtype must be f32 or bf16");
  const size_t align = dtype == Q3_F32 ? 16 : 8;
  Q3_REQUIRE(aligned(q, align) && aligned(k_cache, align) && aligned(v_cache, align) &&
                 aligned(out, align),
             "q3_attn_decode_noalloc: misaligned pointer");
  DecodeParams p{};
  p.q = q; p.k = k_cache; p.v = v_cache; p.out = out;
  p.B = B; p.Hq = Hq; p.Hkv = Hkv;
  p.kv_len = kv_len; p.kv_len_dev = kv_len_dev; p.max_seq = max_seq; p.scale = scale;
  decode_split_plan(B, Hkv, kv_len, &p.splits, &p.chunk);
  if (p.splits > 1) {
    const size_t need = (size_t)B * Hq * p.splits * (kHD + 2) * sizeof(float);
    Q3_REQUIRE(need <= kNoAllocScratchBytes,
               "q3_attn_decode_noalloc: split-K partials need %zu bytes, more than the %zu-byte "
               "built-in scratch (use q3_attn_decode with a caller workspace)",
               need, kNoAllocScratchBytes);
    float* scratch = decode_scratch_address();
    if (!scratch) return Q3_ERR_CUDA;
    p.ws_acc = scratch;
    p.ws_ml = p.ws_acc + (size_t)B * Hq * p.splits * kHD;
  }
  const int G = Hq / Hkv;
  cudaStream_t s = (cudaStream_t)stream;
  return dtype == Q3_F32 ? launch_decode<float>(p, G, s) : launch_decode<__nv_bfloat16>(p, G, s);
}

extern "C" int q3_attn_decode_paged(const void* q, const void* k_pages, const void* v_pages,
                                    void* out, int B, int Hq, int Hkv, int head_dim,
                                    int64_t kv_len, const int32_t* kv_len_dev,
                                    const int32_t* block_table, int64_t table_stride,
                                    int page_tokens, int num_pages, float scale, void* workspace,
                                    size_t workspace_bytes, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(q && k_pages && v_pages && out && block_table, "q3_attn_decode_paged: null pointer");
  Q3_REQUIRE(head_dim == kHD, "q3_attn_decode_paged: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(B > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0,
             "q3_attn_decode_paged: bad heads Hq=%d Hkv=%d", Hq, Hkv);
  Q3_REQUIRE(page_tokens > 0 && page_tokens % kTcTile == 0 && num_pages > 0,
             "q3_attn_decode_paged: page_tokens=%d must be a positive multiple of %d",
             page_tokens, kTcTile);
  Q3_REQUIRE((int64_t)num_pages * Hkv * page_tokens < (1ll << 31),
             "q3_attn_decode_paged: pool of %d pages too large for 32-bit rows", num_pages);
  Q3_REQUIRE(table_stride > 0 && kv_len >= 1 && kv_len <= table_stride * page_tokens,
             "q3_attn_decode_paged: kv_len=%lld beyond the table width (%lld pages of %d)",
             (long long)kv_len, (long long)table_stride, page_tokens);
  Q3_REQUIRE(aligned(q, 8) && aligned(k_pages, 16) && aligned(v_pages, 16) && aligned(out, 8) &&
                 aligned(block_table, 4),
             "q3_attn_decode_paged: misaligned pointer");
  DecodeParams p{};
  p.q = q; p.k = k_pages; p.v = v_pages; p.out = out;
  p.B = B; p.Hq = Hq; p.Hkv = Hkv;
  p.kv_len = kv_len; p.kv_len_dev = kv_len_dev; p.max_seq = table_stride * page_tokens;
  p.scale = scale;
  p.pages = block_table;
  p.pages_stride = table_stride;
  p.page_tokens = page_tokens;
  p.num_pages = num_pages;
  decode_split_plan(B, Hkv, kv_len, &p.splits, &p.chunk);
  if (p.splits > 1) {
    const size_t need = (size_t)B * Hq * p.splits * (kHD + 2) * sizeof(float);
    Q3_REQUIRE(workspace && workspace_bytes >= need && aligned(workspace, 16),
               "q3_attn_decode_paged: workspace of %zu bytes needed (got %zu)", need,
               workspace_bytes);
    p.ws_acc = reinterpret_cast<float*>(workspace);
    p.ws_ml = p.ws_acc + (size_t)B * Hq * p.splits * kHD;
  }
  return launch_decode_tc(p, Hq / Hkv, (cudaStream_t)stream, false, true);
}
