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
};

template <typename T, int G>
__global__ void __launch_bounds__(kDecWarps * 32) attn_decode_kernel(DecodeParams p) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int64_t L = p.kv_len_dev ? (int64_t)(*p.kv_len_dev) : p.kv_len;
  const int64_t start = (int64_t)split * p.chunk;
  const int64_t end = min64(start + p.chunk, L);

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

static void decode_split_plan(int B, int Hkv, int64_t max_kv_len, int* splits, int* chunk) {
  const int64_t L = max_kv_len < 1 ? 1 : max_kv_len;
  const int target = 2 * num_sms();
  int64_t sp = (target + (int64_t)B * Hkv - 1) / ((int64_t)B * Hkv);
  const int64_t max_sp = (L + kDecStep - 1) / kDecStep;
  if (sp > max_sp) sp = max_sp;
  if (sp < 1) sp = 1;
  int64_t ch = (L + sp - 1) / sp;
  ch = (ch + kDecStep - 1) / kDecStep * kDecStep;
  sp = (L + ch - 1) / ch;
  *splits = (int)sp;
  *chunk = (int)ch;
}

template <typename T>
static int launch_decode(DecodeParams& p, int G, cudaStream_t s) {
  dim3 grid(p.splits, p.Hkv, p.B), block(kDecWarps * 32);
  switch (G) {
    case 1: attn_decode_kernel<T, 1><<<grid, block, 0, s>>>(p); break;
    case 2: attn_decode_kernel<T, 2><<<grid, block, 0, s>>>(p); break;
    case 4: attn_decode_kernel<T, 4><<<grid, block, 0, s>>>(p); break;
    case 8: attn_decode_kernel<T, 8><<<grid, block, 0, s>>>(p); break;
    default: return fail(Q3_ERR_UNSUPPORTED, "q3_attn_decode: Hq/Hkv=%d not in {1,2,4,8}", G);
  }
  Q3_LAUNCH_CHECK();
  if (p.splits > 1) {
    const int warps = 4;
    const int64_t n = (int64_t)p.B * p.Hq;
    attn_decode_combine<T><<<(unsigned)((n + warps - 1) / warps), warps * 32, 0, s>>>(p);
    Q3_LAUNCH_CHECK();
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
//    before any stream capture on the device.
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
