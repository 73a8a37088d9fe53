// a13: embedding gather (model_fused.py:281) and greedy argmax
// (model_fused.py:310,320).  Both are HBM-bound copies/scans with 16-byte loads.
// At TP > 1 the argmax is distributed: each rank reduces its vocabulary slice
// to one int64 key per row, and a MAX all-reduce of the keys replaces the
// all_gather of the full logits (model_fused.py:289-292).
#include <float.h>

#include "common.cuh"

namespace q3 {

__global__ void embed_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             __nv_bfloat16* __restrict__ out, int64_t n, int64_t hidden,
                             int64_t vocab, int* err) {
  pdl_wait();
  pdl_launch();
  const int64_t tok = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (tok >= n) return;
  const int64_t id = ids[tok];
  uint4* dst = reinterpret_cast<uint4*>(out + tok * hidden);
  const int64_t nvec = hidden >> 3;
  if (id < 0 || id >= vocab) {
    if (lane == 0 && err) atomicCAS(err, 0, 0x201);
    for (int64_t v = lane; v < nvec; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + id * hidden);
  for (int64_t v = lane; v < nvec; v += 32) dst[v] = __ldg(src + v);
}

// Order-preserving int64 key of (value, global index): the high word orders
// the float (sign-magnitude bits mapped to two's complement order), the low
// word is ~index, so the larger key is the larger value and, on equal values,
// the lower index.  A MAX reduction of the ranks' keys is then the argmax of
// the concatenated vocabulary with torch.argmax's first-index tie rule.
__device__ __forceinline__ int64_t argmax_key(float v, int64_t gidx) {
  // -0.0 + 0.0 = +0.0: equal values get equal high words, as torch.argmax sees them
  const uint32_t u = __float_as_uint(v + 0.0f);
  const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  const int64_t hi = (int64_t)(int32_t)(ord ^ 0x80000000u);
  return (int64_t)((uint64_t)hi << 32) | (int64_t)(0xffffffffu - (uint32_t)gidx);
}

// One CTA per row; ties resolve to the lowest index like torch.argmax.  With
// KEY, writes argmax_key(max, col_offset + index) instead of the index.
template <bool KEY>
__global__ void __launch_bounds__(512) argmax_kernel(const __nv_bfloat16* __restrict__ logits,
                                                     int64_t V, int64_t* __restrict__ out,
                                                     int64_t col_offset) {
  pdl_wait();
  pdl_launch();
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * V;
  float best = -INFINITY;
  int64_t bi = INT64_MAX;
  const int64_t nvec = V >> 3;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  for (int64_t v = threadIdx.x; v < nvec; v += blockDim.x) {
    const uint4 u = __ldg(xv + v);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(w[i]);
      const int64_t j = v * 8 + 2 * i;
      if (f.x > best) { best = f.x; bi = j; }
      if (f.y > best) { best = f.y; bi = j + 1; }
    }
  }
  for (int64_t j = nvec * 8 + threadIdx.x; j < V; j += blockDim.x) {
    const float f = bf2f(x[j]);
    if (f > best) { best = f; bi = j; }
  }
  // warp then block reduction of (best, index)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  __shared__ float sb[16];
  __shared__ int64_t si[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sb[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : INT64_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if (lane == 0) {
      if constexpr (KEY)
        out[row] = argmax_key(best, col_offset + ((bi == INT64_MAX) ? 0 : bi));
      else
        out[row] = (bi == INT64_MAX) ? 0 : bi;
    }
  }
}

__global__ void argmax_key_index_kernel(const int64_t* __restrict__ keys, int64_t rows,
                                        int64_t* __restrict__ out) {
  pdl_wait();
  pdl_launch();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows) out[i] = (int64_t)(0xffffffffu - (uint32_t)(keys[i] & 0xffffffff));
}

// out = bf16(a + b), the bf16 residual add of model_fused.py:269/275.
__global__ void add_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b,
                           uint4* __restrict__ out, int64_t nvec) {
  pdl_wait();
  pdl_launch();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 x = a[i], y = b[i];
    const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fx = unpack_bf16x2(xs[j]), fy = unpack_bf16x2(ys[j]);
      o[j] = pack_bf16x2(fx.x + fy.x, fx.y + fy.y);
    }
    out[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace q3

extern "C" int q3_add(const void* a, const void* b, void* out, int64_t n, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(a && b && out, "q3_add: null pointer");
  Q3_REQUIRE(n >= 0 && n % 8 == 0, "q3_add: n=%lld must be a multiple of 8", (long long)n);
  Q3_REQUIRE(aligned(a, 16) && aligned(b, 16) && aligned(out, 16), "q3_add: misaligned");
  if (n == 0) return Q3_OK;
  const int64_t nvec = n / 8;
  int64_t blocks = (nvec + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  return launch_ex(add_kernel, dim3((unsigned)blocks), dim3(256), 0, (cudaStream_t)stream, 1,
                   (const uint4*)a, (const uint4*)b, (uint4*)out, nvec);
}

extern "C" int q3_embed(const int64_t* ids, const void* table, void* out, int64_t n,
                        int64_t hidden, int64_t vocab, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(ids && table && out, "q3_embed: null pointer");
  Q3_REQUIRE(n >= 0 && hidden > 0 && hidden % 8 == 0 && vocab > 0, "q3_embed: bad shape");
  Q3_REQUIRE(aligned(table, 16) && aligned(out, 16) && aligned(ids, 8), "q3_embed: misaligned");
  if (n == 0) return Q3_OK;
  return launch_ex(embed_kernel, dim3((unsigned)((n + 7) / 8)), dim3(256), 0,
                   (cudaStream_t)stream, 1, ids, (const __nv_bfloat16*)table,
                   (__nv_bfloat16*)out, n, hidden, vocab, device_error_word());
}

extern "C" int q3_argmax(const void* logits, int64_t rows, int64_t V, int64_t* out_idx,
                         q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(logits && out_idx, "q3_argmax: null pointer");
  Q3_REQUIRE(rows >= 0 && V > 0 && V % 8 == 0, "q3_argmax: V=%lld must be a multiple of 8",
             (long long)V);
  Q3_REQUIRE(aligned(logits, 16), "q3_argmax: misaligned logits");
  if (rows == 0) return Q3_OK;
  return launch_ex(argmax_kernel<false>, dim3((unsigned)rows), dim3(512), 0,
                   (cudaStream_t)stream, 1, (const __nv_bfloat16*)logits, V, out_idx,
                   (int64_t)0);
}

extern "C" int q3_argmax_key(const void* logits, int64_t rows, int64_t V, int64_t col_offset,
                             int64_t* out_key, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(logits && out_key, "q3_argmax_key: null pointer");
  Q3_REQUIRE(rows >= 0 && V > 0 && V % 8 == 0, "q3_argmax_key: V=%lld must be a multiple of 8",
             (long long)V);
  Q3_REQUIRE(col_offset >= 0 && col_offset + V <= 0xffffffffLL,
             "q3_argmax_key: indices must fit in 32 bits");
  Q3_REQUIRE(aligned(logits, 16) && aligned(out_key, 8), "q3_argmax_key: misaligned");
  if (rows == 0) return Q3_OK;
  return launch_ex(argmax_kernel<true>, dim3((unsigned)rows), dim3(512), 0,
                   (cudaStream_t)stream, 1, (const __nv_bfloat16*)logits, V, out_key, col_offset);
}

extern "C" int q3_argmax_key_index(const int64_t* keys, int64_t rows, int64_t* out_idx,
                                   q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(keys && out_idx, "q3_argmax_key_index: null pointer");
  Q3_REQUIRE(rows >= 0, "q3_argmax_key_index: bad rows");
  Q3_REQUIRE(aligned(keys, 8) && aligned(out_idx, 8), "q3_argmax_key_index: misaligned");
  if (rows == 0) return Q3_OK;
  return launch_ex(argmax_key_index_kernel, dim3((unsigned)((rows + 127) / 128)), dim3(128), 0,
                   (cudaStream_t)stream, 1, keys, rows, out_idx);
}

namespace q3 {
namespace {
constexpr int64_t kPrefetchPiece = 32 << 10;

// Brings a byte range into L2 with bulk prefetches (no data is written
// anywhere).  One thread per CTA issues its slice.  The kernel lets its
// dependent start at once and completes only after its own predecessor, so
// the stream's order holds for the kernel after it.
__global__ void l2_prefetch_kernel(const uint8_t* base, int64_t bytes, int64_t chunk) {
  pdl_launch();
  const int64_t off = (int64_t)blockIdx.x * chunk;
  if (threadIdx.x == 0 && off < bytes) {
    const int64_t n = min64(chunk, bytes - off);
    for (int64_t o = 0; o < n; o += kPrefetchPiece) {
      const uint32_t sz = (uint32_t)min64(kPrefetchPiece, n - o);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + off + o), "r"(sz)
                   : "memory");
    }
  }
  pdl_wait();
}
}  // namespace
}  // namespace q3

extern "C" int q3_l2_prefetch(const void* ptr, int64_t bytes, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(ptr, "q3_l2_prefetch: null pointer");
  Q3_REQUIRE(bytes >= 0 && bytes % 16 == 0, "q3_l2_prefetch: bytes=%lld must be a multiple of 16",
             (long long)bytes);
  Q3_REQUIRE(aligned(ptr, 16), "q3_l2_prefetch: the range must start 16-byte aligned");
  if (bytes == 0) return Q3_OK;
  int64_t ctas = (bytes + kPrefetchPiece - 1) / kPrefetchPiece;
  if (ctas > num_sms()) ctas = num_sms();
  const int64_t chunk = ((bytes + ctas - 1) / ctas + 15) / 16 * 16;
  ctas = (bytes + chunk - 1) / chunk;
  return launch_ex(l2_prefetch_kernel, dim3((unsigned)ctas), dim3(32), 0, (cudaStream_t)stream,
                   1, (const uint8_t*)ptr, bytes, chunk);
}

extern "C" int q3_lm_head_argmax(const void* hidden, const void* norm_w, float eps,
                                 const void* W_lm, int64_t rows, int64_t V, int64_t K,
                                 int64_t col_offset, void* logits_ws, int keys, int64_t* out,
                                 q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(hidden && W_lm && logits_ws && out, "q3_lm_head_argmax: null pointer");
  Q3_REQUIRE(rows >= 0 && V > 0 && K > 0, "q3_lm_head_argmax: bad shape rows=%lld V=%lld K=%lld",
             (long long)rows, (long long)V, (long long)K);
  Q3_REQUIRE(!norm_w || rows <= 16,
             "q3_lm_head_argmax: the fused final norm is for rows <= 16 (got %lld)",
             (long long)rows);
  Q3_REQUIRE(keys || col_offset == 0,
             "q3_lm_head_argmax: indices over a vocabulary slice need keys (col_offset %lld)",
             (long long)col_offset);
  if (rows == 0) return Q3_OK;
  const int rc = norm_w ? q3_gemm_norm(hidden, norm_w, eps, W_lm, logits_ws, rows, V, K,
                                       Q3_EPI_NONE, nullptr, stream)
                        : q3_gemm(hidden, W_lm, logits_ws, rows, V, K, Q3_EPI_NONE, nullptr,
                                  stream);
  if (rc) return rc;
  return keys ? q3_argmax_key(logits_ws, rows, V, col_offset, out, stream)
              : q3_argmax(logits_ws, rows, V, out, stream);
}
