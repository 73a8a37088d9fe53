// a3 epilogue, a4, a5, a9: RoPE / M-RoPE tables / per-head QK-norm + RoPE +
// KV-cache write.  All three kernels are HBM-bound elementwise passes: one warp
// owns one 128-wide head row, lane l holds elements 4l..4l+3, and the
// rotate_half partner (d +/- 64) sits on lane l^16.
#include "common.cuh"

namespace q3 {

constexpr int kHeadDim = 128;

__device__ __forceinline__ void load4_bf16(const __nv_bfloat16* p, float (&v)[4]) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void store4_bf16(__nv_bfloat16* p, const float (&v)[4]) {
  uint2 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = u;
}

// ---------------------------------------------------------------------------
// a9: qwen3_rope (kernels/rope.py:24-96), checked against the fp32 reference
// rope_ref (test_kernels.py:126-134): out = x*cos + rotate_half(x)*sin in fp32,
// one rounding to bf16.  Products and the sum are kept unfused (no FMA) so the
// result is bit-identical to that reference.
// ---------------------------------------------------------------------------
__global__ void rope_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ cs,
                            __nv_bfloat16* __restrict__ out, int64_t seq, int heads) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= seq * heads) return;
  const int64_t s = row / heads;
  const int d0 = lane * 4;
  const int j0 = d0 & 63;
  float v[4];
  load4_bf16(x + row * kHeadDim + d0, v);
  const float4 c = *reinterpret_cast<const float4*>(cs + s * kHeadDim + j0);
  const float4 sn = *reinterpret_cast<const float4*>(cs + s * kHeadDim + 64 + j0);
  const float cc[4] = {c.x, c.y, c.z, c.w};
  const float ss[4] = {sn.x, sn.y, sn.z, sn.w};
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float p = __shfl_xor_sync(0xffffffffu, v[i], 16);
    const float rot = (lane < 16) ? -p : p;
    o[i] = __fadd_rn(__fmul_rn(v[i], cc[i]), __fmul_rn(rot, ss[i]));
  }
  store4_bf16(out + row * kHeadDim + d0, o);
}

// ---------------------------------------------------------------------------
// a4: interleaved M-RoPE angle tables (transformers modeling_qwen3_vl.py:
// 352-386): angle_j = float(pos[axis(j)]) * inv_freq[j], fp32 cos/sin.
// ---------------------------------------------------------------------------
__global__ void mrope_kernel(const int64_t* __restrict__ pos, const float* __restrict__ inv_freq,
                             int64_t n_tok, int half, int sec_h, int sec_w,
                             float* __restrict__ cos_out, float* __restrict__ sin_out) {
  pdl_wait();
  pdl_launch();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_tok * half) return;
  const int64_t t = i / half;
  const int j = (int)(i - t * half);
  int axis = 0;
  if (j % 3 == 1 && j < 3 * sec_h) axis = 1;
  else if (j % 3 == 2 && j < 3 * sec_w) axis = 2;
  const float p = (float)pos[axis * n_tok + t];
  const float a = __fmul_rn(p, inv_freq[j]);
  float sv, cv;
  sincosf(a, &sv, &cv);
  cos_out[i] = cv;
  sin_out[i] = sv;
}

// ---------------------------------------------------------------------------
// a3 epilogue + a5 (model_fused.py:107-129, :244-246).  Reproduces the
// reference's bf16 rounding points op for op:
//   n   = bf16(bf16(x * rsqrt(mean(x^2)+eps)) * w)            (:113-119)
//   out = bf16(bf16(n*cos) + bf16(rotate_half(n)*sin))          (:122-129)
// with cos/sin rounded to bf16 first (the reference caches them in bf16,
// model_fused.py:49-50; HF casts its M-RoPE tables to the activation dtype).
// ---------------------------------------------------------------------------
template <typename CsT>
__device__ __forceinline__ void load4_cs(const CsT* p, float (&v)[4]);
template <>
__device__ __forceinline__ void load4_cs<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  load4_bf16(p, v);
}
template <>
__device__ __forceinline__ void load4_cs<float>(const float* p, float (&v)[4]) {
  float4 f = *reinterpret_cast<const float4*>(p);
  v[0] = rbf(f.x); v[1] = rbf(f.y); v[2] = rbf(f.z); v[3] = rbf(f.w);
}

// Page-pool addressing of the K/V rows (q3_qkv_norm_rope_paged).
struct PageRef {
  const int32_t* table;  // [B, stride]
  int64_t stride;
  int page_tokens, num_pages;
  int* err;
};

// Element offset of K/V row (b, kv head, position t) in a page pool, or -1
// (recorded in the error word) when the table does not map t into the pool.
__device__ __forceinline__ int64_t page_row(const PageRef& pr, int b, int hkv, int Hkv,
                                            int64_t t) {
  const int64_t slot = t / pr.page_tokens;
  const int pg = (t >= 0 && slot < pr.stride) ? pr.table[(int64_t)b * pr.stride + slot] : -1;
  if (pg < 0 || pg >= pr.num_pages) {
    report_timeout(pr.err, 0x406);
    return -1;
  }
  return (((int64_t)pg * Hkv + hkv) * pr.page_tokens + t % pr.page_tokens) * kHeadDim;
}

template <typename CsT, bool PAGED = false>
__global__ void qkv_norm_rope_kernel(
    const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ qw,
    const __nv_bfloat16* __restrict__ kw, const CsT* __restrict__ cosp,
    const CsT* __restrict__ sinp, int cs_use_pos, int64_t cs_offset, int64_t cs_stride_b,
    __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_out,
    __nv_bfloat16* __restrict__ v_out, __nv_bfloat16* __restrict__ k_cache,
    __nv_bfloat16* __restrict__ v_cache, int B, int S, int Hq, int Hkv, int64_t start_pos,
    const int32_t* __restrict__ pos_dev, int64_t max_seq, float eps, PageRef pr) {
  // dependents first: decode attention streams the cache rows of earlier
  // steps before its own wait, and waits for this kernel before it reads q
  // or the newest row
  pdl_launch();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int heads = Hq + 2 * Hkv;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= (int64_t)B * S * heads) return;
  const int64_t tok = row / heads;
  const int h = (int)(row - tok * heads);
  const int b = (int)(tok / S);
  const int s = (int)(tok - (int64_t)b * S);
  const int64_t pos = pos_dev ? (int64_t)(*pos_dev) : start_pos;
  const int d0 = lane * 4;

  float v[4];
  load4_bf16(qkv + row * kHeadDim + d0, v);

  if (h >= Hq + Hkv) {  // value head: straight copy
    const int hv = h - Hq - Hkv;
    if (v_out) store4_bf16(v_out + (((int64_t)b * Hkv + hv) * S + s) * kHeadDim + d0, v);
    if constexpr (PAGED) {
      const int64_t off = page_row(pr, b, hv, Hkv, pos + s);
      if (off >= 0) store4_bf16(v_cache + off + d0, v);
    } else {
      if (v_cache)
        store4_bf16(v_cache + (((int64_t)b * Hkv + hv) * max_seq + pos + s) * kHeadDim + d0, v);
    }
    return;
  }
  const bool is_q = h < Hq;
  const __nv_bfloat16* w = is_q ? qw : kw;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss * (1.0f / kHeadDim) + eps);  // IEEE, as torch.rsqrt on CPU
  float wv[4];
  load4_bf16(w + d0, wv);
  float n[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = rbf(rbf(v[i] * r) * wv[i]);

  const int64_t cs_row = cs_use_pos * pos + cs_offset + (int64_t)b * cs_stride_b + s;
  const int j0 = d0 & 63;
  float c[4], sn[4];
  load4_cs<CsT>(cosp + cs_row * 64 + j0, c);
  load4_cs<CsT>(sinp + cs_row * 64 + j0, sn);
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float p = __shfl_xor_sync(0xffffffffu, n[i], 16);
    const float rot = (lane < 16) ? -p : p;
    o[i] = rbf(rbf(n[i] * c[i]) + rbf(rot * sn[i]));
  }
  if (is_q) {
    if (q_out) store4_bf16(q_out + (((int64_t)b * Hq + h) * S + s) * kHeadDim + d0, o);
  } else {
    const int hk = h - Hq;
    if (k_out) store4_bf16(k_out + (((int64_t)b * Hkv + hk) * S + s) * kHeadDim + d0, o);
    if constexpr (PAGED) {
      const int64_t off = page_row(pr, b, hk, Hkv, pos + s);
      if (off >= 0) store4_bf16(k_cache + off + d0, o);
    } else {
      if (k_cache)
        store4_bf16(k_cache + (((int64_t)b * Hkv + hk) * max_seq + pos + s) * kHeadDim + d0, o);
    }
  }
}

}  // namespace q3

extern "C" int q3_rope(const void* x, const float* cos_sin, void* out, int64_t seq, int heads,
                       int head_dim, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(x && cos_sin && out, "q3_rope: null pointer");
  Q3_REQUIRE(head_dim == kHeadDim, "q3_rope: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(seq >= 0 && heads > 0, "q3_rope: bad shape");
  Q3_REQUIRE(aligned(x, 8) && aligned(out, 8) && aligned(cos_sin, 16), "q3_rope: misaligned");
  const int64_t rows = seq * heads;
  if (rows == 0) return Q3_OK;
  return launch_ex(rope_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0,
                   (cudaStream_t)stream, 1, (const __nv_bfloat16*)x, cos_sin,
                   (__nv_bfloat16*)out, seq, heads);
}

extern "C" int q3_mrope_cos_sin(const int64_t* pos, const float* inv_freq, int64_t n_tok,
                                int head_dim, int sec_h, int sec_w, float* cos_out,
                                float* sin_out, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(pos && inv_freq && cos_out && sin_out, "q3_mrope_cos_sin: null pointer");
  Q3_REQUIRE(head_dim > 0 && head_dim % 2 == 0 && n_tok >= 0, "q3_mrope_cos_sin: bad shape");
  Q3_REQUIRE(sec_h >= 0 && sec_w >= 0 && 3 * sec_h <= head_dim / 2 + 2 &&
                 3 * sec_w <= head_dim / 2 + 2,
             "q3_mrope_cos_sin: mrope sections exceed head_dim/2");
  const int half = head_dim / 2;
  const int64_t total = n_tok * half;
  if (total == 0) return Q3_OK;
  return launch_ex(mrope_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0,
                   (cudaStream_t)stream, 1, pos, inv_freq, n_tok, half, sec_h, sec_w, cos_out,
                   sin_out);
}

extern "C" int q3_qkv_norm_rope(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                                const void* cos, const void* sin, int cs_dtype, int cs_use_pos,
                                int64_t cs_offset, int64_t cs_stride_b, void* q_out,
                                void* k_out, void* v_out,
                                void* k_cache, void* v_cache, int B, int S, int Hq, int Hkv,
                                int head_dim, int64_t start_pos, const int32_t* pos_dev,
                                int64_t max_seq, float eps, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(qkv && q_norm_w && k_norm_w && cos && sin, "q3_qkv_norm_rope: null input");
  Q3_REQUIRE(head_dim == kHeadDim, "q3_qkv_norm_rope: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(B >= 0 && S >= 0 && Hq > 0 && Hkv > 0, "q3_qkv_norm_rope: bad shape");
  Q3_REQUIRE(cs_dtype == Q3_F32 || cs_dtype == Q3_BF16, "q3_qkv_norm_rope: bad cs_dtype");
  Q3_REQUIRE(!(k_cache || v_cache) || (pos_dev || start_pos + S <= max_seq),
             "q3_qkv_norm_rope: positions %lld..%lld exceed max_seq %lld", (long long)start_pos,
             (long long)(start_pos + S - 1), (long long)max_seq);
  Q3_REQUIRE(aligned(qkv, 8) && (!q_out || aligned(q_out, 8)) && (!k_out || aligned(k_out, 8)) &&
                 (!v_out || aligned(v_out, 8)) && (!k_cache || aligned(k_cache, 8)) &&
                 (!v_cache || aligned(v_cache, 8)) &&
                 aligned(cos, cs_dtype == Q3_F32 ? 16 : 8) &&
                 aligned(sin, cs_dtype == Q3_F32 ? 16 : 8),
             "q3_qkv_norm_rope: misaligned pointer");
  const int64_t rows = (int64_t)B * S * (Hq + 2 * Hkv);
  if (rows == 0) return Q3_OK;
  dim3 grid((unsigned)((rows + 7) / 8)), block(256);
  cudaStream_t st = (cudaStream_t)stream;
  if (cs_dtype == Q3_BF16)
    return launch_ex(qkv_norm_rope_kernel<__nv_bfloat16>, grid, block, 0, st, 1,
        (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)q_norm_w, (const __nv_bfloat16*)k_norm_w,
        (const __nv_bfloat16*)cos, (const __nv_bfloat16*)sin, cs_use_pos, cs_offset, cs_stride_b,
        (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out,
        (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, B, S, Hq, Hkv, start_pos, pos_dev,
        max_seq, eps, PageRef{});
  else
    return launch_ex(qkv_norm_rope_kernel<float>, grid, block, 0, st, 1,
        (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)q_norm_w, (const __nv_bfloat16*)k_norm_w,
        (const float*)cos, (const float*)sin, cs_use_pos, cs_offset, cs_stride_b,
        (__nv_bfloat16*)q_out,
        (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out, (__nv_bfloat16*)k_cache,
        (__nv_bfloat16*)v_cache, B, S, Hq, Hkv, start_pos, pos_dev, max_seq, eps, PageRef{});
}

extern "C" int q3_qkv_norm_rope_paged(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                                      const void* cos, const void* sin, int cs_dtype,
                                      int cs_use_pos, int64_t cs_offset, int64_t cs_stride_b,
                                      void* q_out, void* k_pages, void* v_pages, int B, int S,
                                      int Hq, int Hkv, int head_dim, int64_t start_pos,
                                      const int32_t* pos_dev, const int32_t* block_table,
                                      int64_t table_stride, int page_tokens, int num_pages,
                                      float eps, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(qkv && q_norm_w && k_norm_w && cos && sin && k_pages && v_pages && block_table,
             "q3_qkv_norm_rope_paged: null input");
  Q3_REQUIRE(head_dim == kHeadDim, "q3_qkv_norm_rope_paged: head_dim must be 128 (got %d)",
             head_dim);
  Q3_REQUIRE(B >= 0 && S >= 0 && Hq > 0 && Hkv > 0 && table_stride > 0 && page_tokens > 0 &&
                 num_pages > 0,
             "q3_qkv_norm_rope_paged: bad shape");
  Q3_REQUIRE(cs_dtype == Q3_F32 || cs_dtype == Q3_BF16, "q3_qkv_norm_rope_paged: bad cs_dtype");
  Q3_REQUIRE(pos_dev || start_pos + S <= table_stride * page_tokens,
             "q3_qkv_norm_rope_paged: positions %lld..%lld beyond the table width",
             (long long)start_pos, (long long)(start_pos + S - 1));
  Q3_REQUIRE(aligned(qkv, 8) && (!q_out || aligned(q_out, 8)) && aligned(k_pages, 8) &&
                 aligned(v_pages, 8) && aligned(block_table, 4) &&
                 aligned(cos, cs_dtype == Q3_F32 ? 16 : 8) &&
                 aligned(sin, cs_dtype == Q3_F32 ? 16 : 8),
             "q3_qkv_norm_rope_paged: misaligned pointer");
  const int64_t rows = (int64_t)B * S * (Hq + 2 * Hkv);
  if (rows == 0) return Q3_OK;
  dim3 grid((unsigned)((rows + 7) / 8)), block(256);
  cudaStream_t st = (cudaStream_t)stream;
  const PageRef pr{block_table, table_stride, page_tokens, num_pages, device_error_word()};
  if (cs_dtype == Q3_BF16)
    return launch_ex(qkv_norm_rope_kernel<__nv_bfloat16, true>, grid, block, 0, st, 1,
        (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)q_norm_w, (const __nv_bfloat16*)k_norm_w,
        (const __nv_bfloat16*)cos, (const __nv_bfloat16*)sin, cs_use_pos, cs_offset, cs_stride_b,
        (__nv_bfloat16*)q_out, (__nv_bfloat16*)nullptr, (__nv_bfloat16*)nullptr,
        (__nv_bfloat16*)k_pages, (__nv_bfloat16*)v_pages, B, S, Hq, Hkv, start_pos, pos_dev,
        (int64_t)0, eps, pr);
  return launch_ex(qkv_norm_rope_kernel<float, true>, grid, block, 0, st, 1,
      (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)q_norm_w, (const __nv_bfloat16*)k_norm_w,
      (const float*)cos, (const float*)sin, cs_use_pos, cs_offset, cs_stride_b,
      (__nv_bfloat16*)q_out, (__nv_bfloat16*)nullptr, (__nv_bfloat16*)nullptr,
      (__nv_bfloat16*)k_pages, (__nv_bfloat16*)v_pages, B, S, Hq, Hkv, start_pos, pos_dev,
      (int64_t)0, eps, pr);
}
