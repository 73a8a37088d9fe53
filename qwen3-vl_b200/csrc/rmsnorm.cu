// a1: RMSNorm with optional fused residual add.
//
// Follows RMSNorm.forward (model_fused.py:37-40):
//   h  = x (+ add, rounded to bf16 like the torch bf16 add of :269/:275)
//   y  = bf16( bf16(h * rsqrt(mean(h^2) + eps)) * w )
// One warp per row; rows of up to 4096 elements stay in registers so the row
// is read from HBM once (HBM-bound: 2 bytes read + 2 written per element, plus
// 2 more read and written when the residual add is fused).
#include "common.cuh"

namespace q3 {

template <int kVecs>  // uint4 vectors (8 bf16) per lane; 0 = generic loop
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ add,
                                                      __nv_bfloat16* __restrict__ h_out,
                                                      const __nv_bfloat16* __restrict__ w,
                                                      __nv_bfloat16* __restrict__ y, int64_t rows,
                                                      int hidden, float eps) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * hidden);
  const uint4* ar = add ? reinterpret_cast<const uint4*>(add + row * hidden) : nullptr;
  uint4* hr = h_out ? reinterpret_cast<uint4*>(h_out + row * hidden) : nullptr;
  uint4* yr = reinterpret_cast<uint4*>(y + row * hidden);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  const int nvec = hidden >> 3;

  auto load_h = [&](int v) -> uint4 {
    uint4 a = xr[v];
    if (ar) {
      uint4 b = ar[v];
      uint32_t* pa = reinterpret_cast<uint32_t*>(&a);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 fa = unpack_bf16x2(pa[i]), fb = unpack_bf16x2(pb[i]);
        pa[i] = pack_bf16x2(fa.x + fb.x, fa.y + fb.y);
      }
      if (hr) hr[v] = a;
    }
    return a;
  };
  auto sumsq = [](const uint4& a) -> float {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(&a);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = unpack_bf16x2(p[i]);
      s = fmaf(f.x, f.x, s);
      s = fmaf(f.y, f.y, s);
    }
    return s;
  };
  auto norm_store = [&](int v, const uint4& a, float r) {
    uint4 wv = wr[v];
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wv);
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = unpack_bf16x2(pa[i]), g = unpack_bf16x2(pw[i]);
      po[i] = pack_bf16x2(rbf(f.x * r) * g.x, rbf(f.y * r) * g.y);
    }
    yr[v] = o;
  };

  if constexpr (kVecs > 0) {
    uint4 buf[kVecs];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kVecs; ++i) {
      buf[i] = load_h(lane + 32 * i);
      ss += sumsq(buf[i]);
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / (float)hidden + eps);
#pragma unroll
    for (int i = 0; i < kVecs; ++i) norm_store(lane + 32 * i, buf[i], r);
  } else {
    float ss = 0.f;
    for (int v = lane; v < nvec; v += 32) ss += sumsq(load_h(v));
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / (float)hidden + eps);
    // second pass re-reads h (from h_out when the add was fused)
    for (int v = lane; v < nvec; v += 32) {
      uint4 a = hr ? hr[v] : xr[v];
      if (ar && !hr) {
        // recompute the rounded sum when h was not materialised
        uint4 b = ar[v];
        uint32_t* pa = reinterpret_cast<uint32_t*>(&a);
        const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float2 fa = unpack_bf16x2(pa[i]), fb = unpack_bf16x2(pb[i]);
          pa[i] = pack_bf16x2(fa.x + fb.x, fa.y + fb.y);
        }
      }
      norm_store(v, a, r);
    }
  }
}

}  // namespace q3

extern "C" int q3_rmsnorm(const void* x, const void* add, void* h_out, const void* w, void* y,
                          int64_t rows, int64_t hidden, float eps, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(x && w && y, "q3_rmsnorm: null pointer");
  Q3_REQUIRE(rows >= 0 && hidden > 0 && hidden % 8 == 0 && hidden <= (1 << 20),
             "q3_rmsnorm: hidden=%lld must be a positive multiple of 8", (long long)hidden);
  Q3_REQUIRE(aligned(x, 16) && aligned(w, 16) && aligned(y, 16) && (!add || aligned(add, 16)) &&
                 (!h_out || aligned(h_out, 16)),
             "q3_rmsnorm: pointers must be 16-byte aligned");
  if (rows == 0) return Q3_OK;
  const int warps = 8;
  dim3 grid((unsigned)((rows + warps - 1) / warps)), block(32 * warps);
  cudaStream_t s = (cudaStream_t)stream;
  auto X = (const __nv_bfloat16*)x;
  auto A = (const __nv_bfloat16*)add;
  auto H = (__nv_bfloat16*)h_out;
  auto Wt = (const __nv_bfloat16*)w;
  auto Y = (__nv_bfloat16*)y;
  const int hd = (int)hidden;
  if (hidden == 4096)
    return launch_ex(rmsnorm_kernel<16>, grid, block, 0, s, 1, X, A, H, Wt, Y, rows, hd, eps);
  if (hidden == 2048)
    return launch_ex(rmsnorm_kernel<8>, grid, block, 0, s, 1, X, A, H, Wt, Y, rows, hd, eps);
  if (hidden == 1024)
    return launch_ex(rmsnorm_kernel<4>, grid, block, 0, s, 1, X, A, H, Wt, Y, rows, hd, eps);
  return launch_ex(rmsnorm_kernel<0>, grid, block, 0, s, 1, X, A, H, Wt, Y, rows, hd, eps);
}
