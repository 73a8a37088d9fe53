// Vision tower kernels other than its linears (which are q3_gemm_bias):
// LayerNorm, bilinear position embeddings, the 2-D vision RoPE and
// frame-local (varlen, non-causal) attention at head_dim 72.
//
// Reference: the reference runs transformers' Qwen3VLVisionModel eagerly
// (vision.py:51-53, :74-76); the steps follow transformers 5.5.0
// modeling_qwen3_vl.py:
//   LayerNorm           nn.LayerNorm(eps 1e-6) of Qwen3VLVisionBlock :268-269 and
//                       Qwen3VLVisionPatchMerger :113
//   position embedding  Qwen3VLVisionModel.fast_pos_embed_interpolate :702-763
//   vision RoPE         rot_pos_emb :662-700, apply_rotary_pos_emb_vision :131-142
//   attention           Qwen3VLVisionAttention.forward :196-262 (softmax(q k^T
//                       / sqrt(72)) v within each frame; cu_seqlens :793-801)
//
// Token order.  The tower keeps patches in merge-block order: for an image of
// t frames and an h x w patch grid (merge m), token i of a frame is block
// i / m^2 (row-major over the (h/m) x (w/m) blocks) and inside it row
// (i % m^2) / m, column i % m.  Every kernel maps a token to (image, frame,
// row, column) through a small per-image table built on the host from
// grid_thw (which the reference also reads on the host).
#include <math.h>

#include "common.cuh"

namespace q3 {
namespace {

// --------------------------------------------------------------------------
// image table: int32 [n_img][4] = {t, h, w, first token}; tokens of image g
// are [first, first + t*h*w)
// --------------------------------------------------------------------------
struct TokenPos {
  int img, row, col;
};

__device__ __forceinline__ TokenPos locate(const int* __restrict__ imgs, int n_img, int merge,
                                           int n) {
  int lo = 0, hi = n_img;  // largest g with first(g) <= n
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (imgs[4 * mid + 3] <= n) lo = mid; else hi = mid;
  }
  const int h = imgs[4 * lo + 1], w = imgs[4 * lo + 2];
  const int i = (n - imgs[4 * lo + 3]) % (h * w);
  const int mm = merge * merge;
  const int blk = i / mm, in = i - blk * mm;
  const int bw = w / merge;
  const int br = blk / bw, bc = blk - br * bw;
  return {lo, br * merge + in / merge, bc * merge + in % merge};
}

// ---------------------------------------------------------------- LayerNorm
// One warp per row; fp32 mean and variance (two passes over the row, which
// stays in L1), y = bf16((x - mean) * rstd * w + b).
__global__ void __launch_bounds__(256) layernorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                        const __nv_bfloat16* __restrict__ w,
                                                        const __nv_bfloat16* __restrict__ b,
                                                        __nv_bfloat16* __restrict__ y,
                                                        int64_t rows, int cols, float eps) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * cols);
  const int nv = cols >> 3;
  float s = 0.f;
  for (int v = lane; v < nv; v += 32) {
    const uint4 u = xr[v];
    const uint32_t ws[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(ws[i]);
      s += f.x + f.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)cols;
  float q = 0.f;
  for (int v = lane; v < nv; v += 32) {
    const uint4 u = xr[v];
    const uint32_t ws[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(ws[i]);
      const float a = f.x - mean, c = f.y - mean;
      q += a * a + c * c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = 1.0f / sqrtf(q / (float)cols + eps);
  uint4* yr = reinterpret_cast<uint4*>(y + row * cols);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  const uint4* bv = reinterpret_cast<const uint4*>(b);
  for (int v = lane; v < nv; v += 32) {
    const uint4 u = xr[v], g = wv[v], c = bv[v];
    const uint32_t xs[4] = {u.x, u.y, u.z, u.w}, gs[4] = {g.x, g.y, g.z, g.w},
                   cs[4] = {c.x, c.y, c.z, c.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(xs[i]), gw = unpack_bf16x2(gs[i]), bb = unpack_bf16x2(cs[i]);
      o[i] = pack_bf16x2((f.x - mean) * rstd * gw.x + bb.x, (f.y - mean) * rstd * gw.y + bb.y);
    }
    yr[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ------------------------------------------------------- position embedding
// Token (row r, col c) of an h x w grid samples the side x side learned grid
// bilinearly at (linspace(0, side-1, h)[r], linspace(0, side-1, w)[c]).
// linspace element k of n (start 0): step*k below n/2, and from there on
// end - step*(n-1-k) with one rounding (a fused multiply-add): the form of
// torch's CPU linspace, where the reference computes these indices.
// Corner weights are fp32 products rounded to bf16; each corner term
// bf16(table * weight) and the running sum round to bf16, in the order
// (floor,floor) + (floor,ceil) + (ceil,floor) + (ceil,ceil).
__device__ __forceinline__ float linspace_at(int k, int n, float end) {
  if (n == 1) return 0.f;
  const float step = __fdiv_rn(end, (float)(n - 1));
  return k < n / 2 ? __fmul_rn(step, (float)k) : __fmaf_rn(-step, (float)(n - 1 - k), end);
}

__global__ void __launch_bounds__(256) pos_embed_kernel(const __nv_bfloat16* __restrict__ table,
                                                        int side, int hidden,
                                                        const int* __restrict__ imgs, int n_img,
                                                        int merge, int64_t n_tok,
                                                        __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (n >= n_tok) return;
  const TokenPos tp = locate(imgs, n_img, merge, (int)n);
  const int h = imgs[4 * tp.img + 1], w = imgs[4 * tp.img + 2];
  const float end = (float)(side - 1);
  const float hi = linspace_at(tp.row, h, end), wi = linspace_at(tp.col, w, end);
  const int h0 = (int)hi, w0 = (int)wi;
  const int h1 = min(h0 + 1, side - 1), w1 = min(w0 + 1, side - 1);
  const float dh = __fsub_rn(hi, (float)h0), dw = __fsub_rn(wi, (float)w0);
  const float eh = __fsub_rn(1.f, dh), ew = __fsub_rn(1.f, dw);
  const float wt[4] = {rbf(__fmul_rn(eh, ew)), rbf(__fmul_rn(eh, dw)), rbf(__fmul_rn(dh, ew)),
                       rbf(__fmul_rn(dh, dw))};
  const uint4* src[4] = {reinterpret_cast<const uint4*>(table + (int64_t)(h0 * side + w0) * hidden),
                         reinterpret_cast<const uint4*>(table + (int64_t)(h0 * side + w1) * hidden),
                         reinterpret_cast<const uint4*>(table + (int64_t)(h1 * side + w0) * hidden),
                         reinterpret_cast<const uint4*>(table + (int64_t)(h1 * side + w1) * hidden)};
  uint4* dst = reinterpret_cast<uint4*>(out + n * hidden);
  for (int v = lane; v < (hidden >> 3); v += 32) {
    float acc[8];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 u = src[c][v];
      const uint32_t ws[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(ws[i]);
        const float t0 = rbf(__fmul_rn(f.x, wt[c])), t1 = rbf(__fmul_rn(f.y, wt[c]));
        acc[2 * i] = c ? rbf(__fadd_rn(acc[2 * i], t0)) : t0;
        acc[2 * i + 1] = c ? rbf(__fadd_rn(acc[2 * i + 1], t1)) : t1;
      }
    }
    dst[v] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                        pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
  }
}

// ------------------------------------------------------------- vision RoPE
// In place on the packed qkv [n_tok, 3 * heads * 72] (q heads, k heads, v
// heads): for d < 36, angle e_d = row * inv_freq[d] (d < 18) or col *
// inv_freq[d - 18]; out[d] = x[d] cos e_d - x[d+36] sin e_d and out[d+36] =
// x[d+36] cos e_d + x[d] sin e_d, in fp32 (separately rounded products and
// sum), then bf16.  One warp per (token, head, q|k); lanes 0..35 own a pair.
constexpr int kVisHd = 72;

__global__ void __launch_bounds__(256) vision_rope_kernel(__nv_bfloat16* __restrict__ qkv,
                                                          int heads, const float* __restrict__ inv,
                                                          const int* __restrict__ imgs, int n_img,
                                                          int merge, int64_t n_tok) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const int64_t job = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (job >= n_tok * heads * 2) return;
  const int64_t n = job / (heads * 2);
  const int rest = (int)(job - n * heads * 2);
  const int which = rest / heads, h = rest - which * heads;  // which: 0 q, 1 k
  const TokenPos tp = locate(imgs, n_img, merge, (int)n);
  const int width = 3 * heads * kVisHd;
  __nv_bfloat16* x = qkv + n * width + which * heads * kVisHd + h * kVisHd;
  for (int d = lane; d < kVisHd / 2; d += 32) {
    const float pos = (float)(d < 18 ? tp.row : tp.col);
    const float e = __fmul_rn(pos, inv[d < 18 ? d : d - 18]);
    const float c = cosf(e), s = sinf(e);
    const float a = bf2f(x[d]), b = bf2f(x[d + kVisHd / 2]);
    const float lo = __fadd_rn(__fmul_rn(a, c), __fmul_rn(-b, s));
    const float hi = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
    x[d] = f2bf(lo);
    x[d + kVisHd / 2] = f2bf(hi);
  }
}

// ---------------------------------------------------- frame-local attention
// Flash-style (online softmax in fp32) non-causal attention inside each frame.
// One CTA = 8 warps = 128 query rows of one (frame, head); 64-key K/V tiles
// double-buffered with cp.async into XOR-swizzled rows of 256 bytes, of which
// dims 0..71 are loaded and 72..79 zero-filled so Q K^T runs as 5 k-steps of
// mma.sync m16n8k16 and P V as 10 output tiles of 8 (the 10th is discarded).
constexpr int kVBM = 128, kVBN = 64, kVThreads = 256;
constexpr int kVChunks = 9;        // 16-byte chunks of a 72-dim row
constexpr int kVKSteps = 5;        // 80 padded dims / 16
constexpr int kVSmem = (kVBM + 4 * kVBN) * 256;  // Q + 2 x (K, V) = 96 KB

__device__ __forceinline__ void vcp16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void vcommit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void vwait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void vldsm(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void vldsm_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void vmma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                     uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t vswz(int r, int c) { return r * 256 + ((c ^ (r & 7)) << 4); }

// rows [0, rows) of a 72-dim tile (global row stride ld elements) into smem;
// rows >= valid and dims 72..79 are zero-filled
__device__ __forceinline__ void vload_tile(uint32_t smem, const __nv_bfloat16* g, int64_t ld,
                                           int rows, int valid) {
  for (int i = threadIdx.x; i < rows * (kVChunks + 1); i += kVThreads) {
    const int r = i / (kVChunks + 1), c = i - r * (kVChunks + 1);
    const bool ok = r < valid && c < kVChunks;
    const __nv_bfloat16* src = ok ? g + r * ld + c * 8 : g;
    vcp16(smem + vswz(r, c), src, ok);
  }
}

struct VisAttnParams {
  const __nv_bfloat16* qkv;  // [n_tok, 3 * heads * 72]
  __nv_bfloat16* out;        // [n_tok, heads * 72]
  const int* blocks;         // [n_blocks][3] = {frame first token, frame length, q0}
  int heads;
  float scale_log2;
};

__global__ void __launch_bounds__(kVThreads, 1) vision_attn_kernel(VisAttnParams p) {
  pdl_wait();
  pdl_launch();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t sQ = smem_u32(smem_raw);
  const uint32_t sK0 = sQ + kVBM * 256;
  const uint32_t sV0 = sK0 + 2 * kVBN * 256;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;

  const int* blk = p.blocks + 3 * blockIdx.x;
  const int64_t f0 = blk[0];
  const int flen = blk[1], q0 = blk[2];
  const int h = blockIdx.y;
  const int q_valid = min(kVBM, flen - q0);
  const int hidden = p.heads * kVisHd;
  const int64_t ld = 3 * (int64_t)hidden;
  const int n_kb = (flen + kVBN - 1) / kVBN;

  const __nv_bfloat16* qg = p.qkv + (f0 + q0) * ld + h * kVisHd;
  const __nv_bfloat16* kg = p.qkv + f0 * ld + hidden + h * kVisHd;
  const __nv_bfloat16* vg = p.qkv + f0 * ld + 2 * hidden + h * kVisHd;

  vload_tile(sQ, qg, ld, kVBM, q_valid);
  {
    const int valid = min(kVBN, flen);
    vload_tile(sK0, kg, ld, kVBN, valid);
    vload_tile(sV0, vg, ld, kVBN, valid);
  }
  vcommit();

  uint32_t qf[kVKSteps][4];
  float o[10][4];
#pragma unroll
  for (int i = 0; i < 10; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

  for (int kb = 0; kb < n_kb; ++kb) {
    const int st = kb & 1;
    if (kb + 1 < n_kb) {
      const int k0 = (kb + 1) * kVBN;
      const int valid = min(kVBN, flen - k0);
      vload_tile(sK0 + (st ^ 1) * kVBN * 256, kg + (int64_t)k0 * ld, ld, kVBN, valid);
      vload_tile(sV0 + (st ^ 1) * kVBN * 256, vg + (int64_t)k0 * ld, ld, kVBN, valid);
      vcommit();
      vwait<1>();
    } else {
      vwait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < kVKSteps; ++ks) {
        const int r = warp * 16 + (lane & 15);
        const int c = ks * 2 + (lane >> 4);
        vldsm(qf[ks], sQ + vswz(r, c));
      }
    }
    const uint32_t sK = sK0 + st * kVBN * 256;
    const uint32_t sV = sV0 + st * kVBN * 256;

    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kVKSteps; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t kf[4];
        const int r = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks * 2 + ((lane >> 3) & 1);
        vldsm(kf, sK + vswz(r, c));
        vmma(s[2 * jp], qf[ks], kf[0], kf[1]);
        vmma(s[2 * jp + 1], qf[ks], kf[2], kf[3]);
      }
    }
    const int kbase = kb * kVBN;
    const bool need_mask = kbase + kVBN > flen;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[j][e] * p.scale_log2;
        if (need_mask && kbase + j * 8 + 2 * t4 + (e & 1) >= flen) x = -INFINITY;
        s[j][e] = x;
      }
    }
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
      corr[r] = exp2f(m_r[r] - base_m[r]);
      m_r[r] = mx[r];
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pf[4][4];
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
    for (int i = 0; i < 10; ++i) {
      o[i][0] *= corr[0]; o[i][1] *= corr[0];
      o[i][2] *= corr[1]; o[i][3] *= corr[1];
    }
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int ip = 0; ip < 5; ++ip) {
        uint32_t vf[4];
        const int r = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = ip * 2 + (lane >> 4);
        vldsm_t(vf, sV + vswz(r, c));
        vmma(o[2 * ip], pf[ks], vf[0], vf[1]);
        vmma(o[2 * ip + 1], pf[ks], vf[2], vf[3]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
  const float inv0 = l_r[0] > 0.f ? 1.f / l_r[0] : 0.f;
  const float inv1 = l_r[1] > 0.f ? 1.f / l_r[1] : 0.f;
  const int row0 = warp * 16 + g8;
  __nv_bfloat16* ob = p.out + (f0 + q0) * hidden + h * kVisHd;
#pragma unroll
  for (int i = 0; i < 9; ++i) {
    const int d = i * 8 + 2 * t4;
    if (row0 < q_valid)
      *reinterpret_cast<uint32_t*>(ob + (int64_t)row0 * hidden + d) =
          pack_bf16x2(o[i][0] * inv0, o[i][1] * inv0);
    if (row0 + 8 < q_valid)
      *reinterpret_cast<uint32_t*>(ob + (int64_t)(row0 + 8) * hidden + d) =
          pack_bf16x2(o[i][2] * inv1, o[i][3] * inv1);
  }
}

}  // namespace
}  // namespace q3

extern "C" int q3_layernorm(const void* x, const void* w, const void* b, void* y, int64_t rows,
                            int64_t cols, float eps, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(x && w && b && y, "q3_layernorm: null pointer");
  Q3_REQUIRE(rows >= 0 && cols > 0 && cols % 8 == 0 && cols < (1 << 24),
             "q3_layernorm: cols=%lld must be a positive multiple of 8", (long long)cols);
  Q3_REQUIRE(aligned(x, 16) && aligned(w, 16) && aligned(b, 16) && aligned(y, 16),
             "q3_layernorm: pointers must be 16-byte aligned");
  if (rows == 0) return Q3_OK;
  return launch_ex(layernorm_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0,
                   (cudaStream_t)stream, 1, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w,
                   (const __nv_bfloat16*)b, (__nv_bfloat16*)y, rows, (int)cols, eps);
}

// Host-side check of the image table: every image fits the merge grid and the
// first tokens are the running sums of t*h*w.
static int check_images(const char* fn, const int* imgs_host, int n_img, int merge,
                        int64_t n_tok) {
  using namespace q3;
  int64_t first = 0;
  for (int g = 0; g < n_img; ++g) {
    const int t = imgs_host[4 * g], h = imgs_host[4 * g + 1], w = imgs_host[4 * g + 2];
    Q3_REQUIRE(t > 0 && h > 0 && w > 0 && h % merge == 0 && w % merge == 0,
               "%s: image %d grid (%d, %d, %d) does not fit merge %d", fn, g, t, h, w, merge);
    Q3_REQUIRE(imgs_host[4 * g + 3] == first, "%s: image %d starts at token %d, expected %lld",
               fn, g, imgs_host[4 * g + 3], (long long)first);
    first += (int64_t)t * h * w;
  }
  Q3_REQUIRE(first == n_tok, "%s: images hold %lld tokens, n_tok=%lld", fn, (long long)first,
             (long long)n_tok);
  return Q3_OK;
}

extern "C" int q3_vision_pos_embed(const void* table, int side, int hidden, const int32_t* imgs,
                                   const int32_t* imgs_host, int n_img, int merge, int64_t n_tok,
                                   void* out, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(table && imgs && imgs_host && out, "q3_vision_pos_embed: null pointer");
  Q3_REQUIRE(side > 0 && hidden > 0 && hidden % 8 == 0 && n_img > 0 && merge > 0 && n_tok > 0 &&
                 n_tok < (1ll << 31),
             "q3_vision_pos_embed: bad shape");
  Q3_REQUIRE(aligned(table, 16) && aligned(out, 16) && aligned(imgs, 4),
             "q3_vision_pos_embed: misaligned pointer");
  int rc = check_images("q3_vision_pos_embed", imgs_host, n_img, merge, n_tok);
  if (rc) return rc;
  return launch_ex(pos_embed_kernel, dim3((unsigned)((n_tok + 7) / 8)), dim3(256), 0,
                   (cudaStream_t)stream, 1, (const __nv_bfloat16*)table, side, hidden, imgs,
                   n_img, merge, n_tok, (__nv_bfloat16*)out);
}

extern "C" int q3_vision_rope(void* qkv, int heads, int head_dim, const float* inv_freq,
                              const int32_t* imgs, const int32_t* imgs_host, int n_img, int merge,
                              int64_t n_tok, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(qkv && inv_freq && imgs && imgs_host, "q3_vision_rope: null pointer");
  Q3_REQUIRE(head_dim == kVisHd, "q3_vision_rope: head_dim must be 72 (got %d)", head_dim);
  Q3_REQUIRE(heads > 0 && n_img > 0 && merge > 0 && n_tok > 0 && n_tok < (1ll << 31),
             "q3_vision_rope: bad shape");
  int rc = check_images("q3_vision_rope", imgs_host, n_img, merge, n_tok);
  if (rc) return rc;
  const int64_t jobs = n_tok * heads * 2;
  return launch_ex(vision_rope_kernel, dim3((unsigned)((jobs + 7) / 8)), dim3(256), 0,
                   (cudaStream_t)stream, 1, (__nv_bfloat16*)qkv, heads, inv_freq, imgs, n_img,
                   merge, n_tok);
}

extern "C" int q3_vision_attention(const void* qkv, void* out, int heads, int head_dim,
                                   const int32_t* blocks, const int32_t* blocks_host,
                                   int n_blocks, int64_t n_tok, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(qkv && out && blocks && blocks_host, "q3_vision_attention: null pointer");
  Q3_REQUIRE(head_dim == kVisHd, "q3_vision_attention: head_dim must be 72 (got %d)", head_dim);
  Q3_REQUIRE(heads > 0 && heads < 65536 && n_blocks > 0 && n_tok > 0 && n_tok < (1ll << 31),
             "q3_vision_attention: bad shape");
  Q3_REQUIRE(aligned(qkv, 16) && aligned(out, 4) && aligned(blocks, 4),
             "q3_vision_attention: misaligned pointer");
  for (int i = 0; i < n_blocks; ++i) {
    const int64_t f0 = blocks_host[3 * i], len = blocks_host[3 * i + 1], q0 = blocks_host[3 * i + 2];
    Q3_REQUIRE(f0 >= 0 && len > 0 && f0 + len <= n_tok && q0 >= 0 && q0 < len && q0 % 128 == 0,
               "q3_vision_attention: block %d (frame %lld + %lld, rows from %lld) is not a "
               "128-row block of a frame inside the %lld tokens", i, (long long)f0,
               (long long)len, (long long)q0, (long long)n_tok);
  }
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    Q3_CUDA_CHECK(cudaFuncSetAttribute(vision_attn_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kVSmem));
    attr_set[dev] = true;
  }
  VisAttnParams p;
  p.qkv = (const __nv_bfloat16*)qkv;
  p.out = (__nv_bfloat16*)out;
  p.blocks = blocks;
  p.heads = heads;
  p.scale_log2 = (1.0f / sqrtf((float)kVisHd)) * 1.4426950408889634f;
  return launch_ex(vision_attn_kernel, dim3((unsigned)n_blocks, (unsigned)heads),
                   dim3(kVThreads), kVSmem, (cudaStream_t)stream, 1, p);
}
