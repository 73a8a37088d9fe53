// Persistent decode step: every decoder layer of one greedy decode step in ONE
// kernel launch.
//
// Reference: Qwen3VLDecoderFused.forward_layer (model_fused.py:234-277) at
// S = 1 for every layer of decode_step (model_fused.py:295-300): input
// RMSNorm -> QKV projection -> per-head QK-RMSNorm + RoPE -> KV-cache write ->
// GQA attention over the cache -> o_proj + residual -> post-attention RMSNorm
// -> gate/up + SiLU*up -> down + residual.
//
// Why one kernel: at decode sizes every projection is a weight stream, and a
// kernel boundary costs a few microseconds of ramp and drain during which HBM
// idles.  Here one CTA per SM runs the whole step:
//   * warp 4 (producer) streams every weight tile and K/V tile this CTA will
//     ever need, in order, by TMA into a 10-stage ring.  Weights and the old
//     cache rows never depend on the step's activations, so the producer never
//     waits for other CTAs: HBM streams straight through phase boundaries;
//   * warp 5 (activations) waits for the previous phase of the whole grid (a
//     grid-wide arrival counter, bounded wait), then copies the activation
//     slice of each stage (cp.async), applies the fused RMSNorm where the
//     reference has one, and completes the stage;
//   * warps 0-3 (consumers) run bf16 mma.sync on the staged tiles.
// Work split: each phase's units (64-wide K blocks of 128-row weight tiles, or
// 64-position blocks of a (sequence, KV head) pair) are divided into equal
// contiguous ranges, one per CTA ("stream-K"), so every SM streams the same
// number of bytes.  A tile split across CTAs is reduced by its owner, the CTA
// holding its first units (it meets them last, at the end of its range), which
// waits for the others' arrival counter and sums the partials in CTA order;
// the owner runs the tile's epilogue: QK-norm + RoPE + KV write (one head per
// QKV tile), residual + per-tile sums of squares (o_proj, down), SwiGLU
// (gate/up), or the split-K softmax merge (attention).
// Every wait is bounded; after a timeout the device error word is set and all
// later waits return at once, so a fault unwinds within seconds.
#include <vector>

#include "common.cuh"

namespace q3 {
namespace step {

constexpr int kHD = 128;
constexpr int kRows = 128;        // weight rows per projection tile
constexpr int kBK = 64;           // K elements per stage
constexpr int kStages = 10;
constexpr int kPay = 16384;       // stage payload: 128 rows x 64 K, or 64 positions x 128 dims
constexpr int kAux = 2048;        // stage activations: 16 tokens x 64 K, or the q of one KV head
constexpr int kCons = 4;          // consumer warps
constexpr int kPos = 64;          // positions per attention unit
constexpr int kMaxTok = 16;
constexpr int kMaxTiles = 4096;   // arrival counters (tiles or pairs of one phase)
constexpr int kPhases = 5;
enum { kQKV = 0, kATT = 1, kO = 2, kGU = 3, kDN = 4 };
constexpr int kTileFloats = kRows * kMaxTok;  // fp32 [128 rows][16 tokens]
constexpr int kFullCount = 1 + 32;            // producer arrive.expect_tx + 32 activation lanes
constexpr int kMaxHidden = 8192;              // norm weights staged in shared memory

struct alignas(64) Layer {
  CUtensorMap tm_qkv, tm_o, tm_gu, tm_dn, tm_k, tm_v;
  const __nv_bfloat16* in_norm;
  const __nv_bfloat16* post_norm;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
};

struct Params {
  const Layer* layers;
  int n_layers, M, H, Hq, Hkv, I;
  int64_t max_seq, rope_rows, rope_delta;
  float eps, scale_log2;
  const __nv_bfloat16* cos;  // [rope_rows, 64]
  const __nv_bfloat16* sin;
  const int32_t* kv_len_dev;  // kv_len = pos + 1; the new token is written at pos
  __nv_bfloat16* X;    // [M, H] residual stream (in: layer-0 input, out: last layer)
  __nv_bfloat16* X2;   // [M, H] residual after attention
  __nv_bfloat16* A;    // [M, Hq*128] attention output
  __nv_bfloat16* Q;    // [M, Hq*128] normed, rotated queries
  __nv_bfloat16* act;  // [M, I] SwiGLU output
  float* ss_x;         // [H/128][16] per-tile sums of squares of X
  float* ss_x2;        // [H/128][16] ... of X2
  float* part;         // [C][2][kTileFloats] projection partials
  float* apart;        // [C][2][G * (kHD + 2)] attention partials
  int* cnt;            // [kMaxTiles] arrivals per tile / pair (self-resetting)
  unsigned* bars;      // [1 + kPhases * n_layers] grid arrivals per phase
  unsigned* exit_cnt;
  int* err;
};

// ------------------------------------------------------------------ helpers
__device__ __forceinline__ bool aborted(const int* err) {
  return *reinterpret_cast<const volatile int*>(err) != 0;
}
// mbarrier wait that also gives up as soon as any other wait has timed out
__device__ __forceinline__ bool sw(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 1023u) == 0) {
      if (aborted(err)) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        report_timeout(err, code);
        return false;
      }
    }
  }
  return true;
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Grid-wide phase completion: every CTA adds 1 after its phase work.
__device__ __forceinline__ void grid_arrive(unsigned* bar) {
  __threadfence();
  atomicAdd(bar, 1u);
}
// Called by a whole warp: returns once `target` CTAs have arrived (or on abort).
// One lane per CTA polls, with a short sleep between polls, so the arrivals'
// atomics are not queued behind a storm of loads on the same L2 line.
__device__ __forceinline__ void grid_wait(const unsigned* bar, unsigned target, int* err,
                                          int code) {
  if ((threadIdx.x & 31) == 0) {
    if (ld_acquire_gpu(bar) < target) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_gpu(bar) < target) {
        __nanosleep(40);
        if ((++spins & 63u) == 0) {
          if (aborted(err)) break;
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            report_timeout(err, code);
            break;
          }
        }
      }
    }
  }
  __syncwarp();
  (void)ld_acquire_gpu(bar);  // every lane orders its later reads after the arrivals
}
// The owner of a split tile waits (bounded) until the other `n` contributors
// have published their partials; one thread polls, then resets the counter.
__device__ __forceinline__ void wait_contributors(int* cnt, int n, int* err, int code) {
  if (n <= 0) return;
  const unsigned* cu = reinterpret_cast<const unsigned*>(cnt);
  if ((int)ld_acquire_gpu(cu) < n) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while ((int)ld_acquire_gpu(cu) < n) {
      __nanosleep(32);
      if ((++spins & 63u) == 0) {
        if (aborted(err)) break;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          report_timeout(err, code);
          break;
        }
      }
    }
  }
  *cnt = 0;  // next use of this counter is after a grid-wide phase boundary
}
__device__ __forceinline__ void cons_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kCons * 32) : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// one arrival on `bar` once this thread's earlier cp.async copies have landed
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 rms_scale(uint4 x, float r, uint4 w) {
  uint32_t xs[4] = {x.x, x.y, x.z, x.w};
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(xs[i]), g = unpack_bf16x2(ws[i]);
    xs[i] = pack_bf16x2(rbf(f.x * r) * g.x, rbf(f.y * r) * g.y);
  }
  return make_uint4(xs[0], xs[1], xs[2], xs[3]);
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
// byte offset of 16-byte chunk c (0..15 over 128 dims) of position row r in a
// K or V stage (two 64-dim TMA boxes, 128-byte swizzle)
__device__ __forceinline__ uint32_t kv_off(int r, int c) {
  return (c >> 3) * 8192 + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

// ------------------------------------------------------------ work geometry
struct Geo {
  int U;    // units in the phase
  int KB;   // units per tile (K blocks), or per pair (position blocks)
  int N, K; // projection shape (rows of W, reduction length)
};
__device__ __forceinline__ Geo geo(const Params& p, int ph, int nt) {
  Geo g;
  switch (ph) {
    case kQKV: g.N = (p.Hq + 2 * p.Hkv) * kHD; g.K = p.H; break;
    case kO: g.N = p.H; g.K = p.Hq * kHD; break;
    case kGU: g.N = 2 * p.I; g.K = p.H; break;
    case kDN: g.N = p.H; g.K = p.I; break;
    default: g.N = 0; g.K = 0; break;
  }
  if (ph == kATT) {
    g.KB = nt;
    g.U = p.M * p.Hkv * nt;
  } else {
    g.KB = g.K / kBK;
    g.U = (g.N / kRows) * g.KB;
  }
  return g;
}
// A phase of U units runs on the first min(C, U) CTAs, so every working CTA
// has a non-empty range and the CTAs holding a tile's units are consecutive.
// CTA c owns units [unit_lo(c), unit_lo(c + 1)).
__device__ __forceinline__ int unit_lo(int c, int U, int C) {
  const int Ce = U < C ? U : C;
  return c >= Ce ? U : (int)(((int64_t)c * U) / Ce);
}
// the CTA whose range holds unit u
__device__ __forceinline__ int owner(int u, int U, int C) {
  const int Ce = U < C ? U : C;
  return (int)((((int64_t)u + 1) * Ce - 1) / U);
}
// partial slot of CTA c for tile t: 0 for the first tile of its range, else 1
__device__ __forceinline__ int slot_of(int c, int t, int U, int C, int KB) {
  return (t == unit_lo(c, U, C) / KB) ? 0 : 1;
}

// ------------------------------------------------------------------ kernel
// Warp roles: 0-3 tensor-core consumers, 4 TMA producer, 5 activation stager,
// 6-7 epilogue.  A consumer hands each finished tile segment (fp32 partial
// sums, or per-warp softmax states) to the epilogue warps through one of two
// shared-memory tile buffers and goes straight on with the next stage, so the
// cross-CTA reduction, the epilogue and the global stores never stall the
// weight stream.
constexpr int kWarpProd = kCons;
constexpr int kWarpStage = kCons + 1;
constexpr int kWarpEpi = kCons + 2;
constexpr int kEpiWarps = 2;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kThreadsAll = (kCons + 2 + kEpiWarps) * 32;
constexpr int kTileBufBytes = 8448;  // [128][16] fp32, or [4 warps][4 heads][128] + states

__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads) : "memory");
}

struct Smem {
  uint8_t* pay;
  uint8_t* aux;
  float* tbuf;            // 2 x kTileBufBytes
  __nv_bfloat16* nw;      // norm weights of the current norm phase
  float* r;               // [16] inverse RMS per token
  float* red;             // [kEpiWarps][16]
  int* flag;
  uint64_t *full, *empty, *tfull, *tempty, *phase_ok;
};

// ---- consumers: one projection phase --------------------------------------
template <int NT, bool NORM>
__device__ __forceinline__ bool consume_proj(const Params& p, const Smem& S, const Geo& g,
                                             int u0, int u1, int& it, int& segc, int warp,
                                             int lane) {
  const int g8 = lane >> 2, t4 = lane & 3;
  const uint32_t pay_u = smem_u32(S.pay), aux_u = smem_u32(S.aux), nw_u = smem_u32(S.nw);
  float rr[NT];
#pragma unroll
  for (int n = 0; n < NT; ++n) rr[n] = NORM ? S.r[n * 8 + g8] : 0.f;
  float acc[2][NT][4];
  for (int u = u0; u < u1; ++u) {
    const int kb = u % g.KB;
    if (u == u0 || kb == 0) {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int n = 0; n < NT; ++n)
          acc[mt][n][0] = acc[mt][n][1] = acc[mt][n][2] = acc[mt][n][3] = 0.f;
    }
    const int s = it % kStages;
    const uint32_t par = (it / kStages) & 1;
    ++it;
    if (!sw(&S.full[s], par, p.err, 0x620)) return false;
    const uint32_t wb = pay_u + s * kPay, xb = aux_u + s * kAux;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int cc = 2 * t4 + h;
      uint4 wn = make_uint4(0, 0, 0, 0);
      if (NORM) wn = lds128(nw_u + (kb * kBK + cc * 8) * 2);
      uint4 xv[NT];
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int tok = n * 8 + g8;
        xv[n] = lds128(xb + tok * 128 + ((cc ^ (tok & 7)) << 4));
        if (NORM) xv[n] = rms_scale(xv[n], rr[n], wn);
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const int r0 = warp * 32 + mt * 16 + g8, r1 = r0 + 8;
        const uint4 a0 = lds128(wb + r0 * 128 + ((cc ^ (r0 & 7)) << 4));
        const uint4 a1 = lds128(wb + r1 * 128 + ((cc ^ (r1 & 7)) << 4));
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          mma_bf16_16816(acc[mt][n], a0.x, a1.x, a0.y, a1.y, xv[n].x, xv[n].y);
          mma_bf16_16816(acc[mt][n], a0.z, a1.z, a0.w, a1.w, xv[n].z, xv[n].w);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.empty[s]);
    if (u != u1 - 1 && kb != g.KB - 1) continue;
    // segment ends: hand the partial sums to the epilogue warps
    const int b = segc & 1;
    if (!sw(&S.tempty[b], ((segc >> 1) & 1) ^ 1, p.err, 0x621)) return false;
    ++segc;
    float* tb = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(S.tbuf) + b * kTileBufBytes);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int row = warp * 32 + mt * 16 + g8 + hh * 8;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          const float2 v = n < NT ? make_float2(acc[mt][n < NT ? n : 0][2 * hh],
                                                acc[mt][n < NT ? n : 0][2 * hh + 1])
                                  : make_float2(0.f, 0.f);
          *reinterpret_cast<float2*>(tb + row * kMaxTok + n * 8 + 2 * t4) = v;
        }
      }
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.tfull[b]);
  }
  return true;
}

// ---- consumers: one attention phase ---------------------------------------
template <int G>
__device__ __forceinline__ bool consume_att(const Params& p, const Smem& S, const Geo& g,
                                            int u0, int u1, int nt, int64_t Lold, int& it,
                                            int& segc, int warp, int lane) {
  const int g8 = lane >> 2, t4 = lane & 3;
  const uint32_t pay_u = smem_u32(S.pay), aux_u = smem_u32(S.aux);
  uint32_t qf[8][2];
  float o[16][2];
  float m_r = -INFINITY, l_r = 0.f;
  for (int u = u0; u < u1; ++u) {
    const int j = u % nt;
    const bool seg_start = (u == u0 || j == 0);
    if (seg_start) {
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = 0.f;
      m_r = -INFINITY;
      l_r = 0.f;
    }
    int s = it % kStages;
    uint32_t par = (it / kStages) & 1;
    ++it;
    if (!sw(&S.full[s], par, p.err, 0x630)) return false;
    if (seg_start) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        if (g8 < G) {
          const uint32_t qa = aux_u + s * kAux + (g8 * kHD + ks * 16 + 2 * t4) * 2;
          qf[ks][0] = lds32(qa);
          qf[ks][1] = lds32(qa + 16);
        } else {
          qf[ks][0] = qf[ks][1] = 0u;
        }
      }
    }
    const uint32_t sK = pay_u + s * kPay;
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t kf[4];
      const int r = warp * 16 + (lane & 7) + ((lane >> 4) << 3);
      const int cc = ks * 2 + ((lane >> 3) & 1);
      ldsm_x4(kf, sK + kv_off(r, cc));
      mma_bf16_16816(sc[0], qf[ks][0], 0u, qf[ks][1], 0u, kf[0], kf[1]);
      mma_bf16_16816(sc[1], qf[ks][0], 0u, qf[ks][1], 0u, kf[2], kf[3]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.empty[s]);
    const int64_t pos0 = (int64_t)j * kPos + warp * 16;
    float x[4];
#pragma unroll
    for (int jj = 0; jj < 2; ++jj)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t ps = pos0 + jj * 8 + 2 * t4 + e;
        x[jj * 2 + e] = (ps < Lold) ? sc[jj][e] * p.scale_log2 : -INFINITY;
      }
    float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_r, mx);
    const float bse = (m_new == -INFINITY) ? 0.f : m_new;
    const float corr = exp2f(m_r - bse);
    float pr[4], rs = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      pr[e] = exp2f(x[e] - bse);
      rs += pr[e];
    }
    l_r = l_r * corr + rs;
    m_r = m_new;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= corr;
      o[d][1] *= corr;
    }
    const uint32_t pa0 = pack_bf16x2(pr[0], pr[1]);
    const uint32_t pa2 = pack_bf16x2(pr[2], pr[3]);
    s = it % kStages;
    par = (it / kStages) & 1;
    ++it;
    if (!sw(&S.full[s], par, p.err, 0x631)) return false;
    const uint32_t sV = pay_u + s * kPay;
#pragma unroll
    for (int ip = 0; ip < 8; ++ip) {
      uint32_t vf[4];
      const int r = warp * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
      const int cc = ip * 2 + (lane >> 4);
      ldsm_x4_t(vf, sV + kv_off(r, cc));
      float d0[4] = {o[2 * ip][0], o[2 * ip][1], 0.f, 0.f};
      float d1[4] = {o[2 * ip + 1][0], o[2 * ip + 1][1], 0.f, 0.f};
      mma_bf16_16816(d0, pa0, 0u, pa2, 0u, vf[0], vf[1]);
      mma_bf16_16816(d1, pa0, 0u, pa2, 0u, vf[2], vf[3]);
      o[2 * ip][0] = d0[0]; o[2 * ip][1] = d0[1];
      o[2 * ip + 1][0] = d1[0]; o[2 * ip + 1][1] = d1[1];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.empty[s]);
    if (u != u1 - 1 && j != nt - 1) continue;
    // segment ends: hand this warp's (m, l, o) to the epilogue warps
    float lsum = l_r;
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
    lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
    const int b = segc & 1;
    if (!sw(&S.tempty[b], ((segc >> 1) & 1) ^ 1, p.err, 0x632)) return false;
    ++segc;
    float* tb = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(S.tbuf) + b * kTileBufBytes);
    if (g8 < G) {
#pragma unroll
      for (int d = 0; d < 16; ++d)
        *reinterpret_cast<float2*>(tb + (warp * G + g8) * kHD + d * 8 + 2 * t4) =
            make_float2(o[d][0], o[d][1]);
      if (t4 == 0) {
        tb[kCons * G * kHD + (warp * G + g8) * 2 + 0] = m_r;
        tb[kCons * G * kHD + (warp * G + g8) * 2 + 1] = lsum;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.tfull[b]);
  }
  return true;
}

// ---- epilogue warps: one projection segment --------------------------------
// tb: fp32 [128 rows][16 tokens] of this CTA's partial sums for tile t.
template <int G>
__device__ __forceinline__ void epi_proj(const Params& p, const Layer& Ly, const Smem& S, int ph,
                                         const Geo& g, int t, float* tb, int64_t pos, int et) {
  const int C = gridDim.x, c = blockIdx.x;
  const int lane = et & 31, ew = et >> 5;
  const int cf = owner(t * g.KB, g.U, C), cl = owner((t + 1) * g.KB - 1, g.U, C);
  // issue the epilogue's own global loads early (their data is ready)
  float xr0[kMaxTok], xr1[kMaxTok];
  float co = 0.f, si = 0.f, w0 = 0.f, w1 = 0.f;
  const __nv_bfloat16* xin = ph == kO ? p.X : p.X2;
  if (ph == kO || ph == kDN) {
    const int col = t * kRows + et;
#pragma unroll
    for (int tok = 0; tok < kMaxTok; ++tok) {
      xr0[tok] = tok < p.M ? bf2f(__ldcg(xin + (int64_t)tok * p.H + col)) : 0.f;
      xr1[tok] = tok < p.M ? bf2f(__ldcg(xin + (int64_t)tok * p.H + col + 64)) : 0.f;
    }
  } else if (ph == kQKV && t < p.Hq + p.Hkv) {
    const int64_t crow = pos + p.rope_delta;
    co = bf2f(p.cos[crow * 64 + et]);
    si = bf2f(p.sin[crow * 64 + et]);
    const __nv_bfloat16* nwq = t < p.Hq ? Ly.q_norm : Ly.k_norm;
    w0 = bf2f(nwq[et]);
    w1 = bf2f(nwq[et + 64]);
  }
  if (cl > cf) {
    // Split tile.  Its owner is the CTA holding its first units (cf): they
    // come at the end of that CTA's range, so the other contributors, which
    // meet the tile at the start of theirs, have usually published already.
    if (c != cf) {
      float4* mine = reinterpret_cast<float4*>(
          p.part + ((int64_t)c * 2 + slot_of(c, t, g.U, C, g.KB)) * kTileFloats);
      const float4* tb4 = reinterpret_cast<const float4*>(tb);
#pragma unroll
      for (int i = 0; i < kTileFloats / 4 / kEpiThreads; ++i)
        mine[et + i * kEpiThreads] = tb4[et + i * kEpiThreads];
      epi_bar();
      if (et == 0) {
        __threadfence();  // cumulative over the group's stores (ordered by the barrier)
        atomicAdd(&p.cnt[t], 1);
      }
      return;
    }
    if (et == 0) wait_contributors(&p.cnt[t], cl - cf, p.err, 0x660);
    epi_bar();
    // sum in CTA order: the owner's own partial first, then cf+1 .. cl
    float4 a[kTileFloats / 4 / kEpiThreads];
    const float4* tb4 = reinterpret_cast<const float4*>(tb);
#pragma unroll
    for (int i = 0; i < kTileFloats / 4 / kEpiThreads; ++i) a[i] = tb4[et + i * kEpiThreads];
    for (int cc = cf + 1; cc <= cl; cc += 2) {
      // two partials' loads in flight per round trip
      const bool two = cc + 1 <= cl;
      const float4* src0 = reinterpret_cast<const float4*>(
          p.part + ((int64_t)cc * 2 + slot_of(cc, t, g.U, C, g.KB)) * kTileFloats);
      const float4* src1 = two ? reinterpret_cast<const float4*>(
          p.part + ((int64_t)(cc + 1) * 2 + slot_of(cc + 1, t, g.U, C, g.KB)) * kTileFloats)
                               : src0;
      float4 v0[kTileFloats / 4 / kEpiThreads], v1[kTileFloats / 4 / kEpiThreads];
#pragma unroll
      for (int i = 0; i < kTileFloats / 4 / kEpiThreads; ++i) {
        v0[i] = __ldcg(src0 + et + i * kEpiThreads);
        v1[i] = two ? __ldcg(src1 + et + i * kEpiThreads) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < kTileFloats / 4 / kEpiThreads; ++i) {
        a[i].x += v0[i].x; a[i].y += v0[i].y; a[i].z += v0[i].z; a[i].w += v0[i].w;
        if (two) {
          a[i].x += v1[i].x; a[i].y += v1[i].y; a[i].z += v1[i].z; a[i].w += v1[i].w;
        }
      }
    }
    epi_bar();  // every thread has read its own slice of tb
    float4* tbw = reinterpret_cast<float4*>(tb);
#pragma unroll
    for (int i = 0; i < kTileFloats / 4 / kEpiThreads; ++i) tbw[et + i * kEpiThreads] = a[i];
    epi_bar();
  }
  // ---- epilogue of tile t (thread et owns rows et and et + 64) ----
  const int d0 = et, d1 = et + 64;
  if (ph == kQKV) {
    const int head = t;
    if (head >= p.Hq + p.Hkv) {
      const int hv = head - p.Hq - p.Hkv;
      for (int tok = 0; tok < p.M; ++tok) {
        __nv_bfloat16* dst = Ly.v_cache + (((int64_t)tok * p.Hkv + hv) * p.max_seq + pos) * kHD;
        dst[d0] = f2bf(tb[d0 * kMaxTok + tok]);
        dst[d1] = f2bf(tb[d1 * kMaxTok + tok]);
      }
      return;
    }
    float v0[kMaxTok], v1[kMaxTok];
#pragma unroll
    for (int tok = 0; tok < kMaxTok; ++tok) {
      v0[tok] = tok < p.M ? rbf(tb[d0 * kMaxTok + tok]) : 0.f;
      v1[tok] = tok < p.M ? rbf(tb[d1 * kMaxTok + tok]) : 0.f;
      const float s2 = warp_sum(v0[tok] * v0[tok] + v1[tok] * v1[tok]);
      if (lane == 0) S.red[ew * 16 + tok] = s2;
    }
    epi_bar();
    const bool is_q = head < p.Hq;
#pragma unroll
    for (int tok = 0; tok < kMaxTok; ++tok) {
      if (tok >= p.M) break;
      const float ss = S.red[tok] + S.red[16 + tok];
      const float rr = 1.0f / sqrtf(ss * (1.0f / kHD) + p.eps);
      const float n0 = rbf(rbf(v0[tok] * rr) * w0), n1 = rbf(rbf(v1[tok] * rr) * w1);
      const __nv_bfloat16 o0 = f2bf(rbf(n0 * co) + rbf(-n1 * si));
      const __nv_bfloat16 o1 = f2bf(rbf(n1 * co) + rbf(n0 * si));
      __nv_bfloat16* dst = is_q ? p.Q + ((int64_t)tok * p.Hq + head) * kHD
                                : Ly.k_cache + (((int64_t)tok * p.Hkv + (head - p.Hq)) * p.max_seq +
                                                pos) * kHD;
      dst[d0] = o0;
      dst[d1] = o1;
    }
    epi_bar();  // S.red free
  } else if (ph == kGU) {
    const int j = et >> 3, i = et & 7;
    const int f = t * (kRows / 2) + et;
    for (int tok = 0; tok < p.M; ++tok) {
      const float gt = rbf(tb[(16 * j + i) * kMaxTok + tok]);
      const float up = rbf(tb[(16 * j + 8 + i) * kMaxTok + tok]);
      p.act[(int64_t)tok * p.I + f] = f2bf(silu_ref(gt) * up);
    }
  } else {
    __nv_bfloat16* xout = ph == kO ? p.X2 : p.X;
    float* ssout = ph == kO ? p.ss_x2 : p.ss_x;
    const int col = t * kRows + et;
#pragma unroll
    for (int tok = 0; tok < kMaxTok; ++tok) {
      float q2 = 0.f;
      if (tok < p.M) {
        const __nv_bfloat16 o0 = f2bf(xr0[tok] + rbf(tb[d0 * kMaxTok + tok]));
        const __nv_bfloat16 o1 = f2bf(xr1[tok] + rbf(tb[d1 * kMaxTok + tok]));
        xout[(int64_t)tok * p.H + col] = o0;
        xout[(int64_t)tok * p.H + col + 64] = o1;
        q2 = bf2f(o0) * bf2f(o0) + bf2f(o1) * bf2f(o1);
      }
      q2 = warp_sum(q2);
      if (lane == 0) S.red[ew * 16 + tok] = q2;
    }
    epi_bar();
    if (et < 16) ssout[t * 16 + et] = S.red[et] + S.red[16 + et];
    epi_bar();
  }
}

// ---- epilogue warps: one attention segment ----------------------------------
// tb: [4 warps][G heads][128] fp32 output sums and [4][G][2] (max, sum) states.
template <int G>
__device__ __forceinline__ void epi_att(const Params& p, const Layer& Ly, const Smem& S,
                                        const Geo& g, int pair, bool with_new, int nt,
                                        float* tb, int64_t pos, int et) {
  const int C = gridDim.x, c = blockIdx.x;
  const int lane = et & 31, ew = et >> 5;
  const int b = pair / p.Hkv, kvh = pair % p.Hkv;
  const int d0 = et, d1 = et + 64;
  const float* ml = tb + kCons * G * kHD;
  float s_new[G];
#pragma unroll
  for (int gg = 0; gg < G; ++gg) s_new[gg] = -INFINITY;
  float kn0 = 0.f, kn1 = 0.f, vn0 = 0.f, vn1 = 0.f;
  if (with_new) {
    // the new token's row: written this step by the QKV epilogues
    const int64_t nrow = ((int64_t)pair * p.max_seq + pos) * kHD;
    kn0 = bf2f(__ldcg(Ly.k_cache + nrow + d0));
    kn1 = bf2f(__ldcg(Ly.k_cache + nrow + d1));
    vn0 = bf2f(__ldcg(Ly.v_cache + nrow + d0));
    vn1 = bf2f(__ldcg(Ly.v_cache + nrow + d1));
    float qv0[G], qv1[G];
#pragma unroll
    for (int gg = 0; gg < G; ++gg) {
      const __nv_bfloat16* qh = p.Q + ((int64_t)b * p.Hq + kvh * G + gg) * kHD;
      qv0[gg] = bf2f(__ldcg(qh + d0));
      qv1[gg] = bf2f(__ldcg(qh + d1));
    }
#pragma unroll
    for (int gg = 0; gg < G; ++gg) {
      const float s2 = warp_sum(qv0[gg] * kn0 + qv1[gg] * kn1);
      if (lane == 0) S.red[ew * 16 + gg] = s2;
    }
    epi_bar();
#pragma unroll
    for (int gg = 0; gg < G; ++gg) s_new[gg] = (S.red[gg] + S.red[16 + gg]) * p.scale_log2;
    epi_bar();
  }
  const int cf = owner(pair * nt, g.U, C), cl = owner(pair * nt + nt - 1, g.U, C);
  const bool split = cl > cf;
  const bool own = !split || c == cf;  // the owner merges (see epi_proj)
  float* ap = p.apart + ((int64_t)c * 2 + slot_of(c, pair, g.U, C, nt)) * (G * (kHD + 2));
  float M[G], A0[G], A1[G], Ls[G];
#pragma unroll
  for (int gg = 0; gg < G; ++gg) {
    float Mx = s_new[gg];
#pragma unroll
    for (int w = 0; w < kCons; ++w) Mx = fmaxf(Mx, ml[(w * G + gg) * 2]);
    float a0 = 0.f, a1 = 0.f, lsm = 0.f;
#pragma unroll
    for (int w = 0; w < kCons; ++w) {
      const float mw = ml[(w * G + gg) * 2];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - Mx);
      a0 = fmaf(f, tb[(w * G + gg) * kHD + d0], a0);
      a1 = fmaf(f, tb[(w * G + gg) * kHD + d1], a1);
      lsm = fmaf(f, ml[(w * G + gg) * 2 + 1], lsm);
    }
    if (with_new) {
      const float f = exp2f(s_new[gg] - Mx);
      a0 = fmaf(f, vn0, a0);
      a1 = fmaf(f, vn1, a1);
      lsm += f;
    }
    M[gg] = Mx; A0[gg] = a0; A1[gg] = a1; Ls[gg] = lsm;
    if (!own) {
      ap[gg * (kHD + 2) + 2 + d0] = a0;
      ap[gg * (kHD + 2) + 2 + d1] = a1;
      if (et == 0) {
        ap[gg * (kHD + 2)] = Mx;
        ap[gg * (kHD + 2) + 1] = lsm;
      }
    }
  }
  if (!own) {
    epi_bar();
    if (et == 0) {
      __threadfence();
      atomicAdd(&p.cnt[pair], 1);
    }
    return;
  }
  if (split) {
    if (et == 0) wait_contributors(&p.cnt[pair], cl - cf, p.err, 0x661);
    epi_bar();
    // merge the other segments in CTA order (online: running max, rescaled sums)
    for (int cc = cf + 1; cc <= cl; ++cc) {
      const float* q2 =
          p.apart + ((int64_t)cc * 2 + slot_of(cc, pair, g.U, C, nt)) * (G * (kHD + 2));
      float ms[G], ls[G], x0[G], x1[G];
#pragma unroll
      for (int gg = 0; gg < G; ++gg) {
        ms[gg] = __ldcg(q2 + gg * (kHD + 2));
        ls[gg] = __ldcg(q2 + gg * (kHD + 2) + 1);
        x0[gg] = __ldcg(q2 + gg * (kHD + 2) + 2 + d0);
        x1[gg] = __ldcg(q2 + gg * (kHD + 2) + 2 + d1);
      }
#pragma unroll
      for (int gg = 0; gg < G; ++gg) {
        if (ms[gg] == -INFINITY) continue;
        const float Mn = fmaxf(M[gg], ms[gg]);
        const float fo = (M[gg] == -INFINITY) ? 0.f : exp2f(M[gg] - Mn);
        const float fn = exp2f(ms[gg] - Mn);
        A0[gg] = A0[gg] * fo + fn * x0[gg];
        A1[gg] = A1[gg] * fo + fn * x1[gg];
        Ls[gg] = Ls[gg] * fo + fn * ls[gg];
        M[gg] = Mn;
      }
    }
  }
#pragma unroll
  for (int gg = 0; gg < G; ++gg) {
    __nv_bfloat16* out = p.A + ((int64_t)b * p.Hq + kvh * G + gg) * kHD;
    out[d0] = f2bf(Ls[gg] > 0.f ? A0[gg] / Ls[gg] : 0.f);
    out[d1] = f2bf(Ls[gg] > 0.f ? A1[gg] / Ls[gg] : 0.f);
  }
}

template <int NT, int G>
__global__ void __launch_bounds__(kThreadsAll, 1) decode_step_kernel(Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  Smem S;
  S.pay = base;
  S.aux = S.pay + kStages * kPay;
  S.tbuf = reinterpret_cast<float*>(S.aux + kStages * kAux);
  S.nw = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(S.tbuf) + 2 * kTileBufBytes);
  S.r = reinterpret_cast<float*>(S.nw + kMaxHidden);
  S.red = S.r + 16;
  S.flag = reinterpret_cast<int*>(S.red + kEpiWarps * 16);
  S.full = reinterpret_cast<uint64_t*>(S.flag + 4);
  S.empty = S.full + kStages;
  S.tfull = S.empty + kStages;
  S.tempty = S.tfull + 2;
  S.phase_ok = S.tempty + 2;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = gridDim.x, c = blockIdx.x;
  const int L = p.kv_len_dev ? *p.kv_len_dev : 1;  // set before the launch
  const int64_t pos = L - 1;                       // cache row of the new token
  const int nt = (L + kPos - 1) / kPos;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&S.full[s], kFullCount);
      mbar_init(&S.empty[s], kCons);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S.tfull[b], kCons);
      mbar_init(&S.tempty[b], kEpiWarps);
    }
    mbar_init(S.phase_ok, 1);
    fence_mbar_init();
    if (pos < 0 || pos >= p.max_seq || pos + p.rope_delta < 0 ||
        pos + p.rope_delta >= p.rope_rows)
      report_timeout(p.err, 0x6ff);  // length outside the cache or the rope table
  }
  __syncthreads();
  if (aborted(p.err)) return;

  if (warp == kWarpProd) {
    // =================== producer: weight and K/V tiles =====================
    if (lane == 0) {
      int it = 0;
      for (int l = 0; l < p.n_layers; ++l) {
        const Layer& Ly = p.layers[l];
        for (int ph = 0; ph < kPhases; ++ph) {
          const Geo g = geo(p, ph, nt);
          const int u0 = unit_lo(c, g.U, C), u1 = unit_lo(c + 1, g.U, C);
          const CUtensorMap* tm = ph == kQKV ? &Ly.tm_qkv : ph == kO ? &Ly.tm_o
                                : ph == kGU ? &Ly.tm_gu : &Ly.tm_dn;
          for (int u = u0; u < u1; ++u) {
            if (ph != kATT) {
              const int s = it % kStages;
              const uint32_t par = (it / kStages) & 1;
              ++it;
              if (!sw(&S.empty[s], par ^ 1, p.err, 0x601)) return;
              mbar_arrive_expect_tx(&S.full[s], kPay);
              tma_load_2d(S.pay + s * kPay, tm, &S.full[s], (u % g.KB) * kBK, (u / g.KB) * kRows,
                          kCacheEvictFirst);
            } else {
              const int pair = u / nt, j = u % nt;
              const int y = (int)((int64_t)pair * p.max_seq + (int64_t)j * kPos);
              for (int kv = 0; kv < 2; ++kv) {
                const int s = it % kStages;
                const uint32_t par = (it / kStages) & 1;
                ++it;
                if (!sw(&S.empty[s], par ^ 1, p.err, 0x602)) return;
                const CUtensorMap* tkv = kv == 0 ? &Ly.tm_k : &Ly.tm_v;
                mbar_arrive_expect_tx(&S.full[s], kPay);
                tma_load_2d(S.pay + s * kPay, tkv, &S.full[s], 0, y, kCacheEvictFirst);
                tma_load_2d(S.pay + s * kPay + 8192, tkv, &S.full[s], 64, y, kCacheEvictFirst);
              }
            }
          }
        }
      }
    }
    return;
  }

  if (warp == kWarpStage) {
    // =================== activations: wait for the grid, stage x ============
    int it = 0;
    const int ch = lane & 7;  // 16-byte chunk (8 K values) owned by this lane
    const uint32_t aux_u = smem_u32(S.aux);
    for (int l = 0; l < p.n_layers; ++l) {
      const Layer& Ly = p.layers[l];
      for (int ph = 0; ph < kPhases; ++ph) {
        const Geo g = geo(p, ph, nt);
        const int u0 = unit_lo(c, g.U, C), u1 = unit_lo(c + 1, g.U, C);
        const int q = 1 + kPhases * l + ph;
        const __nv_bfloat16* nw = ph == kQKV ? Ly.in_norm : ph == kGU ? Ly.post_norm : nullptr;
        if (nw && u1 > u0) {
          // this layer's norm weights (static) while the grid finishes the
          // previous phase; this CTA's consumers finished with the buffer two
          // phases ago (this warp has seen that grid arrival)
          for (int k = lane; k < p.H / 8; k += 32)
            cp_async16(smem_u32(S.nw) + k * 16, nw + k * 8, 16);
          cp_async_commit();
          cp_async_wait<0>();
        }
        grid_wait(&p.bars[q - 1], (unsigned)C, p.err, 0x610 + ph);
        if (u1 > u0) {
          if (nw && lane < 16) {
            const float* ssb = ph == kQKV ? p.ss_x : p.ss_x2;
            float r = 0.f;
            if (lane < p.M) {
              float ss = 0.f;  // fixed order over the tiles
              for (int tt = 0; tt < p.H / kRows; ++tt) ss += __ldcg(ssb + tt * 16 + lane);
              r = 1.0f / sqrtf(ss / (float)p.H + p.eps);
            }
            S.r[lane] = r;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(S.phase_ok);  // release r, norm weights, the grid acquire
        }
        if (ph == kATT) {
          for (int u = u0; u < u1; ++u) {
            const int pair = u / nt;
            const int b = pair / p.Hkv, kvh = pair % p.Hkv;
            int s = it % kStages;
            uint32_t par = (it / kStages) & 1;
            ++it;
            if (!sw(&S.empty[s], par ^ 1, p.err, 0x611)) return;
            const __nv_bfloat16* qsrc = p.Q + ((int64_t)b * p.Hq + (int64_t)kvh * G) * kHD;
            for (int k = lane; k < G * 16; k += 32)
              cp_async16(aux_u + s * kAux + k * 16, qsrc + k * 8, 16);
            cp_async_arrive(&S.full[s]);
            s = it % kStages;
            par = (it / kStages) & 1;
            ++it;
            if (!sw(&S.empty[s], par ^ 1, p.err, 0x612)) return;
            mbar_arrive(&S.full[s]);
          }
          continue;
        }
        const __nv_bfloat16* src = ph == kQKV ? p.X : ph == kO ? p.A : ph == kGU ? p.X2 : p.act;
        for (int u = u0; u < u1; ++u) {
          const int s = it % kStages;
          const uint32_t par = (it / kStages) & 1;
          ++it;
          if (!sw(&S.empty[s], par ^ 1, p.err, 0x613)) return;
          const int kb = u % g.KB;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int row = (lane >> 3) + 4 * i;  // rows >= M are zero-filled
            const __nv_bfloat16* gsrc =
                src + (int64_t)(row < p.M ? row : 0) * g.K + kb * kBK + ch * 8;
            cp_async16(aux_u + s * kAux + row * 128 + ((ch ^ (row & 7)) << 4), gsrc,
                       row < p.M ? 16 : 0);
          }
          cp_async_arrive(&S.full[s]);
        }
      }
    }
    return;
  }

  if (warp >= kWarpEpi) {
    // =================== epilogues ===========================================
    const int et = threadIdx.x - kWarpEpi * 32;  // 0..63
    const int ew = et >> 5;
    // P0: per-tile sums of squares of the layer-0 input rows
    if (c < p.H / kRows) {
      const int col = c * kRows + et;
#pragma unroll
      for (int tok = 0; tok < kMaxTok; ++tok) {
        float q2 = 0.f;
        if (tok < p.M) {
          const float v0 = bf2f(p.X[(int64_t)tok * p.H + col]);
          const float v1 = bf2f(p.X[(int64_t)tok * p.H + col + 64]);
          q2 = v0 * v0 + v1 * v1;
        }
        q2 = warp_sum(q2);
        if (lane == 0) S.red[ew * 16 + tok] = q2;
      }
      epi_bar();
      if (et < 16) p.ss_x[c * 16 + et] = S.red[et] + S.red[16 + et];
    }
    epi_bar();
    if (et == 0) grid_arrive(&p.bars[0]);
    int segc = 0;
    for (int l = 0; l < p.n_layers; ++l) {
      const Layer& Ly = p.layers[l];
      for (int ph = 0; ph < kPhases; ++ph) {
        const Geo g = geo(p, ph, nt);
        const int u0 = unit_lo(c, g.U, C), u1 = unit_lo(c + 1, g.U, C);
        for (int u = u0; u < u1;) {
          const int t = u / g.KB;
          const int ue = min(u1, (t + 1) * g.KB);
          const int b = segc & 1;
          if (!sw(&S.tfull[b], (segc >> 1) & 1, p.err, 0x650)) return;
          ++segc;
          float* tb = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(S.tbuf) + b * kTileBufBytes);
          if (ph == kATT)
            epi_att<G>(p, Ly, S, g, t, ue == (t + 1) * g.KB, nt, tb, pos, et);
          else
            epi_proj<G>(p, Ly, S, ph, g, t, tb, pos, et);
          epi_bar();
          if (lane == 0) mbar_arrive(&S.tempty[b]);
          u = ue;
        }
        epi_bar();
        if (et == 0) grid_arrive(&p.bars[1 + kPhases * l + ph]);
      }
    }
    // the last CTA out resets the phase counters for the next launch
    if (et == 0) {
      __threadfence();
      const unsigned old = atomicAdd(p.exit_cnt, 1u);
      if (old == (unsigned)C - 1) {
        const int nb = 1 + kPhases * p.n_layers;
        for (int i = 0; i < nb; ++i) p.bars[i] = 0u;
        *p.exit_cnt = 0u;
        __threadfence();
      }
    }
    return;
  }

  // ======================= consumers (warps 0..3) ===========================
  int it = 0, segc = 0;
  uint32_t nphase = 0;  // phases with work so far (parity of phase_ok)
  for (int l = 0; l < p.n_layers; ++l) {
    for (int ph = 0; ph < kPhases; ++ph) {
      const Geo g = geo(p, ph, nt);
      const int u0 = unit_lo(c, g.U, C), u1 = unit_lo(c + 1, g.U, C);
      if (u1 == u0) continue;
      if (!sw(S.phase_ok, nphase & 1, p.err, 0x640 + ph)) return;
      ++nphase;
      bool ok;
      if (ph == kATT)
        ok = consume_att<G>(p, S, g, u0, u1, nt, pos, it, segc, warp, lane);
      else if (ph == kQKV || ph == kGU)
        ok = consume_proj<NT, true>(p, S, g, u0, u1, it, segc, warp, lane);
      else
        ok = consume_proj<NT, false>(p, S, g, u0, u1, it, segc, warp, lane);
      if (!ok) return;
    }
  }
}

// ------------------------------------------------------------------ host
struct Plan {
  int dev = -1;
  int n_layers = 0, M = 0, H = 0, Hq = 0, Hkv = 0, I = 0, C = 0;
  int64_t max_seq = 0, rope_rows = 0;
  float eps = 1e-6f;
  const void* cos = nullptr;
  const void* sin = nullptr;
  Layer* d_layers = nullptr;
  void* d_mem = nullptr;  // one allocation for every workspace below
  __nv_bfloat16 *X2 = nullptr, *A = nullptr, *Q = nullptr, *act = nullptr;
  float *ss_x2 = nullptr, *part = nullptr, *apart = nullptr;
  int* cnt = nullptr;
  unsigned *bars = nullptr, *exit_cnt = nullptr;
};

constexpr size_t kSmem = 1024 + (size_t)kStages * (kPay + kAux) + 2 * kTileBufBytes +
                         kMaxHidden * 2 + 16 * 4 + kEpiWarps * 16 * 4 + 4 * 4 +
                         (2 * kStages + 5) * 8;

template <int NT, int G>
static int launch(const Plan& pl, const Params& prm, cudaStream_t s) {
  auto kern = decode_step_kernel<NT, G>;
  static bool attr[64] = {false};
  if (pl.dev >= 0 && pl.dev < 64 && !attr[pl.dev]) {
    Q3_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmem));
    int per_sm = 0;
    Q3_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreadsAll, kSmem));
    if (per_sm < 1) return fail(Q3_ERR_UNSUPPORTED, "q3_decode_step: kernel does not fit an SM");
    attr[pl.dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.C);
  cfg.blockDim = dim3(kThreadsAll);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  Q3_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, prm));
  count_launch();
  return Q3_OK;
}

}  // namespace step
}  // namespace q3

extern "C" int q3_decode_step_create(const q3_step_layer* layers, int n_layers, int batch,
                                     int hidden, int q_heads, int kv_heads, int inter,
                                     int64_t max_seq, float eps, const void* rope_cos,
                                     const void* rope_sin, int64_t rope_rows, void** plan_out) {
  using namespace q3;
  using namespace q3::step;
  Q3_REQUIRE(layers && plan_out && n_layers > 0 && rope_cos && rope_sin,
             "q3_decode_step_create: null argument");
  *plan_out = nullptr;
  Q3_REQUIRE(batch >= 1 && batch <= kMaxTok, "q3_decode_step_create: batch %d not in [1, 16]",
             batch);
  Q3_REQUIRE(kv_heads > 0 && q_heads % kv_heads == 0 && q_heads / kv_heads == 4,
             "q3_decode_step_create: %d/%d heads: only 4 query heads per KV head are built",
             q_heads, kv_heads);
  Q3_REQUIRE(hidden <= kMaxHidden, "q3_decode_step_create: hidden %d > %d", hidden, kMaxHidden);
  Q3_REQUIRE(hidden % kRows == 0 && inter % (kRows / 2) == 0 && (q_heads * kHD) % kBK == 0 &&
                 inter % kBK == 0,
             "q3_decode_step_create: hidden %% 128, inter %% 64 required");
  Q3_REQUIRE(2 * inter / kRows <= kMaxTiles && (q_heads + 2 * kv_heads) <= kMaxTiles &&
                 (int64_t)batch * kv_heads <= kMaxTiles && hidden / kRows <= num_sms(),
             "q3_decode_step_create: shape too large");
  Q3_REQUIRE(max_seq % kPos == 0 && max_seq > 0,
             "q3_decode_step_create: max_seq must be a multiple of 64");
  auto* pl = new Plan();
  cudaGetDevice(&pl->dev);
  pl->n_layers = n_layers; pl->M = batch; pl->H = hidden; pl->Hq = q_heads; pl->Hkv = kv_heads;
  pl->I = inter; pl->max_seq = max_seq; pl->eps = eps; pl->cos = rope_cos; pl->sin = rope_sin;
  pl->rope_rows = rope_rows;
  pl->C = num_sms();
  std::vector<Layer> hl(n_layers);
  int rc = Q3_OK;
  for (int l = 0; l < n_layers && rc == Q3_OK; ++l) {
    const q3_step_layer& s = layers[l];
    Layer& d = hl[l];
    if (!s.w_qkv || !s.w_o || !s.w_gate_up || !s.w_down || !s.input_norm || !s.post_norm ||
        !s.q_norm || !s.k_norm || !s.k_cache || !s.v_cache) {
      rc = fail(Q3_ERR_INVALID, "q3_decode_step_create: layer %d has a null pointer", l);
      break;
    }
    const int64_t kv_rows = (int64_t)batch * kv_heads * max_seq;
    if ((rc = make_tmap_2d(&d.tm_qkv, s.w_qkv, (int64_t)(q_heads + 2 * kv_heads) * kHD, hidden,
                           kRows, kBK)) ||
        (rc = make_tmap_2d(&d.tm_o, s.w_o, hidden, (int64_t)q_heads * kHD, kRows, kBK)) ||
        (rc = make_tmap_2d(&d.tm_gu, s.w_gate_up, 2 * (int64_t)inter, hidden, kRows, kBK)) ||
        (rc = make_tmap_2d(&d.tm_dn, s.w_down, hidden, inter, kRows, kBK)) ||
        (rc = make_tmap_2d(&d.tm_k, s.k_cache, kv_rows, kHD, kPos, 64)) ||
        (rc = make_tmap_2d(&d.tm_v, s.v_cache, kv_rows, kHD, kPos, 64)))
      break;
    d.in_norm = (const __nv_bfloat16*)s.input_norm;
    d.post_norm = (const __nv_bfloat16*)s.post_norm;
    d.q_norm = (const __nv_bfloat16*)s.q_norm;
    d.k_norm = (const __nv_bfloat16*)s.k_norm;
    d.k_cache = (__nv_bfloat16*)s.k_cache;
    d.v_cache = (__nv_bfloat16*)s.v_cache;
  }
  if (rc != Q3_OK) {
    delete pl;
    return rc;
  }
  const int G = q_heads / kv_heads;
  const int C = pl->C;
  const size_t nb = 1 + (size_t)kPhases * n_layers;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  const size_t o_layers = take(sizeof(Layer) * n_layers);
  const size_t o_x2 = take((size_t)batch * hidden * 2);
  const size_t o_a = take((size_t)batch * q_heads * kHD * 2);
  const size_t o_q = take((size_t)batch * q_heads * kHD * 2);
  const size_t o_act = take((size_t)batch * inter * 2);
  const size_t o_ss2 = take((size_t)(hidden / kRows) * 16 * 4);
  const size_t o_part = take((size_t)C * 2 * kTileFloats * 4);
  const size_t o_apart = take((size_t)C * 2 * G * (kHD + 2) * 4);
  const size_t o_cnt = take((size_t)kMaxTiles * 4);
  const size_t o_bars = take(nb * 4);
  const size_t o_exit = take(4);
  cudaError_t e = cudaMalloc(&pl->d_mem, off);
  if (e != cudaSuccess) {
    delete pl;
    return fail(Q3_ERR_CUDA, "q3_decode_step_create: cudaMalloc(%zu): %s", off,
                cudaGetErrorString(e));
  }
  char* m = static_cast<char*>(pl->d_mem);
  e = cudaMemset(m, 0, off);
  if (e == cudaSuccess)
    e = cudaMemcpy(m + o_layers, hl.data(), sizeof(Layer) * n_layers, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(pl->d_mem);
    delete pl;
    return fail(Q3_ERR_CUDA, "q3_decode_step_create: %s", cudaGetErrorString(e));
  }
  pl->d_layers = reinterpret_cast<Layer*>(m + o_layers);
  pl->X2 = reinterpret_cast<__nv_bfloat16*>(m + o_x2);
  pl->A = reinterpret_cast<__nv_bfloat16*>(m + o_a);
  pl->Q = reinterpret_cast<__nv_bfloat16*>(m + o_q);
  pl->act = reinterpret_cast<__nv_bfloat16*>(m + o_act);
  pl->ss_x2 = reinterpret_cast<float*>(m + o_ss2);
  pl->part = reinterpret_cast<float*>(m + o_part);
  pl->apart = reinterpret_cast<float*>(m + o_apart);
  pl->cnt = reinterpret_cast<int*>(m + o_cnt);
  pl->bars = reinterpret_cast<unsigned*>(m + o_bars);
  pl->exit_cnt = reinterpret_cast<unsigned*>(m + o_exit);
  *plan_out = pl;
  return Q3_OK;
}

extern "C" int q3_decode_step(void* plan, void* x, float* ss, const int32_t* kv_len_dev,
                              int64_t rope_delta, q3_stream_t stream) {
  using namespace q3;
  using namespace q3::step;
  Q3_REQUIRE(plan && x && ss && kv_len_dev, "q3_decode_step: null argument");
  const Plan& pl = *static_cast<const Plan*>(plan);
  Q3_REQUIRE(aligned(x, 16), "q3_decode_step: x must be 16-byte aligned");
  Params p;
  p.layers = pl.d_layers;
  p.n_layers = pl.n_layers; p.M = pl.M; p.H = pl.H; p.Hq = pl.Hq; p.Hkv = pl.Hkv; p.I = pl.I;
  p.max_seq = pl.max_seq; p.rope_rows = pl.rope_rows; p.rope_delta = rope_delta;
  p.eps = pl.eps;
  p.scale_log2 = (1.0f / sqrtf((float)kHD)) * 1.4426950408889634f;
  p.cos = (const __nv_bfloat16*)pl.cos;
  p.sin = (const __nv_bfloat16*)pl.sin;
  p.kv_len_dev = kv_len_dev;
  p.X = (__nv_bfloat16*)x;
  p.X2 = pl.X2; p.A = pl.A; p.Q = pl.Q; p.act = pl.act;
  p.ss_x = ss; p.ss_x2 = pl.ss_x2;
  p.part = pl.part; p.apart = pl.apart; p.cnt = pl.cnt; p.bars = pl.bars;
  p.exit_cnt = pl.exit_cnt;
  p.err = device_error_word();
  cudaStream_t s = (cudaStream_t)stream;
  return pl.M > 8 ? launch<2, 4>(pl, p, s) : launch<1, 4>(pl, p, s);
}

extern "C" int q3_decode_step_destroy(void* plan) {
  using namespace q3::step;
  if (!plan) return Q3_OK;
  Plan* pl = static_cast<Plan*>(plan);
  cudaDeviceSynchronize();
  if (pl->d_mem) cudaFree(pl->d_mem);
  delete pl;
  return Q3_OK;
}
