// Decode-shaped projections (M <= 16 tokens): C = A W^T with fused epilogues.
//
// Reference: the compiled matmuls of model_fused.py (:103, :141, :165-169,
// :172, :183) at decode time, where the activation is B x 1 tokens.  Tensor
// cores are idle at this M, so the kernel is built around HBM streaming:
//
//   * one CTA owns a 64-row tile of W ([N, K], K-major) over a K slice;
//   * a producer warp issues TMA 2-D loads of 64 rows x 64 K (8 KB, 128-byte
//     swizzle) into a 6-stage shared-memory ring guarded by mbarriers, so up
//     to 48 KB of weights per CTA (144 KB per SM at 3 CTAs/SM) is in flight;
//   * four consumer warps each take 16 rows and run bf16 mma.sync m16n8k16
//     with W as the 16-row A operand and the tokens as B.  The producer loads
//     the matching 64-wide K slice of the activations (<= 16 rows, 2 KB) into
//     the same stage by TMA, so consumers never wait on a global load;
//     Lane (g, t) reads the 16-byte chunks 2t+h (h = 0, 1) of rows g and g+8:
//     with the 128-byte swizzle (chunk c of row r lives at c ^ (r % 8)) the two
//     rows of a quarter-warp hit disjoint even/odd chunk sets, so the shared
//     loads are bank-conflict free; A and B use the same K permutation;
//   * K is split over the CTAs of a thread-block cluster (up to 8); partials
//     are reduced over distributed shared memory by cluster rank 0, which runs
//     the epilogue (plain, residual add, or SwiGLU on 8-row gate/up blocks);
//   * optional fusions, chosen at compile time so the plain kernel keeps its
//     short inner loop: the RMSNorm that precedes the projection (a sixth,
//     normaliser warp rescales each staged activation tile in shared memory
//     once, between the TMA landing and the consumers), and, after a residual
//     epilogue, per-tile sums of squares of the outputs for the next norm.
#include "comm.h"
#include "common.cuh"

namespace q3 {

constexpr int kGvRows = 64;                 // W rows per CTA
constexpr int kGvBK = 64;                   // K elements per stage (one 128-byte row)
constexpr int kGvStages = 6;
constexpr int kGvWBytes = kGvRows * kGvBK * 2;       // 8 KB of W per stage
constexpr int kGvXBytes = 16 * kGvBK * 2;            // 2 KB of activations (<= 16 tokens)
constexpr int kGvStageBytes = kGvWBytes + kGvXBytes;  // 1024-byte multiple
constexpr int kGvConsumers = 4;
constexpr int kGvSmem = kGvStages * kGvStageBytes + 1024 /*align*/ + 256 /*barriers*/;

// Compile-time fusion flags of gemv_tma_kernel.
constexpr int kFlNorm = 1;   // RMSNorm of the activations (normaliser warp)
constexpr int kFlSsOut = 2;  // residual epilogue: per-tile output sums of squares

// warps: consumers, the TMA producer, and with kFlNorm the normaliser
__host__ __device__ constexpr int gv_threads(int fl) {
  return (kGvConsumers + 1 + ((fl & kFlNorm) ? 1 : 0)) * 32;
}

// Internal epilogue id (not part of the public enum): row-parallel partial,
// all-reduced across the tensor-parallel ranks through peer memory, plus the
// optional residual.
constexpr int kEpiAllReduce = 3;

struct GemvParams {
  const __nv_bfloat16* A;
  __nv_bfloat16* C;
  const __nv_bfloat16* R;
  int M, N, K, ldc;
  int kb_per_cta;  // 64-wide K blocks per CTA
  int* err;
  CommDev comm;    // used by kEpiAllReduce only
  // Fused input RMSNorm (model_fused.py:37-40) when norm_w != nullptr: the
  // activations are normalised on the fly, x -> bf16(bf16(x * rsqrt(mean(x^2)
  // + eps)) * norm_w), with the per-token rsqrt computed over the full row.
  const __nv_bfloat16* norm_w;
  float eps;
  // When ss_in is set, the per-token sum of squares of A comes precomputed as
  // ss_tiles partial sums [ss_tiles][16] (written by the kernel that produced
  // A, see ss_out) instead of being recomputed from the rows of A.
  const float* ss_in;
  int ss_tiles;
  // Residual epilogue only: per-tile partial sums of squares of the stored
  // (bf16) outputs, [gridDim.x][16], for the RMSNorm of the next projection.
  float* ss_out;
};

__device__ __forceinline__ uint4 rms_scale_chunk(uint4 x, float r, uint4 w) {
  uint32_t xs[4] = {x.x, x.y, x.z, x.w};
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(xs[i]), g = unpack_bf16x2(ws[i]);
    xs[i] = pack_bf16x2(rbf(f.x * r) * g.x, rbf(f.y * r) * g.y);
  }
  return make_uint4(xs[0], xs[1], xs[2], xs[3]);
}

__device__ __forceinline__ void consumer_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kGvConsumers * 32) : "memory");
}
__device__ __forceinline__ void st_word_peer(uint2* p, uint32_t data, uint32_t flag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(data), "r"(flag)
               : "memory");
}
__device__ __forceinline__ uint2 ld_word_inbox(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p)
               : "memory");
  return v;
}

// All-reduce epilogue of one 64-column tile, run by the 128 consumer threads
// of cluster rank 0.  part[col][tok] holds this rank's partial, already
// rounded to bf16 like the reference's projection output.
//
// Protocol (one-shot, flag in every word): the tile's call number f comes from
// this rank's per-tile counter, which every rank advances identically (all
// ranks make the same calls).  Each thread owns word w = (column w / 8, token
// pair w % 8) of the tile and stores {data, f} into every peer's inbox
// (parity f & 1, source slot = this rank) with one 8-byte store; then it
// polls the same word of every peer in its own inbox until the flag reads f
// (bounded wait), and sums the ranks' bf16 values in fp32 in rank order, so
// every rank stores identical values.  A peer can be at most one call ahead
// (it cannot finish call f+1 before receiving this rank's call f+1 words,
// which this rank sends after its call f finished), so two parities suffice.
__device__ __forceinline__ void allreduce_tile(const GemvParams& p, int tile, int row0,
                                               __nv_bfloat16 (*part)[kArTokens],
                                               uint32_t* f_s) {
  const int tid = threadIdx.x;  // consumers are threads 0..127
  const CommDev& cm = p.comm;
  if (tid == 0) *f_s = cm.counters[tile] + 1u;  // this rank's own memory
  consumer_bar();
  const uint32_t f = *f_s;
  const int par = (int)(f & 1u);
  const int pairs = (p.M + 1) >> 1;  // token pairs that carry data
  constexpr int kWordsPerThread = kArWords / (kGvConsumers * 32);
  uint32_t mine[kWordsPerThread];
#pragma unroll
  for (int i = 0; i < kWordsPerThread; ++i) {
    const int w = tid + i * kGvConsumers * 32;
    mine[i] = reinterpret_cast<const uint32_t*>(&part[w >> 3][0])[w & 7];
  }
  // push this rank's words to every peer
  const size_t slot_self = ((size_t)(par * kMaxRanks + cm.rank) * cm.max_tiles + tile) * kArWords;
  for (int r = 0; r < cm.world; ++r) {
    if (r == cm.rank) continue;
    uint2* dst = cm.inbox[r] + slot_self;
#pragma unroll
    for (int i = 0; i < kWordsPerThread; ++i) {
      const int w = tid + i * kGvConsumers * 32;
      if ((w & 7) < pairs) st_word_peer(dst + w, mine[i], f);
    }
  }
  // collect the peers' words and reduce in rank order
  float s0[kWordsPerThread], s1[kWordsPerThread];
#pragma unroll
  for (int i = 0; i < kWordsPerThread; ++i) s0[i] = s1[i] = 0.f;
  bool gave_up = false;
  for (int r = 0; r < cm.world; ++r) {
#pragma unroll
    for (int i = 0; i < kWordsPerThread; ++i) {
      const int w = tid + i * kGvConsumers * 32;
      if ((w & 7) >= pairs) continue;
      uint32_t d;
      if (r == cm.rank) {
        d = mine[i];
      } else {
        const uint2* src = cm.inbox[cm.rank] +
                           ((size_t)(par * kMaxRanks + r) * cm.max_tiles + tile) * kArWords + w;
        uint2 v = ld_word_inbox(src);
        if (v.y != f && !gave_up) {
          const uint64_t t0 = globaltimer_ns();
          uint32_t spins = 0;
          while ((v = ld_word_inbox(src)).y != f) {
            if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > cm.wait_ns) {
              report_timeout(p.err, 0x501);
              gave_up = true;
              break;
            }
          }
        }
        d = v.x;
      }
      const float2 fv = unpack_bf16x2(d);
      s0[i] += fv.x;
      s1[i] += fv.y;
    }
  }
  // every thread holds token pair tid & 7 (128 threads cover 8 pairs x 16 columns)
  float sq0 = 0.f, sq1 = 0.f;
#pragma unroll
  for (int i = 0; i < kWordsPerThread; ++i) {
    const int w = tid + i * kGvConsumers * 32;
    const int col = w >> 3, tok0 = (w & 7) * 2;
    const int n = row0 + col;
    if (n >= p.N) continue;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int tok = tok0 + e;
      if (tok >= p.M) continue;
      float val = rbf(e ? s1[i] : s0[i]);
      if (p.R) val = bf2f(p.R[(int64_t)tok * p.ldc + n]) + val;
      const __nv_bfloat16 o = f2bf(val);
      p.C[(int64_t)tok * p.ldc + n] = o;
      const float vr = bf2f(o);
      if (e) sq1 = fmaf(vr, vr, sq1);
      else sq0 = fmaf(vr, vr, sq0);
    }
  }
  if (p.ss_out) {
    // per-tile sums of squares of the stored outputs (identical on every rank)
    // for the RMSNorm fused into the next projection
    __shared__ float ssw[kGvConsumers][16];
    sq0 += __shfl_xor_sync(0xffffffffu, sq0, 8);
    sq0 += __shfl_xor_sync(0xffffffffu, sq0, 16);
    sq1 += __shfl_xor_sync(0xffffffffu, sq1, 8);
    sq1 += __shfl_xor_sync(0xffffffffu, sq1, 16);
    const int lane = tid & 31, warp = tid >> 5;
    if (lane < 8) {
      ssw[warp][2 * lane] = sq0;
      ssw[warp][2 * lane + 1] = sq1;
    }
    consumer_bar();
    if (tid < 16)
      p.ss_out[tile * 16 + tid] = ssw[0][tid] + ssw[1][tid] + ssw[2][tid] + ssw[3][tid];
  }
  if (tid == 0) cm.counters[tile] = f;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Normaliser warp of the fused-RMSNorm projection: computes every token's
// inverse RMS (from the producer kernel's per-tile sums of squares, or from
// the rows of A), then, for each ring stage, rescales the staged activation
// tile in place, x -> bf16(bf16(x * r_tok) * norm_w[k]) (model_fused.py:37-40),
// and releases the stage to the consumers through ready[s].  Lane l owns the
// 16-byte chunk c = l % 8 (8 K elements) of token rows l / 8 + 4j.
template <int NT>
__device__ __forceinline__ void gemv_normaliser(const GemvParams& p, uint32_t ring_base,
                                                uint64_t* full, uint64_t* ready, int kb_begin,
                                                int nkb, int lane) {
  __shared__ float rs[16];
  pdl_wait();  // sums of squares / rows of A come from the previous kernel
  if (p.ss_in) {
    if (lane < p.M) {
      float ss = 0.f;  // fixed order: tile 0, 1, ...
      for (int t2 = 0; t2 < p.ss_tiles; ++t2) ss += p.ss_in[t2 * 16 + lane];
      rs[lane] = 1.0f / sqrtf(ss / (float)p.K + p.eps);
    }
  } else {
    for (int tok = 0; tok < p.M; ++tok) {
      const uint4* xr = reinterpret_cast<const uint4*>(p.A + (int64_t)tok * p.K);
      float ss = 0.f;
#pragma unroll 8
      for (int v = lane; v < p.K / 8; v += 32) {
        const uint4 u = xr[v];
        const uint32_t us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(us[j]);
          ss = fmaf(f.x, f.x, ss);
          ss = fmaf(f.y, f.y, ss);
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) rs[tok] = 1.0f / sqrtf(ss / (float)p.K + p.eps);
    }
  }
  __syncwarp();
  constexpr int kRowsPerLane = NT * 2;
  const int c = lane & 7;
  float r[kRowsPerLane];
#pragma unroll
  for (int j = 0; j < kRowsPerLane; ++j) {
    const int tok = (lane >> 3) + 4 * j;
    r[j] = tok < p.M ? rs[tok] : 0.f;  // rows past M stay zero
  }
  auto wchunk = [&](int i) {
    const int k = (kb_begin + i) * kGvBK + c * 8;
    return k < p.K ? __ldg(reinterpret_cast<const uint4*>(p.norm_w + k)) : make_uint4(0, 0, 0, 0);
  };
  uint4 wn_next = nkb > 0 ? wchunk(0) : make_uint4(0, 0, 0, 0);
  for (int i = 0; i < nkb; ++i) {
    const int s = i % kGvStages;
    const uint32_t ph = (i / kGvStages) & 1;
    const uint4 wn = wn_next;
    if (i + 1 < nkb) wn_next = wchunk(i + 1);  // one stage ahead
    if (!mbar_wait(&full[s], ph, p.err, 0x303)) break;
    const uint32_t xbase = ring_base + s * kGvStageBytes + kGvWBytes;
#pragma unroll
    for (int j = 0; j < kRowsPerLane; ++j) {
      const int row = (lane >> 3) + 4 * j;
      const uint32_t addr = xbase + row * 128 + ((c ^ (row & 7)) << 4);
      sts128(addr, rms_scale_chunk(lds128(addr), r[j], wn));
    }
    mbar_arrive(&ready[s]);  // all 32 lanes arrive: each lane's stores are released
  }
}

template <int NT, int EPI, int FL>
__global__ void __launch_bounds__(gv_threads(FL)) gemv_tma_kernel(
    const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
    GemvParams p) {
  constexpr bool kNorm = (FL & kFlNorm) != 0;
  constexpr bool kSsOut = (FL & kFlSsOut) != 0 && EPI == Q3_EPI_RESIDUAL;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kGvStages * kGvStageBytes);
  uint64_t* empty = full + kGvStages;
  uint64_t* ready = empty + kGvStages;  // kNorm: stage normalised
  __shared__ float red[kGvConsumers][NT * 4][32];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int row0 = tile * kGvRows;
  const int kb_begin = blockIdx.y * p.kb_per_cta;
  const int nkb_total = (p.K + kGvBK - 1) / kGvBK;
  const int kb_end = min(nkb_total, kb_begin + p.kb_per_cta);
  const int nkb = max(0, kb_end - kb_begin);

  // Let the next kernel start its prologue early -- except around the
  // all-reduce, whose cross-GPU exchange is latency-critical: there the
  // dependents start when the CTAs exit.
  if constexpr (EPI != kEpiAllReduce) pdl_launch();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kGvStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGvConsumers);
      if constexpr (kNorm) mbar_init(&ready[s], 32);
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  __syncthreads();

  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

  if (warp == kGvConsumers) {
    // ---------------- producer ----------------
    if (lane == 0) {
      constexpr uint32_t kTx = kGvWBytes + NT * 8 * kGvBK * 2;
      // Weights never depend on the previous kernel: fill the ring with W
      // tiles before waiting for it, then add the activation tiles.
      const int pre = min(nkb, kGvStages);
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], kTx);
        tma_load_2d(ring + i * kGvStageBytes, &tmW, &full[i], (kb_begin + i) * kGvBK, row0,
                    kCacheEvictFirst);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(ring + i * kGvStageBytes + kGvWBytes, &tmX, &full[i],
                    (kb_begin + i) * kGvBK, 0, kCacheEvictLast);
      for (int i = pre; i < nkb; ++i) {
        const int s = i % kGvStages;
        const uint32_t ph = (i / kGvStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, p.err, 0x301)) break;
        uint8_t* st = ring + s * kGvStageBytes;
        mbar_arrive_expect_tx(&full[s], kTx);
        tma_load_2d(st, &tmW, &full[s], (kb_begin + i) * kGvBK, row0, kCacheEvictFirst);
        tma_load_2d(st + kGvWBytes, &tmX, &full[s], (kb_begin + i) * kGvBK, 0,
                    kCacheEvictLast);
      }
    }
  } else if (warp > kGvConsumers) {
    // ---------------- normaliser (kNorm only) ----------------
    if constexpr (kNorm) gemv_normaliser<NT>(p, smem_u32(ring), full, ready, kb_begin, nkb, lane);
  } else {
    // ---------------- consumers ----------------
    pdl_wait();  // the epilogue reads R and writes C
    const int g = lane >> 2, t = lane & 3;
    const int r0 = warp * 16 + g, r1 = r0 + 8;
    const uint32_t ring_base = smem_u32(ring);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % kGvStages;
      const uint32_t ph = (i / kGvStages) & 1;
      if (!mbar_wait(kNorm ? &ready[s] : &full[s], ph, p.err, 0x302)) break;
      const uint32_t base = ring_base + s * kGvStageBytes;
      const uint32_t xbase = base + kGvWBytes;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int c = 2 * t + h;
        const uint4 a0 = lds128(base + r0 * 128 + ((c ^ (r0 & 7)) << 4));
        const uint4 a1 = lds128(base + r1 * 128 + ((c ^ (r1 & 7)) << 4));
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          // token rows past M and K past the end arrive zero-filled by TMA
          const int tok = n * 8 + g;
          const uint4 x = lds128(xbase + tok * 128 + ((c ^ (tok & 7)) << 4));
          mma_bf16_16816(acc[n], a0.x, a1.x, a0.y, a1.y, x.x, x.y);
          mma_bf16_16816(acc[n], a0.z, a1.z, a0.w, a1.w, x.z, x.w);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) red[warp][n * 4 + e][lane] = acc[n][e];
  }

  // ---------------- split-K reduction over the cluster ----------------
  const uint32_t csize = cluster_nctarank();
  const uint32_t crank = cluster_ctarank();
  if (csize > 1) cluster_sync_all();
  else __syncthreads();
  // All-reduce epilogue with early dependents: this CTA's weight stream is
  // done, so the next kernel may launch and start its own weight stream
  // while this one exchanges partials with its peers.
  if constexpr (EPI == kEpiAllReduce) {
    if (p.comm.early_dependents) pdl_launch();
  }
  if (crank == 0 && warp < kGvConsumers) {
    const int g = lane >> 2, t = lane & 3;
    float v[NT * 4];
#pragma unroll
    for (int i = 0; i < NT * 4; ++i) v[i] = red[warp][i][lane];
    const uint32_t local = smem_u32(&red[warp][0][lane]);
    for (uint32_t r = 1; r < csize; ++r) {
      const uint32_t remote = map_shared_rank(local, r);
#pragma unroll
      for (int i = 0; i < NT * 4; ++i) v[i] += ld_shared_cluster_f32(remote + i * 32 * 4);
    }
    // c0,c1 = (row g, tokens 2t, 2t+1); c2,c3 = (row g+8, tokens 2t, 2t+1)
    const int rbase = row0 + warp * 16;
    if constexpr (EPI == kEpiAllReduce) {
      __shared__ __align__(16) __nv_bfloat16 part[kArCols][kArTokens];
      __shared__ uint32_t f_s;
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = warp * 16 + g + (e >= 2 ? 8 : 0);
          const int tok = n * 8 + 2 * t + (e & 1);
          part[col][tok] = f2bf((n < NT) ? v[(n < NT ? n : 0) * 4 + e] : 0.f);
        }
      consumer_bar();
      allreduce_tile(p, tile, row0, part, &f_s);
    } else if constexpr (EPI == Q3_EPI_SWIGLU) {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int tok0 = n * 8 + 2 * t;
        const int f = rbase / 2 + g;  // rows g / g+8 are gate / up of feature f
        if (rbase + g + 8 < p.N) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int tok = tok0 + e;
            if (tok < p.M) {
              const float gt = rbf(v[n * 4 + e]), up = rbf(v[n * 4 + 2 + e]);
              p.C[(int64_t)tok * p.ldc + f] = f2bf(silu_ref(gt) * up);
            }
          }
        }
      }
    } else {
      // squares of the stored outputs, per token (2 tokens x NT per lane)
      float sq[NT][2];
#pragma unroll
      for (int n = 0; n < NT; ++n) sq[n][0] = sq[n][1] = 0.f;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int tok0 = n * 8 + 2 * t;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = rbase + g + (e >= 2 ? 8 : 0);
          const int tok = tok0 + (e & 1);
          if (tok < p.M && row < p.N) {
            float val = rbf(v[n * 4 + e]);
            if (EPI == Q3_EPI_RESIDUAL) val = bf2f(p.R[(int64_t)tok * p.ldc + row]) + val;
            const __nv_bfloat16 o = f2bf(val);
            p.C[(int64_t)tok * p.ldc + row] = o;
            if constexpr (kSsOut) {
              const float vr = bf2f(o);
              sq[n][e & 1] = fmaf(vr, vr, sq[n][e & 1]);
            }
          }
        }
      }
      if constexpr (kSsOut) {
        // reduce over the 8 lanes that share t (rows g), then over the 4 warps
        __shared__ float ssw[kGvConsumers][16];
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float x = sq[n][e];
            x += __shfl_xor_sync(0xffffffffu, x, 4);
            x += __shfl_xor_sync(0xffffffffu, x, 8);
            x += __shfl_xor_sync(0xffffffffu, x, 16);
            if (g == 0) ssw[warp][n * 8 + 2 * t + e] = x;
          }
        if (NT == 1 && g == 0) ssw[warp][8 + 2 * t] = ssw[warp][9 + 2 * t] = 0.f;
        consumer_bar();
        const int tid = warp * 32 + lane;
        if (tid < 16)
          p.ss_out[tile * 16 + tid] = ssw[0][tid] + ssw[1][tid] + ssw[2][tid] + ssw[3][tid];
      }
    }
  }
  // keep every CTA's shared memory alive until rank 0 has read it
  if (csize > 1) cluster_sync_all();
}

template <int NT, int EPI, int FL>
static int launch_gemv_t(const void* A, const void* W, void* C, const void* R, int M, int N,
                         int K, cudaStream_t s, const CommDev* comm, const GemvOpts& o) {
  auto kern = gemv_tma_kernel<NT, EPI, FL>;
  constexpr int kThreads = gv_threads(FL);
  CUtensorMap tw, tx;
  int rc = cached_tmap_2d(&tw, W, N, K, kGvRows, kGvBK);
  if (rc) return rc;
  rc = make_tmap_2d(&tx, A, M, K, NT * 8, kGvBK);
  if (rc) return rc;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    Q3_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kGvSmem));
    attr_set[dev] = true;
  }
  const int tiles = (N + kGvRows - 1) / kGvRows;
  const int nkb = (K + kGvBK - 1) / kGvBK;
  // Split K over a cluster as far as the grid still fits in ONE wave of
  // resident CTAs (a second, partial wave would double the tail), keeping at
  // least 4 K blocks per CTA.
  static int per_sm_cache[64] = {0};
  int per_sm = (dev >= 0 && dev < 64) ? per_sm_cache[dev] : 0;
  if (per_sm == 0) {
    Q3_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads,
                                                                kGvSmem));
    if (dev >= 0 && dev < 64) per_sm_cache[dev] = per_sm;
  }
  const int slots = (per_sm > 0 ? per_sm : 1) * num_sms();
  int ks = 1;
  while (ks < 8 && tiles * ks * 2 <= slots && nkb / (ks * 2) >= 4) ks *= 2;
  // The all-reduce epilogue waits on the same tile of every peer, so every
  // CTA of the grid must be resident at once.
  if (EPI == kEpiAllReduce && tiles * ks > slots)
    return fail(Q3_ERR_UNSUPPORTED, "q3_gemm_ar: %d tiles exceed one wave (%d CTAs)", tiles,
                slots);
  GemvParams p;
  p.A = (const __nv_bfloat16*)A;
  p.C = (__nv_bfloat16*)C;
  p.R = (const __nv_bfloat16*)R;
  p.M = M; p.N = N; p.K = K;
  p.ldc = EPI == Q3_EPI_SWIGLU ? N / 2 : N;
  p.kb_per_cta = (nkb + ks - 1) / ks;
  p.err = device_error_word();
  p.comm = comm ? *comm : CommDev{};
  p.norm_w = (const __nv_bfloat16*)o.norm_w;
  p.eps = o.eps;
  p.ss_in = o.ss_in;
  p.ss_tiles = o.ss_tiles;
  p.ss_out = o.ss_out;
  return launch_ex(kern, dim3(tiles, ks, 1), dim3(kThreads), kGvSmem, s, ks, tw, tx, p);
}

template <int NT, int EPI>
static int launch_gemv_fl(const void* A, const void* W, void* C, const void* R, int M, int N,
                          int K, cudaStream_t s, const GemvOpts& o) {
  if (o.norm_w) {
    if (o.ss_out) return fail(Q3_ERR_UNSUPPORTED, "decode projection: norm_w with ss_out");
    return launch_gemv_t<NT, EPI, kFlNorm>(A, W, C, R, M, N, K, s, nullptr, o);
  }
  if (o.ss_out) {
    if constexpr (EPI == Q3_EPI_RESIDUAL)
      return launch_gemv_t<NT, EPI, kFlSsOut>(A, W, C, R, M, N, K, s, nullptr, o);
    return fail(Q3_ERR_INVALID, "decode projection: ss_out needs the residual epilogue");
  }
  return launch_gemv_t<NT, EPI, 0>(A, W, C, R, M, N, K, s, nullptr, o);
}

int launch_gemv(const void* A, const void* W, void* C, const void* R, int M, int N, int K,
                int epilogue, cudaStream_t s, const GemvOpts& o) {
  if (M < 1 || M > 16) return fail(Q3_ERR_INVALID, "decode projection needs 1 <= M <= 16");
  if (K % 8 != 0) return fail(Q3_ERR_INVALID, "decode projection needs K %% 8 == 0");
  const bool two = M > 8;
  switch (epilogue) {
    case Q3_EPI_NONE:
      return two ? launch_gemv_fl<2, Q3_EPI_NONE>(A, W, C, R, M, N, K, s, o)
                 : launch_gemv_fl<1, Q3_EPI_NONE>(A, W, C, R, M, N, K, s, o);
    case Q3_EPI_RESIDUAL:
      return two ? launch_gemv_fl<2, Q3_EPI_RESIDUAL>(A, W, C, R, M, N, K, s, o)
                 : launch_gemv_fl<1, Q3_EPI_RESIDUAL>(A, W, C, R, M, N, K, s, o);
    default:
      return two ? launch_gemv_fl<2, Q3_EPI_SWIGLU>(A, W, C, R, M, N, K, s, o)
                 : launch_gemv_fl<1, Q3_EPI_SWIGLU>(A, W, C, R, M, N, K, s, o);
  }
}

// Q3VL_AR_EARLY_PDL=1: the all-reduce projection lets its dependent kernel
// launch once its own weights are consumed, before the exchange with peers.
static int ar_early_dependents() {
  static const int on = [] {
    const char* v = getenv("Q3VL_AR_EARLY_PDL");
    return (v && v[0] == '1') ? 1 : 0;
  }();
  return on;
}

int launch_gemv_ar(const void* A, const void* W, void* C, const void* R, int M, int N, int K,
                   float* ss_out, const CommDev& comm, cudaStream_t s) {
  if (M < 1 || M > 16) return fail(Q3_ERR_INVALID, "decode projection needs 1 <= M <= 16");
  GemvOpts o;
  o.ss_out = ss_out;
  CommDev cd = comm;
  cd.early_dependents = ar_early_dependents();
  return M > 8 ? launch_gemv_t<2, kEpiAllReduce, 0>(A, W, C, R, M, N, K, s, &cd, o)
               : launch_gemv_t<1, kEpiAllReduce, 0>(A, W, C, R, M, N, K, s, &cd, o);
}

}  // namespace q3
