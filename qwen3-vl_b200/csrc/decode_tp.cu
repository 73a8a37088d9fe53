// a12/a13 + 8(e): every decoder layer of one greedy decode step in ONE launch
// per GPU, with the tensor-parallel all-reduce of o_proj and down inside it.
//
// Reference: Qwen3VLDecoderFused.forward_layer (model_fused.py:234-277) at
// S = 1 for every layer of decode_step (:295-300), including the two
// dist.all_reduce calls per layer (:267, :274) over the ranks' row shards
// (loader_fused.py:87-109).
//
// Why: at tensor-parallel decode a rank streams only a few MB per projection
// (a TP8 rank: 53 MB per layer), while every kernel launch costs several
// microseconds of ramp, drain and dependency resolution whatever it streams.
// Here one CTA per SM runs the whole step; the phases of a layer are
//   QKV      rmsnorm(x) @ Wqkv          -> qkv          (raw, bf16)
//   ATT      per (sequence, KV head, split): QK-RMSNorm + RoPE of q and of the
//            new k, KV write, attention over the cache; the split holding the
//            last arrival merges the splits               -> attn
//   O        attn @ Wo, all-reduce, + x                   -> x2
//   GU       rmsnorm(x2) @ Wgate_up, silu(gate) * up      -> h
//   DN       h @ Wdown, all-reduce, + x2                  -> x
// separated by grid-wide barriers (an arrival counter in global memory).
//
// Work split.  A projection's weight rows are cut into granules of 8 rows,
// and CTA c owns a contiguous, equal share of the granules with the full
// reduction length, so no partial sum ever crosses CTAs.  The o_proj and down
// phases give every CTA the same rows on every rank, which makes the
// all-reduce a per-CTA exchange: the CTA pushes its rows' bf16 partials into
// every peer's inbox over NVLink (8-byte words carrying two values and the
// call number, so a word is its own arrival flag), then waits for the peers'
// words of the same rows and sums the ranks in rank order in fp32; every
// rank therefore holds identical bits.  Call numbers grow by two per layer
// and by 2 x layers per launch (a counter in device memory), so stale words
// never match; two parities of inbox slots let a peer run one call ahead.
//
// Warps: 0-3 consume (tensor-core mma.sync on staged weight tiles, softmax,
// epilogues, the exchange), warp 4 is the TMA producer.  The producer walks
// the same static schedule as the consumers and fills a ring of 16 KB slots
// with every weight tile and old cache tile this CTA will read, across phase
// and layer boundaries: none of them depends on the step's activations, so
// HBM keeps streaming while the consumers sit at a barrier.  The activations
// of a phase (x, attn, x2 or h: at most 8 tokens) are staged once per phase
// into shared memory by the consumers, with the RMSNorm applied as they are
// staged; the SwiGLU is applied once, by the gate/up CTA that owns both halves
// of a feature.
//
// Every wait is bounded: a grid barrier or ring wait gives up after 2 s, a
// peer word after the communicator's wait limit; the kernel then records the
// code in the device error word, raises an abort flag that every later wait
// checks, and unwinds.
#include <cstdlib>
#include <vector>

#include "comm.h"
#include "common.cuh"

namespace q3 {
namespace tp {

constexpr int kCons = 4;                      // consumer warps
constexpr int kThreads = (kCons + 1) * 32;    // + the TMA producer warp
constexpr int kSlot = 16384;                  // ring slot
constexpr int kMaxSlots = 12;
constexpr int kTok = 8;                       // tokens per step, at most
constexpr int kGran = 8;                      // weight rows per granule
constexpr int kMaxGran = 16;                  // granules per CTA in one phase
constexpr int kMaxPairs = kMaxGran / 2;       // granule pairs (16-row MMA tiles)
constexpr int kHD = 128;
constexpr int kPos = 64;                      // cache positions per attention tile
constexpr int kMaxG = 8;                      // query heads per KV head
constexpr int kPairs = kTok / 2;              // token pairs per exchanged row
constexpr int kMaxSplitsMerge = 256;          // attention splits of one pair, at most
constexpr int kSmemLimit = 232448;
enum { kQKV = 0, kATT = 1, kO = 2, kGU = 3, kDN = 4, kPhases = 5 };

constexpr int kDepths = 4;                    // weight boxes of 1, 2, 4 or 8 K blocks
struct alignas(64) LayerMaps {
  // qkv, o, gate_up, down ([N, K] K-major) as 3-D (64, N, K / 64) views with
  // boxes of all of a CTA's rows (8 g, for the phase's two granule counts g,
  // the Params' gbox) x 64 x 2^d K blocks (d = 0..3): one copy moves a CTA's
  // whole share of up to 8 K blocks, laid out [K block][row][64]
  CUtensorMap w[4][2][kDepths];
  CUtensorMap k, v;  // caches [B * Hkv * max_seq, 128], boxes of 64 rows x 64
};
struct LayerPtrs {
  const __nv_bfloat16* in_norm;
  const __nv_bfloat16* post_norm;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
};

struct Params {
  const LayerMaps* maps;
  const LayerPtrs* lp;
  int n_layers, M, H, Hq, Hkv, I;
  int64_t max_seq;
  float eps, scale_log2;
  const __nv_bfloat16* cos;  // [rope_rows, 64]
  const __nv_bfloat16* sin;
  int64_t rope_rows, rope_delta;
  const int32_t* kv_len_dev;  // new position + 1
  // paged caches (table != nullptr): the caches are page pools [num_pages,
  // Hkv, page_tokens, 128] and sequence b's position t lives in page
  // table[b * table_stride + t / page_tokens]
  const int32_t* table;
  int table_stride, page_tokens;
  int64_t num_pages;
  __nv_bfloat16* X;           // [M, H] residual stream (in: embedded tokens, out: last layer)
  __nv_bfloat16* X2;          // [M, H]
  __nv_bfloat16* qkv;         // [M, (Hq + 2 Hkv) * 128]
  __nv_bfloat16* attn;        // [M, Hq * 128]
  __nv_bfloat16* gu;          // h = silu(gate) * up [M, I]
  float* apart;               // [grid][kMaxG][kHD + 2] attention split partials
  float* ssx;                 // [grid][8] per-CTA sums of squares of x's rows (down epilogue)
  float* ssx2;                // [grid][8] the same for x2 (o_proj epilogue)
  int* pair_cnt;              // [M * Hkv] split arrivals (zeroed before each launch)
  unsigned* gbar;             // grid barrier arrivals (zeroed before each launch)
  unsigned* step_no;          // launches so far (exchange call numbers)
  uint2* inbox[kMaxRanks];    // every rank's exchange buffer (own included)
  int rank, world;
  uint64_t wait_ns;
  int* err;
  int* abort;
  int x_stride;               // bytes per staged-activation row
  int x_bytes;                // staged-activation buffer
  int nslots;
  int gbox[4][2];             // granule counts the weight maps' boxes were made for
  int inflight;               // producer: slots issued but not landed, at most
  int prod_sleep, cons_sleep; // ring-wait back-off (ns) of the producer and the consumers
};

// --------------------------------------------------------- work geometry
__host__ __device__ inline int proj_n(const Params& p, int ph) {
  return ph == kQKV ? (p.Hq + 2 * p.Hkv) * kHD : ph == kGU ? 2 * p.I : p.H;
}
__host__ __device__ inline int proj_k(const Params& p, int ph) {
  return ph == kO ? p.Hq * kHD : ph == kDN ? p.I : p.H;
}
__host__ __device__ inline int widx(int ph) { return ph == kQKV ? 0 : ph == kO ? 1 : ph == kGU ? 2 : 3; }
// granules [lo, hi) of CTA c out of ng over C CTAs
__host__ __device__ inline void gran_range(int ng, int c, int C, int& lo, int& hi) {
  lo = (int)((int64_t)ng * c / C);
  hi = (int)((int64_t)ng * (c + 1) / C);
}
// this CTA's granules of a projection phase (the step kernel's gate/up rows
// come in granules of 4 gate rows then the 4 up rows of the same 4 features,
// so every granule holds whole features and the CTA that owns it applies the
// SwiGLU)
__host__ __device__ inline void phase_range(const Params& p, int ph, int c, int C, int& lo,
                                            int& hi) {
  gran_range(proj_n(p, ph) / kGran, c, C, lo, hi);
}
// 64-wide K blocks per ring slot for g granules: as many as fill the 16 KB
// slot (a stage of n blocks is loaded by one copy per set bit of n, boxes of
// 8, 4, 2 and 1 blocks): the bytes in flight per SM, not the copies, bound
// the stream
__host__ __device__ inline int kb_per_stage(int g, int nkb) {
  const int k = 16 / g;
  return k < nkb ? k : nkb;
}
// map index of a box of 2^d blocks
__host__ __device__ inline int depth_index(int depth) {
  return depth >= 8 ? 3 : depth >= 4 ? 2 : depth >= 2 ? 1 : 0;
}
struct AttPlan {
  int splits, chunk;
};
// splits of each (sequence, KV head) pair over at most C CTAs, in whole tiles
__host__ __device__ inline AttPlan att_plan(int pairs, int L, int C) {
  int sp = C / pairs;
  if (sp < 1) sp = 1;
  const int max_sp = (L + kPos - 1) / kPos;
  if (sp > max_sp) sp = max_sp;
  int ch = (L + sp - 1) / sp;
  ch = (ch + kPos - 1) / kPos * kPos;
  sp = (L + ch - 1) / ch;
  return AttPlan{sp, ch};
}

// ------------------------------------------------------------- helpers
__device__ __forceinline__ bool aborted(const Params& p) {
  return *reinterpret_cast<const volatile int*>(p.abort) != 0;
}
__device__ __forceinline__ void raise_abort(const Params& p, int code) {
  report_timeout(p.err, code);
  atomicExch(p.abort, 1);
}
// cache row ([rows, 128] view) of sequence b, KV head kvh, position t; -1 for
// a table entry outside the pool
__device__ __forceinline__ int64_t kv_row(const Params& p, int b, int kvh, int t) {
  if (p.table == nullptr) return ((int64_t)b * p.Hkv + kvh) * p.max_seq + t;
  const int pg = p.table[(int64_t)b * p.table_stride + t / p.page_tokens];
  if (pg < 0 || pg >= p.num_pages) return -1;
  return ((int64_t)pg * p.Hkv + kvh) * p.page_tokens + t % p.page_tokens;
}
__device__ __forceinline__ void cons_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kCons * 32) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* q) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(q) : "memory");
  return v;
}
// mbarrier wait of one thread that also gives up once the kernel aborted;
// between polls it sleeps sleep_ns, so that a waiting warp leaves its
// scheduler's issue slots to the warps that work.  The polling loop is out of
// line: every call site then costs a few instructions of the step's text.
__device__ __noinline__ bool ring_wait_slow(const Params& p, uint64_t* bar, uint32_t parity,
                                            int code, int sleep_ns) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (sleep_ns) __nanosleep(sleep_ns);
    if ((++spins & 255u) == 0) {
      if (aborted(p)) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_abort(p, code);
        return false;
      }
    }
  }
  return true;
}
__device__ __forceinline__ bool ring_wait(const Params& p, uint64_t* bar, uint32_t parity,
                                          int code, int sleep_ns = 0) {
  return mbar_try_wait(bar, parity) || ring_wait_slow(p, bar, parity, code, sleep_ns);
}
// the same, with the outcome shared by the whole warp
__device__ __forceinline__ bool ring_wait_warp(const Params& p, uint64_t* bar, uint32_t parity,
                                               int code) {
  return __all_sync(0xffffffffu, ring_wait(p, bar, parity, code, p.cons_sleep));
}
// Grid-wide barrier of the consumer threads of every CTA.
__device__ __forceinline__ void grid_sync(const Params& p, unsigned& target) {
  target += gridDim.x;
  cons_bar();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(p.gbar, 1u);
    if (ld_acquire_gpu_u32(p.gbar) < target) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_gpu_u32(p.gbar) < target) {
        __nanosleep(20);
        if ((++spins & 63u) == 0) {
          if (aborted(p)) break;
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            raise_abort(p, 0x801);
            break;
          }
        }
      }
    }
  }
  cons_bar();
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
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
// 16-byte chunk c (0..15 over 128 dims) of position row r of a K or V slot
// (two 64-dim TMA boxes of 64 rows, 128-byte swizzle)
__device__ __forceinline__ uint32_t kv_off(int r, int c) {
  return (c >> 3) * 8192 + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}
__device__ __forceinline__ void st_word(uint2* q, uint32_t data, uint32_t flag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(q), "r"(data), "r"(flag)
               : "memory");
}
__device__ __forceinline__ uint2 ld_word(const uint2* q) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(q)
               : "memory");
  return v;
}
// inbox word of (parity, source rank, hidden row, token pair)
__device__ __forceinline__ size_t word_at(const Params& p, int par, int src, int row, int tp) {
  return (((size_t)par * kMaxRanks + src) * p.H + row) * kPairs + tp;
}

// -------------------------------------------------------------- producer
// Keeps at most p.inflight slots issued but not landed.  The HBM stream needs
// only a few tens of KB in flight per SM to run at full bandwidth; more only
// lengthens the memory system's queues, and every latency-bound access of the
// step (activation staging from L2, the grid barrier, the peer exchange)
// waits behind them.  Landed slots may still fill the whole ring.
__device__ __forceinline__ bool throttle(const Params& p, uint64_t* full, uint32_t it) {
  if (it < (uint32_t)p.inflight) return true;
  const uint32_t k = it - (uint32_t)p.inflight;
  return ring_wait(p, &full[k % p.nslots], (k / p.nslots) & 1, 0x806, p.prod_sleep);
}
// Issues every TMA load of this CTA's schedule in consumption order.
// Issues every TMA load of this CTA's schedule in consumption order.
// Issues every TMA load of this CTA's schedule in consumption order.
__device__ void producer(const Params& p, uint8_t* ring, uint64_t* full, uint64_t* empty, int L,
                         AttPlan ap) {
  const int C = gridDim.x, c = blockIdx.x, ns = p.nslots;
  uint32_t it = 0;
  bool ok = true;
  for (int l = 0; ok && l < p.n_layers && !aborted(p); ++l) {
    const LayerMaps* mp = p.maps + l;
#pragma unroll 1
    for (int ph = 0; ok && ph < kPhases; ++ph) {
      if (ph == kATT) {
        const int pairs = p.M * p.Hkv;
        if (c < pairs * ap.splits) {
          const int pair = c / ap.splits, split = c % ap.splits;
          const int b = pair / p.Hkv, kvh = pair % p.Hkv;
          const int start = split * ap.chunk, end = min(start + ap.chunk, L - 1);
          for (int t0 = start; ok && t0 < end; t0 += kPos) {
            int64_t r64 = kv_row(p, b, kvh, t0);  // a tile never straddles two pages
            if (r64 < 0) {
              raise_abort(p, 0x809);
              r64 = 0;
            }
            const int row = (int)r64;
            for (int kv = 0; ok && kv < 2; ++kv) {
              const int s = (int)(it % ns);
              if (!ring_wait(p, &empty[s], ((it / ns) & 1) ^ 1, 0x802, p.prod_sleep) ||
                  !throttle(p, full, it)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&full[s], kSlot);
              const CUtensorMap* m = kv ? &mp->v : &mp->k;
              tma_load_2d(ring + s * kSlot, m, &full[s], 0, row, kCacheEvictFirst);
              tma_load_2d(ring + s * kSlot + kSlot / 2, m, &full[s], 64, row, kCacheEvictFirst);
              ++it;
            }
          }
        }
        continue;
      }
      const int nkb = proj_k(p, ph) / 64;
      int lo, hi;
      phase_range(p, ph, c, C, lo, hi);
      const int g = hi - lo;
      if (g == 0) continue;
      const int kbs = kb_per_stage(g, nkb);
      const int wi = widx(ph);
      const CUtensorMap* mg = &mp->w[wi][g == p.gbox[wi][1] ? 1 : 0][0];
      for (int kb0 = 0; kb0 < nkb; kb0 += kbs) {
        const int n = min(kbs, nkb - kb0);
        const int s = (int)(it % ns);
        if (!ring_wait(p, &empty[s], ((it / ns) & 1) ^ 1, 0x803, p.prod_sleep) ||
            !throttle(p, full, it)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], (uint32_t)(g * n * 1024));
        // copies of 8, 4, 2 and 1 K blocks, largest first (16 blocks: two of
        // 8): blocks [q, q + 2^d) land at q * g KB, the consumers' [K block][row]
        // order
#pragma unroll 1
        for (int q = 0; q < n;) {
          const int r = n - q;
          const int d = r >= 8 ? 3 : r >= 4 ? 2 : r >= 2 ? 1 : 0;
          tma_load_3d(ring + s * kSlot + q * g * 1024, mg + d, &full[s], 0, lo * kGran, kb0 + q,
                      kCacheEvictFirst);
          q += 1 << d;
        }
        ++it;
      }
    }
  }
  // the consumers may leave early after an abort: let the loads in flight land
  // before the CTA exits (bounded waits, no error code)
  const uint32_t first = it > (uint32_t)ns ? it - ns : 0;
  for (uint32_t k = first; k < it; ++k) mbar_wait(&full[k % ns], (k / ns) & 1, nullptr, 0);
}

// ------------------------------------------------------------- staging
// pin(x...) makes values opaque at this point of each call, so that the
// address arithmetic derived from them stays inside the phase: left free, the
// compiler hoists every phase's addresses out of the layer loop and keeps them
// live across the whole step, which spills registers.
__device__ __forceinline__ void pin1(int& a) { asm volatile("" : "+r"(a)); }
__device__ __forceinline__ void pin1(uint32_t& a) { asm volatile("" : "+r"(a)); }
template <class T>
__device__ __forceinline__ void pin1(T*& a) {
  asm volatile("" : "+l"(a));
}
template <class... T>
__device__ __forceinline__ void pin(T&... a) {
  (pin1(a), ...);
}
// the thread index, opaque (see pin)
__device__ __forceinline__ int tid_pinned() {
  int t = threadIdx.x;
  pin1(t);
  return t;
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Rows 0..M-1 of a [M, K] activation into the staging buffer (row stride
// x_stride bytes), rows M..7 zero; with a weight w, RMSNorm
// (model_fused.py:37-40: x * rsqrt(mean(x^2) + eps) rounded to bf16, times w
// rounded to bf16).
// The activations come from L2 (written by other CTAs in this launch): one
// thread issues a bulk copy per row (and one for w, as a ninth row) onto the
// stage barrier `sbar`.  The RMSNorm needs the rows' sums of squares: with
// `ssp` ([CTAs][8], the per-CTA partials that the producing all-reduce
// epilogue wrote) they arrive with the rows; without it (the first layer's
// input) thread t sums its 16-byte chunks t, t + 128, ... of every row.  The
// four warps' sums meet in `nscr` ([4][8] floats, then the [8] reciprocal
// RMS values) before the scaling pass.  Ends with the consumers' barrier.
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ void stage(const Params& p, uint32_t xs, const __nv_bfloat16* src, int K,
                      const __nv_bfloat16* w, const float* ssp, float* nscr, uint64_t* sbar,
                      uint32_t& sphase) {
  const int tid = tid_pinned();
  pin(xs, src, w);
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int kT = kCons * 32;
  const int cpr = K / 8;  // 16-byte chunks per row
  const int xst = p.x_stride;
  const uint32_t ss_buf = xs + (kTok + 1) * xst;  // [CTAs][8] partial sums
  if (tid == 0) {
    const uint32_t rowb = (uint32_t)K * 2;
    const int nr = min(p.M, kTok);
    mbar_arrive_expect_tx(sbar, rowb * (nr + (w ? 1 : 0)) +
                                    (ssp ? (uint32_t)gridDim.x * kTok * 4 : 0u));
    for (int r = 0; r < nr; ++r) bulk_g2s(xs + r * xst, src + (int64_t)r * K, rowb, sbar);
    if (w) bulk_g2s(xs + kTok * xst, w, rowb, sbar);
    if (ssp) bulk_g2s(ss_buf, ssp, gridDim.x * kTok * 4, sbar);
  }
  for (int i = p.M * cpr + tid; i < kTok * cpr; i += kT)  // rows past M: zeros
    sts128(xs + (i / cpr) * xst + (i % cpr) * 16, make_uint4(0, 0, 0, 0));
  ring_wait(p, sbar, sphase, 0x808);  // after an abort the rows are not used
  sphase ^= 1u;
  cons_bar();
  if (w == nullptr) return;
  float ss[kTok];
#pragma unroll
  for (int r = 0; r < kTok; ++r) ss[r] = 0.f;
  if (ssp) {
    // thread (warp, lane): token lane & 7, CTAs (lane >> 3) + 4 warp + 16 i
    const float* sb = reinterpret_cast<const float*>(__cvta_shared_to_generic(ss_buf));
    float t = 0.f;
#pragma unroll 1
    for (int c = (lane >> 3) + 4 * warp; c < (int)gridDim.x; c += 16) t += sb[c * kTok + (lane & 7)];
    t += __shfl_xor_sync(0xffffffffu, t, 8);
    t += __shfl_xor_sync(0xffffffffu, t, 16);
    if (lane < kTok) nscr[warp * kTok + lane] = t;
  } else {
#pragma unroll 1
    for (int k8 = tid; k8 < cpr; k8 += kT) {
      uint4 u[kTok];
#pragma unroll
      for (int r = 0; r < kTok; ++r) u[r] = lds128(xs + r * xst + k8 * 16);
#pragma unroll
      for (int r = 0; r < kTok; ++r) {
        const uint32_t ua[4] = {u[r].x, u[r].y, u[r].z, u[r].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(ua[e]);
          ss[r] = fmaf(f.x, f.x, ss[r]);
          ss[r] = fmaf(f.y, f.y, ss[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kTok; ++r) ss[r] = warp_sum(ss[r]);
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < kTok; ++r) nscr[warp * kTok + r] = ss[r];
    }
  }
  cons_bar();
  if (tid < kTok) {  // one thread per row
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < kCons; ++q) t += nscr[q * kTok + tid];
    nscr[kCons * kTok + tid] = 1.0f / sqrtf(t / (float)K + p.eps);
  }
  cons_bar();
  float rinv[kTok];
#pragma unroll
  for (int r = 0; r < kTok; ++r) rinv[r] = nscr[kCons * kTok + r];
  // bf16(bf16(x * rinv) * w): the bf16 product of two bf16 values is the
  // rounded exact product, the same as rounding an fp32 product
#pragma unroll 1
  for (int k8 = tid; k8 < cpr; k8 += kT) {
    const uint4 wv = lds128(xs + kTok * xst + k8 * 16);
    const uint32_t wa[4] = {wv.x, wv.y, wv.z, wv.w};
    uint4 u[kTok];
#pragma unroll
    for (int r = 0; r < kTok; ++r) u[r] = lds128(xs + r * xst + k8 * 16);
#pragma unroll
    for (int r = 0; r < kTok; ++r) {
      uint32_t xa[4] = {u[r].x, u[r].y, u[r].z, u[r].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(xa[e]);
        xa[e] = mul_bf16x2(pack_bf16x2(f.x * rinv[r], f.y * rinv[r]), wa[e]);
      }
      sts128(xs + r * xst + k8 * 16, make_uint4(xa[0], xa[1], xa[2], xa[3]));
    }
  }
  cons_bar();
}

// ---------------------------------------------------- projection phase
// One mma.sync m16n8k16 multiplies a granule pair (16 weight rows, A) by the
// staged tokens (8 columns, B) over 16 K: warp w takes the k16 step w of
// every 64-wide K block, so the four warps' partial sums are added at the end.
// A comes from the ring by ldmatrix.x4 (a stage holds [K block][row][64]:
// granule gi of K block j at (j g + gi) KB, and the TMA's 128-byte swizzle
// puts chunk c of row r at chunk c ^ r), B from the staging buffer by
// ldmatrix.x2.  An
// odd last granule is paired with itself (its second half is discarded).
// A stage's (K block j, pair gp) items are taken eight at a time, item
// i = j * P + gp with P the pair count rounded up to a power of two, into
// accumulator i % 8: every group issues its loads first and then up to eight
// independent MMAs, however few pairs the CTA has; accumulator v holds pair
// v % P, and the P-way split is folded at the end.
// acc[gp] ends as: [0], [1] = (row g8 of granule 2 gp, tokens 2 t4, 2 t4 + 1);
// [2], [3] = (row g8 of granule 2 gp + 1, the same tokens).
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
__device__ bool project(const Params& p, int ph, uint32_t ring_u, uint32_t xs, uint64_t* full,
                        uint64_t* empty, uint32_t& it, int g, float (&acc)[kMaxPairs][4]) {
  const int tid = tid_pinned();
  pin(xs, ring_u);
  const int warp = tid >> 5, lane = tid & 31;
  const int ns = p.nslots;
  const int nkb = proj_k(p, ph) / 64;
  const int kbs = kb_per_stage(g, nkb);
  const int np = (g + 1) >> 1;
  const int lg = np <= 1 ? 0 : np <= 2 ? 1 : np <= 4 ? 2 : 3;  // P = 1 << lg
  const int msk = (1 << lg) - 1;
  // ldmatrix.x4 of A: lanes 8 m .. 8 m + 7 address matrix m = (granule 2 gp +
  // (m & 1), chunk 2 warp + (m >> 1)), row lane & 7
  const int rr = lane & 7, gsel = (lane >> 3) & 1;
  const uint32_t a_off = rr * 128 + ((((2 * warp) + (lane >> 4)) ^ rr) << 4);
  // ldmatrix.x2 of B: lanes 0-7 address token rows at K 16 warp, lanes 8-15 at + 8
  const uint32_t b_base = xs + rr * p.x_stride + (warp * 16 + ((lane >> 3) & 1) * 8) * 2;
#pragma unroll
  for (int i = 0; i < kMaxPairs; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  bool ok = true;
  for (int kb0 = 0; kb0 < nkb; kb0 += kbs) {
    const int n = min(kbs, nkb - kb0);
    const int s = (int)(it % ns);
    if (ok && !ring_wait_warp(p, &full[s], (it / ns) & 1, 0x804)) ok = false;
    if (ok) {
      const uint32_t slot = ring_u + s * kSlot;
      const int items = n << lg;
#pragma unroll 1
      for (int i0 = 0; i0 < items; i0 += kMaxPairs) {
        uint32_t a[kMaxPairs][4], b[kMaxPairs][2];
#pragma unroll
        for (int v = 0; v < kMaxPairs; ++v) {
          const int gp = v & msk, j = (i0 + v) >> lg;
          if (gp < np && j < n) {
            const int gi = min(2 * gp + gsel, g - 1);
            ldsm_x2(b[v], b_base + (kb0 + j) * 128);
            ldsm_x4(a[v], slot + (j * g + gi) * 1024 + a_off);
          }
        }
#pragma unroll
        for (int v = 0; v < kMaxPairs; ++v) {
          const int gp = v & msk, j = (i0 + v) >> lg;
          if (gp < np && j < n)
            mma_bf16_16816(acc[v], a[v][0], a[v][1], a[v][2], a[v][3], b[v][0], b[v][1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // released even after an abort
    ++it;
  }
  // fold accumulator v into v % P
#pragma unroll
  for (int h = kMaxPairs / 2; h >= 1; h >>= 1) {
    if ((1 << lg) <= h) {
#pragma unroll
      for (int v = 0; v < h; ++v)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[v][e] += acc[v + h][e];
    }
  }
  return ok;
}

// The four warps' partial sums into the reduction scratch at the start of the
// staging buffer, red[warp][granule][row][token] (fp32); the caller then adds
// the warps with red_sum.
__device__ __forceinline__ float* red_scratch(uint32_t xs) {
  return reinterpret_cast<float*>(__cvta_shared_to_generic(xs));
}
__device__ void spill_partials(uint32_t xs, int g, const float (&acc)[kMaxPairs][4]) {
  const int tid = tid_pinned();
  const int warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  float* red = red_scratch(xs);
  cons_bar();  // every warp is done with the staged activations
#pragma unroll
  for (int gp = 0; gp < kMaxPairs; ++gp) {
    if (2 * gp < g)
      *reinterpret_cast<float2*>(red + ((warp * kMaxGran + 2 * gp) * kGran + g8) * kTok + 2 * t4) =
          make_float2(acc[gp][0], acc[gp][1]);
    if (2 * gp + 1 < g)
      *reinterpret_cast<float2*>(red + ((warp * kMaxGran + 2 * gp + 1) * kGran + g8) * kTok +
                                 2 * t4) = make_float2(acc[gp][2], acc[gp][3]);
  }
  cons_bar();
}
__device__ __forceinline__ float red_sum(const float* red, int gi, int r, int t) {
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kCons; ++w) s += red[((w * kMaxGran + gi) * kGran + r) * kTok + t];
  return s;
}

// Sum the four warps' partials; thread (warp w, lane) then holds, for
// granules gi = w, w + 4, ..., the values of token g8 and rows 2 t4, 2 t4 + 1
// of the granule in v[gi / 4][0..1].
__device__ void reduce_warps(uint32_t xs, int g, const float (&acc)[kMaxPairs][4],
                             float (&v)[kMaxGran / kCons][2]) {
  const int tid = tid_pinned();
  const int warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  spill_partials(xs, g, acc);
  const float* red = red_scratch(xs);
#pragma unroll
  for (int q = 0; q < kMaxGran / kCons; ++q) {
    const int gi = q * kCons + warp;
    v[q][0] = v[q][1] = 0.f;
    if (gi < g) {
      v[q][0] = red_sum(red, gi, 2 * t4, g8);
      v[q][1] = red_sum(red, gi, 2 * t4 + 1, g8);
    }
  }
}

// Gate/up epilogue: gate and up are rounded to bf16 (the matmul's output),
// then h = silu(gate) * up with the reference's rounding after each op
// (model_fused.py:169), written to h [M, I] for the 4 features of each of this
// CTA's granules [lo, lo + g) (rows 0-3 gate, rows 4-7 up).
__device__ void store_swiglu(const Params& p, uint32_t xs, int lo, int g,
                             const float (&acc)[kMaxPairs][4]) {
  constexpr int kF = kGran / 2;  // features per granule
  spill_partials(xs, g, acc);
  const float* red = red_scratch(xs);
  const int tid = tid_pinned();
  const int nout = g * kF * kTok;
  for (int idx = tid; idx < nout; idx += kCons * 32) {
    const int gi = idx / (kF * kTok), t = (idx / kF) % kTok, r = idx % kF;
    if (t < p.M) {
      const float gate = rbf(red_sum(red, gi, r, t));
      const float up = rbf(red_sum(red, gi, r + kF, t));
      p.gu[(int64_t)t * p.I + (lo + gi) * kF + r] = f2bf(silu_ref(gate) * up);
    }
  }
}

// Plain epilogue (QKV, gate/up): bf16 outputs [M, N] (the matmul's rounding).
__device__ void store_rows(const Params& p, __nv_bfloat16* out, int N, int lo, int g,
                           const float (&v)[kMaxGran / kCons][2]) {
  const int tid = tid_pinned();
  const int warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  if (g8 >= p.M) return;
#pragma unroll
  for (int q = 0; q < kMaxGran / kCons; ++q) {
    const int gi = q * kCons + warp;
    if (gi < g) {
      const int row = (lo + gi) * kGran + 2 * t4;
      *reinterpret_cast<uint32_t*>(out + (int64_t)g8 * N + row) = pack_bf16x2(v[q][0], v[q][1]);
    }
  }
}

// All-reduce epilogue (o_proj, down): out = bf16(res + bf16(sum over ranks of
// the bf16 partials)), for this CTA's rows; the rows are the same on every
// rank, so the exchange is between the CTAs of one index on every GPU.  Each
// thread loads its residuals and all the peers' words of a row at once (one
// round trip, then polls only what had not arrived), and the CTA leaves the
// per-token sums of squares of its outputs in ssp_out[CTA][8] for the next
// RMSNorm.
__device__ void allreduce_rows(const Params& p, uint32_t xs, int lo, int g,
                               const float (&v)[kMaxGran / kCons][2], uint32_t call,
                               const __nv_bfloat16* res, __nv_bfloat16* out, float* ssp_out) {
  const int tid = tid_pinned();
  const int warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  // this rank's partials as bf16 [row][token] after the reduction scratch,
  // then the outputs' squares [row][token]
  __nv_bfloat16* part = reinterpret_cast<__nv_bfloat16*>(red_scratch(xs) +
                                                       kCons * kMaxGran * kGran * kTok);
  float* sq = red_scratch(xs) + kCons * kMaxGran * kGran * kTok + kMaxGran * kGran * kTok / 2;
#pragma unroll
  for (int q = 0; q < kMaxGran / kCons; ++q) {
    const int gi = q * kCons + warp;
    if (gi < g) {
      part[(gi * kGran + 2 * t4) * kTok + g8] = f2bf(v[q][0]);
      part[(gi * kGran + 2 * t4 + 1) * kTok + g8] = f2bf(v[q][1]);
    }
  }
  for (int i = tid; i < g * kGran * kTok; i += kCons * 32) sq[i] = 0.f;
  cons_bar();
  const int par = (int)(call & 1u);
  const int tps = (p.M + 1) / 2;
  const int nwords = g * kGran * tps;
  for (int w = tid; w < nwords; w += kCons * 32) {
    const int rl = w / tps, tp = w % tps;
    const int row = lo * kGran + rl;
    const __nv_bfloat16 lo_v = part[rl * kTok + 2 * tp];
    const __nv_bfloat16 hi_v = (2 * tp + 1 < p.M) ? part[rl * kTok + 2 * tp + 1] : f2bf(0.f);
    const uint32_t mine =
        (uint32_t)__bfloat16_as_ushort(lo_v) | ((uint32_t)__bfloat16_as_ushort(hi_v) << 16);
    for (int r = 0; r < p.world; ++r)
      if (r != p.rank) st_word(p.inbox[r] + word_at(p, par, p.rank, row, tp), mine, call);
  }
#pragma unroll 1
  for (int w = tid; w < nwords; w += kCons * 32) {
    const int rl = w / tps, tp = w % tps;
    const int row = lo * kGran + rl;
    const bool two = 2 * tp + 1 < p.M;
    const float r0 = bf2f(__ldcg(res + (int64_t)(2 * tp) * p.H + row));
    const float r1 = two ? bf2f(__ldcg(res + (int64_t)(2 * tp + 1) * p.H + row)) : 0.f;
    uint2 x[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < p.world && r != p.rank) x[r] = ld_word(p.inbox[p.rank] + word_at(p, par, r, row, tp));
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 1
    for (int r = 0; r < p.world; ++r) {
      uint32_t d;
      if (r == p.rank) {
        d = (uint32_t)__bfloat16_as_ushort(part[rl * kTok + 2 * tp]) |
            (two ? (uint32_t)__bfloat16_as_ushort(part[rl * kTok + 2 * tp + 1]) << 16 : 0u);
      } else {
        if (x[r].y != call && !aborted(p)) {
          const uint2* src = p.inbox[p.rank] + word_at(p, par, r, row, tp);
          const uint64_t t0 = globaltimer_ns();
          uint32_t spins = 0;
          while ((x[r] = ld_word(src)).y != call) {
            if ((++spins & 255u) == 0) {
              if (aborted(p)) break;
              if (globaltimer_ns() - t0 > p.wait_ns) {
                raise_abort(p, 0x501);
                break;
              }
            }
          }
        }
        d = x[r].x;
      }
      const float2 f = unpack_bf16x2(d);
      s0 += f.x;
      s1 += f.y;
    }
    const __nv_bfloat16 o0 = f2bf(r0 + rbf(s0));
    out[(int64_t)(2 * tp) * p.H + row] = o0;
    sq[rl * kTok + 2 * tp] = bf2f(o0) * bf2f(o0);
    if (two) {
      const __nv_bfloat16 o1 = f2bf(r1 + rbf(s1));
      out[(int64_t)(2 * tp + 1) * p.H + row] = o1;
      sq[rl * kTok + 2 * tp + 1] = bf2f(o1) * bf2f(o1);
    }
  }
  cons_bar();
  // per-token sums over this CTA's rows, in row order: warp w sums tokens w, w + 4
#pragma unroll 1
  for (int t = warp; t < kTok; t += kCons) {
    float a = 0.f;
    for (int rl = lane; rl < g * kGran; rl += 32) a += sq[rl * kTok + t];
    a = warp_sum(a);
    if (lane == 0) ssp_out[blockIdx.x * kTok + t] = a;
  }
}

// ------------------------------------------------------ attention phase
// One head row of q or k (128 dims; lane owns dims 4 lane .. 4 lane + 3):
// RMSNorm over the head (model_fused.py:113-119) then rotate-half RoPE
// (:122-129), with the reference's bf16 rounding points.
__device__ __noinline__ void norm_rope_head(const __nv_bfloat16* x, const __nv_bfloat16* w,
                                            const __nv_bfloat16* cs_cos,
                                               const __nv_bfloat16* cs_sin, int64_t crow,
                                               float eps, int lane, float (&o)[4]) {
  const int d0 = lane * 4, j0 = d0 & 63;
  const uint2 u = __ldcg(reinterpret_cast<const uint2*>(x + d0));
  const float2 a = unpack_bf16x2(u.x), bb = unpack_bf16x2(u.y);
  const float vx[4] = {a.x, a.y, bb.x, bb.y};
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(vx[i], vx[i], ss);
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss * (1.0f / kHD) + eps);
  const uint2 wu = *reinterpret_cast<const uint2*>(w + d0);
  const uint2 cu = *reinterpret_cast<const uint2*>(cs_cos + crow * 64 + j0);
  const uint2 su = *reinterpret_cast<const uint2*>(cs_sin + crow * 64 + j0);
  const float2 w0 = unpack_bf16x2(wu.x), w1 = unpack_bf16x2(wu.y);
  const float2 c0 = unpack_bf16x2(cu.x), c1 = unpack_bf16x2(cu.y);
  const float2 s0 = unpack_bf16x2(su.x), s1 = unpack_bf16x2(su.y);
  const float wv[4] = {w0.x, w0.y, w1.x, w1.y};
  const float cv[4] = {c0.x, c0.y, c1.x, c1.y}, sv[4] = {s0.x, s0.y, s1.x, s1.y};
  float n[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = rbf(rbf(vx[i] * r) * wv[i]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float pp = __shfl_xor_sync(0xffffffffu, n[i], 16);
    const float rot = (lane < 16) ? -pp : pp;
    o[i] = rbf(rbf(n[i] * cv[i]) + rbf(rot * sv[i]));
  }
}

// Attention of this CTA's (sequence, KV head, split) unit, if it has one.
// Scratch in the staging buffer: q_s [G][128] bf16 | sm_o [4][G][128] f32 |
// sm_ml [4][G][2] f32 | new_s [2][128] f32 | snew [G] f32; the pair merge then
// reuses sm_o as [splits][G][2] weights | [G] 1 / sum | [splits][slice] products.
template <int G>
__device__ bool attention(const Params& p, int l, uint32_t ring_u, uint32_t xs, uint64_t* full,
                          uint64_t* empty, uint32_t& it, int L, AttPlan ap) {
  const int tid = tid_pinned();
  const int warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int c = blockIdx.x, ns = p.nslots;
  const int pairs = p.M * p.Hkv;
  if (c >= pairs * ap.splits) return true;
  const LayerPtrs lp = p.lp[l];
  const int pair = c / ap.splits, split = c % ap.splits;
  const int b = pair / p.Hkv, kvh = pair % p.Hkv;
  const int start = split * ap.chunk;
  const int end = min(start + ap.chunk, L - 1);  // old rows; row L - 1 is the new token
  const bool with_new = start <= L - 1 && L - 1 < start + ap.chunk;
  const int64_t crow = (int64_t)(L - 1) + p.rope_delta;
  uint8_t* sbase = reinterpret_cast<uint8_t*>(__cvta_shared_to_generic(xs));
  __nv_bfloat16* q_s = reinterpret_cast<__nv_bfloat16*>(sbase);
  float* sm_o = reinterpret_cast<float*>(sbase + kMaxG * kHD * 2);
  float* sm_ml = sm_o + kCons * kMaxG * kHD;
  float* new_s = sm_ml + kCons * kMaxG * 2;
  float* snew = new_s + 2 * kHD;
  const int ld = (p.Hq + 2 * p.Hkv) * kHD;
  const __nv_bfloat16* qrow = p.qkv + (int64_t)b * ld;

#pragma unroll 1
  for (int gg = warp; gg < G; gg += kCons) {
    float o4[4];
    norm_rope_head(qrow + (kvh * G + gg) * kHD, lp.q_norm, p.cos, p.sin, crow, p.eps, lane, o4);
    *reinterpret_cast<uint2*>(&q_s[gg * kHD + lane * 4]) =
        make_uint2(pack_bf16x2(o4[0], o4[1]), pack_bf16x2(o4[2], o4[3]));
  }
  cons_bar();
  uint32_t qf[8][2];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    if (g8 < G) {
      qf[ks][0] = *reinterpret_cast<const uint32_t*>(&q_s[g8 * kHD + ks * 16 + 2 * t4]);
      qf[ks][1] = *reinterpret_cast<const uint32_t*>(&q_s[g8 * kHD + ks * 16 + 8 + 2 * t4]);
    } else {
      qf[ks][0] = qf[ks][1] = 0u;
    }
  }
  float o[16][2];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = 0.f;
  float m_r = -INFINITY, l_r = 0.f;
  bool ok = true;
  for (int t0 = start; t0 < end; t0 += kPos) {
    const int sk = (int)(it % ns), sv = (int)((it + 1) % ns);
    if (ok && (!ring_wait_warp(p, &full[sk], (it / ns) & 1, 0x805) ||
               !ring_wait_warp(p, &full[sv], ((it + 1) / ns) & 1, 0x805)))
      ok = false;
    if (ok) {
      const uint32_t sK = ring_u + sk * kSlot, sV = ring_u + sv * kSlot;
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
      const int pos0 = t0 + warp * 16;
      float x[4];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int pos = pos0 + j * 8 + 2 * t4 + e;
          x[j * 2 + e] = (pos < end) ? sc[j][e] * p.scale_log2 : -INFINITY;
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
      const uint32_t pa0 = pack_bf16x2(pr[0], pr[1]);
      const uint32_t pa2 = pack_bf16x2(pr[2], pr[3]);
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
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&empty[sk]);
      mbar_arrive(&empty[sv]);
    }
    it += 2;
  }
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);
  if (g8 < G) {
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      sm_o[(warp * kMaxG + g8) * kHD + d * 8 + 2 * t4] = o[d][0];
      sm_o[(warp * kMaxG + g8) * kHD + d * 8 + 2 * t4 + 1] = o[d][1];
    }
    if (t4 == 0) {
      sm_ml[(warp * kMaxG + g8) * 2 + 0] = m_r;
      sm_ml[(warp * kMaxG + g8) * 2 + 1] = l_r;
    }
  }
  if (with_new) {
    // the new token's k (normed, rotated) and v rows: into the caches and into
    // this split's merge
    const int64_t row = kv_row(p, b, kvh, L - 1);
    const int64_t off = (row < 0 ? 0 : row) * kHD;
    if (row < 0 && tid == 0) raise_abort(p, 0x809);
    if (row < 0) {
      // no cache row to write: the step is abandoned (the abort stops every CTA)
    } else if (warp == 0) {
      float o4[4];
      norm_rope_head(qrow + (p.Hq + kvh) * kHD, lp.k_norm, p.cos, p.sin, crow, p.eps, lane, o4);
      const uint2 pk = make_uint2(pack_bf16x2(o4[0], o4[1]), pack_bf16x2(o4[2], o4[3]));
      *reinterpret_cast<uint2*>(lp.k_cache + off + lane * 4) = pk;
      const float2 a0 = unpack_bf16x2(pk.x), a1 = unpack_bf16x2(pk.y);
      new_s[lane * 4 + 0] = a0.x; new_s[lane * 4 + 1] = a0.y;
      new_s[lane * 4 + 2] = a1.x; new_s[lane * 4 + 3] = a1.y;
    } else if (warp == 1) {
      const uint2 pv =
          __ldcg(reinterpret_cast<const uint2*>(qrow + (p.Hq + p.Hkv + kvh) * kHD + lane * 4));
      *reinterpret_cast<uint2*>(lp.v_cache + off + lane * 4) = pv;
      const float2 a0 = unpack_bf16x2(pv.x), a1 = unpack_bf16x2(pv.y);
      new_s[kHD + lane * 4 + 0] = a0.x; new_s[kHD + lane * 4 + 1] = a0.y;
      new_s[kHD + lane * 4 + 2] = a1.x; new_s[kHD + lane * 4 + 3] = a1.y;
    }
    cons_bar();
    for (int gg = warp; gg < G; gg += kCons) {
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        acc = fmaf(bf2f(q_s[gg * kHD + lane * 4 + i]), new_s[lane * 4 + i], acc);
      acc = warp_sum(acc);
      if (lane == 0) snew[gg] = acc * p.scale_log2;
    }
  }
  cons_bar();
  // merge the warps (and the new row): one split's partial, or the output
  float* apart = p.apart + (size_t)c * kMaxG * (kHD + 2);
#pragma unroll 1
  for (int idx = tid; idx < G * kHD; idx += kCons * 32) {
    const int gg = idx / kHD, d = idx % kHD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCons; ++w) M = fmaxf(M, sm_ml[(w * kMaxG + gg) * 2]);
    if (with_new) M = fmaxf(M, snew[gg]);
    float a = 0.f, lsum = 0.f;
#pragma unroll
    for (int w = 0; w < kCons; ++w) {
      const float mw = sm_ml[(w * kMaxG + gg) * 2];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      a = fmaf(f, sm_o[(w * kMaxG + gg) * kHD + d], a);
      lsum = fmaf(f, sm_ml[(w * kMaxG + gg) * 2 + 1], lsum);
    }
    if (with_new) {
      const float f = exp2f(snew[gg] - M);
      a = fmaf(f, new_s[kHD + d], a);
      lsum += f;
    }
    if (ap.splits == 1) {
      p.attn[(int64_t)b * p.Hq * kHD + (kvh * G + gg) * kHD + d] = f2bf(lsum > 0.f ? a / lsum : 0.f);
    } else {
      apart[gg * (kHD + 2) + d] = a;
      if (d == 0) {
        apart[gg * (kHD + 2) + kHD] = M;
        apart[gg * (kHD + 2) + kHD + 1] = lsum;
      }
    }
  }
  if (ap.splits == 1) return ok;
  // Every split of the pair merges a slice of the pair's G x 128 outputs once
  // all the pair's splits have published their partials: the arrivals count
  // up by one per split and layer (the counter is zeroed before each launch).
  cons_bar();
  if (tid == 0) {
    __threadfence();
    atomicAdd(&p.pair_cnt[pair], 1);
    const int target = ap.splits * (l + 1);
    if (ld_acquire_gpu_u32(reinterpret_cast<const unsigned*>(&p.pair_cnt[pair])) < (unsigned)target &&
        !aborted(p)) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_gpu_u32(reinterpret_cast<const unsigned*>(&p.pair_cnt[pair])) <
             (unsigned)target) {
        __nanosleep(20);
        if ((++spins & 63u) == 0) {
          if (aborted(p)) break;
          if (globaltimer_ns() - t0 > p.wait_ns) {
            raise_abort(p, 0x807);
            break;
          }
        }
      }
    }
  }
  cons_bar();
  const float* pp = p.apart + (size_t)pair * ap.splits * kMaxG * (kHD + 2);
  // per split and head: (max, sum) -> (weight, sum); scratch after q_s
  float* ml = sm_o;                                  // [splits][G][2]
  float* inv = sm_o + 2 * kMaxSplitsMerge * kMaxG;  // [G]
  float* prod = inv + kMaxG;                        // [splits][per]
#pragma unroll 1
  for (int i = tid; i < ap.splits * G; i += kCons * 32) {
    const int sp = i / G, gg = i % G;
    const float* q = pp + ((size_t)sp * kMaxG + gg) * (kHD + 2);
    ml[i * 2] = __ldcg(q + kHD);
    ml[i * 2 + 1] = __ldcg(q + kHD + 1);
  }
  cons_bar();
#pragma unroll 1
  for (int gg = warp; gg < G; gg += kCons) {  // one warp per head, lanes over splits
    float M = -INFINITY;
    for (int sp = lane; sp < ap.splits; sp += 32) M = fmaxf(M, ml[(sp * G + gg) * 2]);
    M = warp_max(M);
    float lsum = 0.f;
    for (int sp = lane; sp < ap.splits; sp += 32) {
      const float ms = ml[(sp * G + gg) * 2];
      const float f = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
      ml[(sp * G + gg) * 2] = f;  // now the split's weight
      lsum = fmaf(f, ml[(sp * G + gg) * 2 + 1], lsum);
    }
    lsum = warp_sum(lsum);
    if (lane == 0) inv[gg] = lsum > 0.f ? 1.f / lsum : 0.f;
  }
  cons_bar();
  // this split's slice of outputs: every (split, output) product loaded at once
  const int per = (G * kHD + ap.splits - 1) / ap.splits;
  const int o0 = split * per, n_out = max(0, min(per, G * kHD - o0));
#pragma unroll 4
  for (int i = tid; i < ap.splits * n_out; i += kCons * 32) {
    const int sp = i / n_out, k = i % n_out;
    const int gg = (o0 + k) / kHD, d = (o0 + k) % kHD;
    prod[i] = ml[(sp * G + gg) * 2] * __ldcg(pp + ((size_t)sp * kMaxG + gg) * (kHD + 2) + d);
  }
  cons_bar();
  for (int k = tid; k < n_out; k += kCons * 32) {
    const int gg = (o0 + k) / kHD, d = (o0 + k) % kHD;
    float a = 0.f;
    for (int sp = 0; sp < ap.splits; ++sp) a += prod[sp * n_out + k];
    p.attn[(int64_t)b * p.Hq * kHD + (kvh * G + gg) * kHD + d] = f2bf(a * inv[gg]);
  }
  return ok;
}

// ---------------------------------------------------------------- kernel
template <int G>
__global__ void __launch_bounds__(kThreads, 1) decode_tp_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = base;
  const uint32_t ring_u = smem_u32(ring);
  const uint32_t xs = ring_u + p.nslots * kSlot;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + p.nslots * kSlot + p.x_bytes);
  uint64_t* empty = full + kMaxSlots;
  float* nscr = reinterpret_cast<float*>(empty + kMaxSlots);  // RMSNorm: [4][8] sums, [8] 1/rms
  uint64_t* sbar = reinterpret_cast<uint64_t*>(nscr + (kCons + 1) * kTok);  // staging copies
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.nslots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCons);
    }
    mbar_init(sbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int L = *p.kv_len_dev;
  {  // the new position must have a cache row: otherwise no CTA runs the step
    const int64_t cap = p.table ? (int64_t)p.table_stride * p.page_tokens : p.max_seq;
    if (L < 1 || L > cap) {
      if (blockIdx.x == 0 && threadIdx.x == 0) raise_abort(p, 0x80a);
      return;
    }
  }
  const AttPlan ap = att_plan(p.M * p.Hkv, L, gridDim.x);

  if (warp == kCons) {
    if (lane == 0) producer(p, ring, full, empty, L, ap);
    return;
  }
  // ------------------------------------------------------------ consumers
  const uint32_t call0 = *reinterpret_cast<const volatile unsigned*>(p.step_no) * 2u *
                         (uint32_t)p.n_layers;
  const int C = gridDim.x, c = blockIdx.x;
  uint32_t it = 0;
  unsigned target = 0;
  uint32_t sphase = 0;
  float acc[kMaxPairs][4];
  float v[kMaxGran / kCons][2];
  // The layer's five phases run through one copy of the code: the step kernel
  // executes its whole text once per layer, and a text larger than the SM's
  // instruction cache is refetched from the (busy) L2 every layer.
  for (int l = 0; l < p.n_layers; ++l) {
#pragma unroll 1
    for (int ph0 = 0; ph0 < kPhases; ++ph0) {
      int ph = ph0;
      pin(ph);
      if (ph == kATT) {
        attention<G>(p, l, ring_u, xs, full, empty, it, L, ap);  // -> attn
      } else {
        int lo, hi;
        phase_range(p, ph, c, C, lo, hi);
        if (hi > lo) {
          // QKV: rmsnorm(x) @ Wqkv -> qkv; O: attn @ Wo + all-reduce + x -> x2;
          // GU: rmsnorm(x2) @ Wgate_up, silu(gate) * up -> h;
          // DN: h @ Wdown + all-reduce + x2 -> x
          const __nv_bfloat16* src = ph == kQKV ? p.X : ph == kO ? p.attn : ph == kGU ? p.X2 : p.gu;
          const __nv_bfloat16* nw = ph == kQKV ? p.lp[l].in_norm
                                   : ph == kGU ? p.lp[l].post_norm
                                               : nullptr;
          const float* ssp = ph == kGU ? p.ssx2 : (ph == kQKV && l > 0) ? p.ssx : nullptr;
          stage(p, xs, src, proj_k(p, ph), nw, ssp, nscr, sbar, sphase);
          project(p, ph, ring_u, xs, full, empty, it, hi - lo, acc);
          if (ph == kGU) {
            store_swiglu(p, xs, lo, hi - lo, acc);
          } else {
            reduce_warps(xs, hi - lo, acc, v);
            if (ph == kQKV)
              store_rows(p, p.qkv, proj_n(p, kQKV), lo, hi - lo, v);
            else
              allreduce_rows(p, xs, lo, hi - lo, v, call0 + 2u * l + (ph == kO ? 1u : 2u),
                             ph == kO ? p.X : p.X2, ph == kO ? p.X2 : p.X,
                             ph == kO ? p.ssx2 : p.ssx);
          }
        } else if ((ph == kO || ph == kDN) && threadIdx.x < kTok) {
          (ph == kO ? p.ssx2 : p.ssx)[c * kTok + threadIdx.x] = 0.f;  // no rows here
        }
      }
      grid_sync(p, target);
    }
  }
  // every CTA has read step_no (at its start) and finished: advance it
  if (c == 0 && threadIdx.x == 0) *p.step_no += 1u;
}

// ------------------------------------------------------------------ host
struct Plan {
  Params p{};
  int device = 0;
  int G = 0;
  size_t smem = 0;
  int grid = 0;
  void* dmem = nullptr;  // one allocation: maps, pointers, buffers, counters
};

}  // namespace tp
}  // namespace q3

namespace {
int decode_tp_create_impl(const q3_step_layer* layers, int n_layers, int batch, int hidden,
                          int q_heads, int kv_heads, int inter, int64_t max_seq, float eps,
                          const void* rope_cos, const void* rope_sin, int64_t rope_rows,
                          void* comm, const int32_t* table, int table_stride, int page_tokens,
                          int64_t num_pages, void** plan_out) {
  using namespace q3;
  using namespace q3::tp;
  Q3_REQUIRE(layers && rope_cos && rope_sin && comm && plan_out, "q3_decode_tp_create: null pointer");
  if (table) {
    Q3_REQUIRE(page_tokens > 0 && page_tokens % kPos == 0 && table_stride > 0 && num_pages > 0 &&
                   num_pages * kv_heads * page_tokens < (1ll << 31) &&
                   (int64_t)table_stride * page_tokens >= max_seq,
               "q3_decode_tp_create_paged: pages of %d tokens (a multiple of %d), %d table "
               "columns covering max_seq %lld, %lld pages",
               page_tokens, kPos, table_stride, (long long)max_seq, (long long)num_pages);
  }
  Q3_REQUIRE(n_layers > 0 && batch >= 1 && batch <= kTok,
             "q3_decode_tp_create: %d layers, batch %d (1..%d)", n_layers, batch, kTok);
  Q3_REQUIRE(q_heads > 0 && kv_heads > 0 && q_heads % kv_heads == 0,
             "q3_decode_tp_create: bad heads %d / %d", q_heads, kv_heads);
  const int G = q_heads / kv_heads;
  Q3_REQUIRE(G == 1 || G == 2 || G == 4 || G == 8,
             "q3_decode_tp_create: %d query heads per KV head not in {1, 2, 4, 8}", G);
  Q3_REQUIRE(hidden > 0 && hidden % 64 == 0 && inter > 0 && inter % 64 == 0 &&
                 (q_heads * 128) % 64 == 0,
             "q3_decode_tp_create: hidden %d and inter %d must be multiples of 64", hidden, inter);
  Q3_REQUIRE(max_seq > 0 && (table || batch * kv_heads * max_seq < (1ll << 31)) && rope_rows > 0,
             "q3_decode_tp_create: bad max_seq / rope_rows");
  Comm* cm = static_cast<Comm*>(comm);
  Q3_REQUIRE(cm->open || cm->world == 1, "q3_decode_tp_create: communicator peers not opened");
  const size_t inbox_bytes = (size_t)2 * kMaxRanks * hidden * kPairs * sizeof(uint2);
  Q3_REQUIRE(comm_data_bytes(cm->max_tiles) >= inbox_bytes,
             "q3_decode_tp_create: the communicator holds %zu bytes, the exchange needs %zu "
             "(create it with max_cols >= %d)",
             comm_data_bytes(cm->max_tiles), inbox_bytes, hidden);
  int dev = 0;
  Q3_CUDA_CHECK(cudaGetDevice(&dev));
  const int C = num_sms();
  // every phase's granules must fit kMaxGran per CTA
  const int nmax = max(max((q_heads + 2 * kv_heads) * 128, hidden), 2 * inter);
  Q3_REQUIRE((nmax / kGran + C - 1) / C <= kMaxGran,
             "q3_decode_tp_create: %d output rows need more than %d granules per SM (a "
             "larger tensor-parallel degree fits)",
             nmax, kMaxGran);
  const int kmax = max(max(hidden, q_heads * 128), inter);
  const int x_stride = kmax * 2 + 16;
  // staged activations, or the reduction scratch, or the attention scratch
  const int red_bytes = kCons * kMaxGran * kGran * kTok * 4 + kMaxGran * kGran * kTok * 2 +
                        kMaxGran * kGran * kTok * 4;
  const int att_bytes = kMaxG * kHD * 2 +
                        max(kCons * kMaxG * kHD + kCons * kMaxG * 2 + 2 * kHD + kMaxG + 1,
                            2 * kMaxSplitsMerge * kMaxG + kMaxG + kMaxG * kHD + kMaxSplitsMerge) *
                            4;
  // eight rows, the norm weight row, the per-CTA sums of squares
  int x_bytes = max(max((kTok + 1) * x_stride + C * kTok * 4, red_bytes), att_bytes);
  x_bytes = (x_bytes + 1023) / 1024 * 1024;
  const int fixed = x_bytes + 1024 /*align*/ + 2 * kMaxSlots * 8 + (kCons + 1) * kTok * 4 + 8;
  const int nslots = min(kMaxSlots, (kSmemLimit - fixed) / kSlot);
  Q3_REQUIRE(nslots >= 3,
             "q3_decode_tp_create: reduction length %d leaves no room for the weight ring", kmax);
  const size_t smem = (size_t)nslots * kSlot + fixed;

  tp::Plan* pl = new tp::Plan();
  pl->device = dev;
  pl->G = G;
  pl->smem = smem;
  pl->grid = C;
  Params& p = pl->p;
  p.n_layers = n_layers; p.M = batch; p.H = hidden; p.Hq = q_heads; p.Hkv = kv_heads;
  p.I = inter; p.max_seq = max_seq; p.eps = eps;
  p.scale_log2 = (1.0f / sqrtf(128.0f)) * 1.4426950408889634f;
  p.cos = (const __nv_bfloat16*)rope_cos; p.sin = (const __nv_bfloat16*)rope_sin;
  p.rope_rows = rope_rows;
  p.table = table;
  p.table_stride = table_stride;
  p.page_tokens = page_tokens;
  p.num_pages = num_pages;
  p.rank = cm->rank; p.world = cm->world;
  p.wait_ns = cm->wait_ns;
  for (int r = 0; r < kMaxRanks; ++r)
    p.inbox[r] = (r == cm->rank) ? static_cast<uint2*>(cm->local)
                                 : static_cast<uint2*>(cm->peers[r]);
  p.x_stride = x_stride;
  p.x_bytes = x_bytes;
  p.nslots = nslots;
  p.inflight = nslots;
  if (const char* e = getenv("Q3VL_TP_INFLIGHT")) p.inflight = max(1, min(nslots, atoi(e)));
  p.prod_sleep = 0;
  p.cons_sleep = 0;
  if (const char* e = getenv("Q3VL_TP_PSLEEP")) p.prod_sleep = max(0, min(1000, atoi(e)));
  if (const char* e = getenv("Q3VL_TP_CSLEEP")) p.cons_sleep = max(0, min(1000, atoi(e)));
  p.err = device_error_word();

  // device memory: maps | layer pointers | x2 | qkv | attn | gu | apart | pair_cnt | gbar,
  // step_no, abort
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t nqkv = (size_t)(q_heads + 2 * kv_heads) * 128;
  size_t off = 0;
  const size_t o_maps = off; off = al(off + sizeof(LayerMaps) * n_layers);
  const size_t o_lp = off; off = al(off + sizeof(LayerPtrs) * n_layers);
  const size_t o_x2 = off; off = al(off + (size_t)batch * hidden * 2);
  const size_t o_qkv = off; off = al(off + (size_t)batch * nqkv * 2);
  const size_t o_attn = off; off = al(off + (size_t)batch * q_heads * 128 * 2);
  const size_t o_gu = off; off = al(off + (size_t)batch * 2 * inter * 2);
  const size_t o_ap = off; off = al(off + (size_t)C * kMaxG * (kHD + 2) * 4);
  const size_t o_ss = off; off = al(off + (size_t)2 * C * kTok * 4);
  const size_t o_cnt = off; off = al(off + (size_t)batch * kv_heads * 4);
  const size_t o_ctr = off; off = al(off + 3 * 4);
  cudaError_t e = cudaMalloc(&pl->dmem, off);
  if (e != cudaSuccess) {
    delete pl;
    return fail(Q3_ERR_CUDA, "q3_decode_tp_create: cudaMalloc(%zu): %s", off,
                cudaGetErrorString(e));
  }
  char* d = static_cast<char*>(pl->dmem);
  e = cudaMemset(d, 0, off);
  // every CTA owns g = floor or ceil(granules / CTAs) granules of a phase, one
  // weight-map box height each
  int gbox[4][2];
  {
    const int ng[4] = {(int)(nqkv / kGran), hidden / kGran, 2 * inter / kGran, hidden / kGran};
    for (int w = 0; w < 4; ++w) {
      gbox[w][0] = ng[w] / C;
      gbox[w][1] = (ng[w] + C - 1) / C;
      pl->p.gbox[w][0] = gbox[w][0];
      pl->p.gbox[w][1] = gbox[w][1];
    }
  }
  const int64_t kv_rows = table ? num_pages * kv_heads * page_tokens
                                : (int64_t)batch * kv_heads * max_seq;
  std::vector<LayerMaps> maps(n_layers);
  std::vector<LayerPtrs> ptrs(n_layers);
  int rc = Q3_OK;
  for (int i = 0; i < n_layers && rc == Q3_OK && e == cudaSuccess; ++i) {
    const q3_step_layer& L = layers[i];
    if (!(L.w_qkv && L.w_o && L.w_gate_up && L.w_down && L.input_norm && L.post_norm &&
          L.q_norm && L.k_norm && L.k_cache && L.v_cache)) {
      rc = fail(Q3_ERR_INVALID, "q3_decode_tp_create: layer %d has a null pointer", i);
      break;
    }
    const void* wp[4] = {L.w_qkv, L.w_o, L.w_gate_up, L.w_down};
    const int64_t wn[4] = {(int64_t)nqkv, hidden, 2 * (int64_t)inter, hidden};
    const int64_t wk[4] = {hidden, (int64_t)q_heads * 128, hidden, inter};
    for (int w = 0; w < 4 && !rc; ++w)
      for (int gc = 0; gc < 2 && !rc; ++gc)
        for (int d = 0; d < kDepths && !rc && gbox[w][gc] > 0; ++d)
          rc = make_tmap_wblocks(&maps[i].w[w][gc][d], wp[w], wn[w], wk[w], kGran * gbox[w][gc],
                                 1 << d);
    if (!rc)
      rc = make_tmap_2d(&maps[i].k, L.k_cache, kv_rows, kHD, kPos, 64);
    if (!rc)
      rc = make_tmap_2d(&maps[i].v, L.v_cache, kv_rows, kHD, kPos, 64);
    ptrs[i] = LayerPtrs{(const __nv_bfloat16*)L.input_norm, (const __nv_bfloat16*)L.post_norm,
                        (const __nv_bfloat16*)L.q_norm, (const __nv_bfloat16*)L.k_norm,
                        (__nv_bfloat16*)L.k_cache, (__nv_bfloat16*)L.v_cache};
  }
  if (rc == Q3_OK && e == cudaSuccess)
    e = cudaMemcpy(d + o_maps, maps.data(), sizeof(LayerMaps) * n_layers, cudaMemcpyHostToDevice);
  if (rc == Q3_OK && e == cudaSuccess)
    e = cudaMemcpy(d + o_lp, ptrs.data(), sizeof(LayerPtrs) * n_layers, cudaMemcpyHostToDevice);
  if (rc == Q3_OK && e == cudaSuccess)
    e = cudaFuncSetAttribute(G == 1 ? decode_tp_kernel<1> : G == 2 ? decode_tp_kernel<2>
                             : G == 4 ? decode_tp_kernel<4> : decode_tp_kernel<8>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (rc != Q3_OK || e != cudaSuccess) {
    cudaFree(pl->dmem);
    delete pl;
    return rc != Q3_OK ? rc : fail(Q3_ERR_CUDA, "q3_decode_tp_create: %s", cudaGetErrorString(e));
  }
  p.maps = reinterpret_cast<const LayerMaps*>(d + o_maps);
  p.lp = reinterpret_cast<const LayerPtrs*>(d + o_lp);
  p.X2 = reinterpret_cast<__nv_bfloat16*>(d + o_x2);
  p.qkv = reinterpret_cast<__nv_bfloat16*>(d + o_qkv);
  p.attn = reinterpret_cast<__nv_bfloat16*>(d + o_attn);
  p.gu = reinterpret_cast<__nv_bfloat16*>(d + o_gu);
  p.apart = reinterpret_cast<float*>(d + o_ap);
  p.ssx = reinterpret_cast<float*>(d + o_ss);
  p.ssx2 = p.ssx + C * kTok;
  p.pair_cnt = reinterpret_cast<int*>(d + o_cnt);
  p.gbar = reinterpret_cast<unsigned*>(d + o_ctr);
  p.step_no = p.gbar + 1;
  p.abort = reinterpret_cast<int*>(p.gbar + 2);
  *plan_out = pl;
  return Q3_OK;
}
}  // namespace

extern "C" int q3_decode_tp_create(const q3_step_layer* layers, int n_layers, int batch,
                                   int hidden, int q_heads, int kv_heads, int inter,
                                   int64_t max_seq, float eps, const void* rope_cos,
                                   const void* rope_sin, int64_t rope_rows, void* comm,
                                   void** plan_out) {
  return decode_tp_create_impl(layers, n_layers, batch, hidden, q_heads, kv_heads, inter, max_seq,
                               eps, rope_cos, rope_sin, rope_rows, comm, nullptr, 0, 0, 0,
                               plan_out);
}

extern "C" int q3_decode_tp_create_paged(const q3_step_layer* layers, int n_layers, int batch,
                                         int hidden, int q_heads, int kv_heads, int inter,
                                         int64_t max_seq, float eps, const void* rope_cos,
                                         const void* rope_sin, int64_t rope_rows, void* comm,
                                         const int32_t* block_table, int table_stride,
                                         int page_tokens, int64_t num_pages, void** plan_out) {
  using namespace q3;
  Q3_REQUIRE(block_table, "q3_decode_tp_create_paged: null block table");
  return decode_tp_create_impl(layers, n_layers, batch, hidden, q_heads, kv_heads, inter, max_seq,
                               eps, rope_cos, rope_sin, rope_rows, comm, block_table,
                               table_stride, page_tokens, num_pages, plan_out);
}

extern "C" int q3_decode_tp(void* plan, void* x, const int32_t* kv_len_dev, int64_t rope_delta,
                            q3_stream_t stream) {
  using namespace q3;
  using namespace q3::tp;
  Q3_REQUIRE(plan && x && kv_len_dev, "q3_decode_tp: null pointer");
  tp::Plan* pl = static_cast<tp::Plan*>(plan);
  Q3_REQUIRE(aligned(x, 16), "q3_decode_tp: x must be 16-byte aligned");
  Q3_REQUIRE(rope_delta >= 0, "q3_decode_tp: rope_delta must be >= 0");
  Params p = pl->p;
  p.X = static_cast<__nv_bfloat16*>(x);
  p.kv_len_dev = kv_len_dev;
  p.rope_delta = rope_delta;
  cudaStream_t s = (cudaStream_t)stream;
  // the grid barrier's and the attention pairs' arrival counters
  Q3_CUDA_CHECK(cudaMemsetAsync(p.pair_cnt, 0,
                                reinterpret_cast<char*>(p.gbar + 1) -
                                    reinterpret_cast<char*>(p.pair_cnt),
                                s));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl->grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = pl->smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  void (*kern)(Params) = pl->G == 1 ? decode_tp_kernel<1> : pl->G == 2 ? decode_tp_kernel<2>
                         : pl->G == 4 ? decode_tp_kernel<4> : decode_tp_kernel<8>;
  Q3_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, p));
  count_launch();
  return Q3_OK;
}

extern "C" int q3_decode_tp_destroy(void* plan) {
  using namespace q3;
  if (!plan) return Q3_OK;
  tp::Plan* pl = static_cast<tp::Plan*>(plan);
  cudaDeviceSynchronize();
  if (pl->dmem) cudaFree(pl->dmem);
  delete pl;
  return Q3_OK;
}
