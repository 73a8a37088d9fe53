// a10/a11 + 8(e), prefill shapes: the row-parallel projection fused with the
// tensor-parallel all-reduce as a two-shot exchange over NVLink peer memory.
// Replaces `x @ W`, dist.all_reduce(SUM) and the residual add of forward_layer
// (model_fused.py:265-269 for o_proj, :272-275 for down_proj) when the call
// carries many tokens (prefill), where the decode path's one-shot push
// (every rank sends its whole partial to every peer) would move world - 1
// times the data.
//
//   1. reduce-scatter, inside the GEMM: the output rows are cut into `world`
//      stripes of whole 128-row tiles, stripe o owned by rank o.  The tcgen05
//      GEMM's epilogue (gemm.cu, kEpiPushStripe) writes each bf16 partial tile
//      straight into its owner's receive stripe for this source rank, then each
//      epilogue warp publishes a flag for its 32 rows (a system-scope release
//      store of the call number).  The transfer of finished tiles overlaps the
//      MMAs of the next ones.
//   2. reduce + all-gather (rs_ag_kernel, next on the stream): each rank waits
//      for the flags of its own tiles from every source, sums the partials in
//      rank order in fp32, rounds to bf16, adds the residual (bf16(residual +
//      bf16(sum)), the reference's rounding points), writes the rows to its
//      output and to its reduced stripe, and publishes a flag per tile; then
//      it pulls every other owner's reduced tiles with peer loads as their
//      flags appear.  All ranks hold identical bits.
//
// Flags carry call numbers (which only grow), so nothing is ever reset.  No
// rank can overwrite data a peer still reads: a rank pushes call f + 1 only
// after it has gathered every owner's reduced tiles of call f, so every owner
// has finished reading the partials of call f, and an owner rewrites its
// reduced stripe for f + 1 only after every source pushed f + 1, i.e. after
// every rank finished gathering call f.  Buffers still alternate by call
// parity, as a margin.  Every wait is bounded: after the
// communicator's wait limit (2 s unless set) the kernel records 0x701 (partials) or 0x702 (reduced tiles)
// in the device error word and skips the tile.  No TMA or bulk copy touches
// peer memory: peer traffic is plain stores (epilogue) and loads (gather).
#include <string.h>

#include "comm.h"
#include "common.cuh"

namespace q3 {

int launch_gemm_push(const void* A, const void* W, int M, int N, int K,
                     __nv_bfloat16* const* recv, uint32_t* const* flags, int world, int stripe,
                     uint32_t call, cudaStream_t s);

namespace {

constexpr int kPTile = 128;   // rows per GEMM tile (and stripe granule)
constexpr int kPTileN = 256;  // columns per GEMM tile
constexpr int kRsThreads = 256;

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct PrefillComm {
  int rank = 0, world = 1;
  int64_t max_rows = 0, max_cols = 0;
  int64_t stripe_max = 0, max_tiles = 0;
  size_t off_recv = 0, off_red = 0, off_pflag = 0, off_rflag = 0, bytes = 0;
  char* local = nullptr;
  char* peers[kMaxRanks] = {nullptr};
  bool attached[kMaxRanks] = {false};  // peers set by q3_prefill_comm_attach_peer (not IPC)
  bool open = false;
  uint32_t calls = 0;
  uint64_t wait_ns = 2000000000ull;    // q3_prefill_comm_set_wait_limit

  char* base(int r) const { return r == rank ? local : peers[r]; }
  // recv[parity][src]: stripe_max x max_cols bf16
  size_t recv_at(int par, int src) const {
    return off_recv + ((size_t)par * world + src) * (size_t)stripe_max * max_cols * 2;
  }
  size_t red_at(int par) const { return off_red + (size_t)par * stripe_max * max_cols * 2; }
  // pflag[parity][src][tile][4]
  size_t pflag_at(int par, int src) const {
    return off_pflag + ((size_t)par * world + src) * (size_t)max_tiles * 4 * sizeof(uint32_t);
  }
  size_t rflag_at(int par) const { return off_rflag + (size_t)par * max_tiles * sizeof(uint32_t); }
};

struct RsParams {
  const __nv_bfloat16* recv[kMaxRanks];  // own receive stripes, per source
  const uint32_t* pflag[kMaxRanks];      // own push flags, per source
  __nv_bfloat16* red_own;
  uint32_t* rflag_own;
  const __nv_bfloat16* red_peer[kMaxRanks];  // every owner's reduced stripe
  const uint32_t* rflag_peer[kMaxRanks];
  __nv_bfloat16* C;
  const __nv_bfloat16* R;
  int M, N, stripe, n_tiles, world, rank;
  uint32_t call;
  uint64_t wait_ns;  // the communicator's wait limit
  int* err;
};

// Spin until *f == want or the tile's deadline (one budget of `limit` ns for
// all the flags of a tile) passes.
__device__ bool wait_flag(const uint32_t* f, uint32_t want, uint64_t t0, uint64_t limit, int* err,
                          int code) {
  uint32_t spins = 0;
  while (ld_acquire_sys(f) != want) {
    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > limit) {
      report_timeout(err, code);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void add8(float (&a)[8], uint4 u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    a[2 * i] += f.x;
    a[2 * i + 1] += f.y;
  }
}

__global__ void __launch_bounds__(kRsThreads) rs_ag_kernel(RsParams p) {
  // the GEMM that pushed this rank's partials has completed before any wait
  pdl_wait();
  pdl_launch();
  __shared__ int go;
  const int m_tiles = (p.M + kPTile - 1) / kPTile;
  const int own_r0 = p.rank * p.stripe;
  const int own_r1 = min(own_r0 + p.stripe, p.M);
  const int own_m0 = min(own_r0 / kPTile, m_tiles);
  const int own_m1 = own_r1 > own_r0 ? (own_r1 + kPTile - 1) / kPTile : own_m0;
  const int n_own = (own_m1 - own_m0) * p.n_tiles;
  const int n_all = m_tiles * p.n_tiles;

  for (int item = blockIdx.x; item < n_all; item += gridDim.x) {
    const bool mine = item < n_own;
    int mt, nt;
    if (mine) {
      mt = own_m0 + item / p.n_tiles;
      nt = item % p.n_tiles;
    } else {
      const int j = item - n_own;
      mt = j / p.n_tiles;
      if (mt >= own_m0) mt += own_m1 - own_m0;
      nt = j % p.n_tiles;
    }
    const int tile = mt * p.n_tiles + nt;
    const int r0 = mt * kPTile, r1 = min(r0 + kPTile, p.M);
    const int c0 = nt * kPTileN, c1 = min(c0 + kPTileN, p.N);
    const int owner = r0 / p.stripe;
    if (threadIdx.x == 0) {
      bool ok = true;
      const uint64_t t0 = globaltimer_ns();
      if (mine) {
        for (int src = 0; src < p.world && ok; ++src)
          for (int sub = 0; sub < 4 && ok; ++sub)
            ok = wait_flag(p.pflag[src] + (int64_t)tile * 4 + sub, p.call, t0, p.wait_ns,
                           p.err, 0x701);
      } else {
        ok = wait_flag(p.rflag_peer[owner] + tile, p.call, t0, p.wait_ns, p.err, 0x702);
      }
      go = ok;
    }
    __syncthreads();
    if (go) {
      const int nvec = (c1 - c0) / 8;
      const int total = (r1 - r0) * nvec;
      if (mine) {
        for (int i = threadIdx.x; i < total; i += kRsThreads) {
          const int row = r0 + i / nvec, col = c0 + (i % nvec) * 8;
          const int64_t lo = (int64_t)(row - own_r0) * p.N + col;
          float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          // data written by peers: read at L2 (ld.global.cg), never from a
          // line this SM may hold from an earlier call
          for (int src = 0; src < p.world; ++src)
            add8(a, __ldcg(reinterpret_cast<const uint4*>(p.recv[src] + lo)));
          uint32_t o[4];
          if (p.R) {
            const uint4 ru = *reinterpret_cast<const uint4*>(p.R + (int64_t)row * p.N + col);
            const uint32_t rw[4] = {ru.x, ru.y, ru.z, ru.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 r = unpack_bf16x2(rw[k]);
              o[k] = pack_bf16x2(r.x + rbf(a[2 * k]), r.y + rbf(a[2 * k + 1]));
            }
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) o[k] = pack_bf16x2(a[2 * k], a[2 * k + 1]);
          }
          const uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(p.C + (int64_t)row * p.N + col) = ov;
          *reinterpret_cast<uint4*>(p.red_own + lo) = ov;
        }
      } else {
        const __nv_bfloat16* src = p.red_peer[owner];
        const int o_r0 = owner * p.stripe;
        // four peer loads in flight per thread before their stores
        for (int i0 = threadIdx.x; i0 < total; i0 += 4 * kRsThreads) {
          uint4 v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = i0 + u * kRsThreads;
            if (i < total) {
              const int row = r0 + i / nvec, col = c0 + (i % nvec) * 8;
              v[u] = __ldcg(reinterpret_cast<const uint4*>(src + (int64_t)(row - o_r0) * p.N + col));
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = i0 + u * kRsThreads;
            if (i < total) {
              const int row = r0 + i / nvec, col = c0 + (i % nvec) * 8;
              *reinterpret_cast<uint4*>(p.C + (int64_t)row * p.N + col) = v[u];
            }
          }
        }
      }
    }
    __syncthreads();
    if (mine && go && threadIdx.x == 0) {
      __threadfence_system();
      st_release_sys(p.rflag_own + tile, p.call);
    }
  }
}

}  // namespace
}  // namespace q3

extern "C" int q3_prefill_comm_create(int rank, int world, int64_t max_rows, int64_t max_cols,
                                      void** comm_out, void* ipc_handle_out) {
  using namespace q3;
  Q3_REQUIRE(comm_out && ipc_handle_out, "q3_prefill_comm_create: null pointer");
  Q3_REQUIRE(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world,
             "q3_prefill_comm_create: rank %d / world %d unsupported (max %d ranks)", rank, world,
             kMaxRanks);
  Q3_REQUIRE(max_rows > 0 && max_rows <= (1 << 20) && max_cols > 0 && max_cols % 32 == 0 &&
                 max_cols <= (1 << 16),
             "q3_prefill_comm_create: bad max_rows=%lld / max_cols=%lld (a multiple of 32)",
             (long long)max_rows, (long long)max_cols);
  PrefillComm* c = new PrefillComm();
  c->rank = rank;
  c->world = world;
  c->max_rows = max_rows;
  c->max_cols = max_cols;
  c->stripe_max = ((max_rows + world - 1) / world + kPTile - 1) / kPTile * kPTile;
  c->max_tiles = ((max_rows + kPTile - 1) / kPTile) * ((max_cols + kPTileN - 1) / kPTileN);
  size_t off = 0;
  c->off_recv = off;
  off = align256(off + (size_t)2 * world * c->stripe_max * max_cols * 2);
  c->off_red = off;
  off = align256(off + (size_t)2 * c->stripe_max * max_cols * 2);
  c->off_pflag = off;
  off = align256(off + (size_t)2 * world * c->max_tiles * 4 * sizeof(uint32_t));
  c->off_rflag = off;
  off = align256(off + (size_t)2 * c->max_tiles * sizeof(uint32_t));
  c->bytes = off;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&c->local), c->bytes);
  if (e != cudaSuccess) {
    const size_t want = c->bytes;
    delete c;
    return fail(Q3_ERR_CUDA, "q3_prefill_comm_create: cudaMalloc(%zu) failed: %s", want,
                cudaGetErrorString(e));
  }
  // flags start at 0 (call numbers start at 1); the data regions need no init
  e = cudaMemset(c->local + c->off_pflag, 0, c->bytes - c->off_pflag);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->local);
  if (e != cudaSuccess) {
    cudaFree(c->local);
    delete c;
    return fail(Q3_ERR_CUDA, "q3_prefill_comm_create: %s", cudaGetErrorString(e));
  }
  memcpy(ipc_handle_out, &h, sizeof(h));
  *comm_out = c;
  return Q3_OK;
}

extern "C" int q3_prefill_comm_open(void* comm, const void* all_handles) {
  using namespace q3;
  Q3_REQUIRE(comm && all_handles, "q3_prefill_comm_open: null pointer");
  PrefillComm* c = static_cast<PrefillComm*>(comm);
  Q3_REQUIRE(!c->open, "q3_prefill_comm_open: already open");
  const char* hs = static_cast<const char*>(all_handles);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hs + (size_t)r * sizeof(h), sizeof(h));
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (c->peers[q]) { cudaIpcCloseMemHandle(c->peers[q]); c->peers[q] = nullptr; }
      return fail(Q3_ERR_COMM, "q3_prefill_comm_open: opening rank %d's buffer failed: %s", r,
                  cudaGetErrorString(e));
    }
    c->peers[r] = static_cast<char*>(ptr);
  }
  c->open = true;
  return Q3_OK;
}

extern "C" int q3_prefill_comm_buffer(const void* comm, void** buffer_out, size_t* bytes_out) {
  using namespace q3;
  Q3_REQUIRE(comm && buffer_out, "q3_prefill_comm_buffer: null pointer");
  const PrefillComm* c = static_cast<const PrefillComm*>(comm);
  *buffer_out = c->local;
  if (bytes_out) *bytes_out = c->bytes;
  return Q3_OK;
}

extern "C" int q3_prefill_comm_attach_peer(void* comm, int peer_rank, void* peer_buffer) {
  using namespace q3;
  Q3_REQUIRE(comm && peer_buffer, "q3_prefill_comm_attach_peer: null pointer");
  PrefillComm* c = static_cast<PrefillComm*>(comm);
  Q3_REQUIRE(peer_rank >= 0 && peer_rank < c->world && peer_rank != c->rank,
             "q3_prefill_comm_attach_peer: peer rank %d is not another rank of world %d",
             peer_rank, c->world);
  Q3_REQUIRE(!c->peers[peer_rank], "q3_prefill_comm_attach_peer: rank %d already has a buffer",
             peer_rank);
  Q3_REQUIRE(aligned(peer_buffer, 256),
             "q3_prefill_comm_attach_peer: buffer must be 256-byte aligned");
  c->peers[peer_rank] = static_cast<char*>(peer_buffer);
  c->attached[peer_rank] = true;
  bool all = true;
  for (int r = 0; r < c->world; ++r)
    if (r != c->rank && !c->peers[r]) all = false;
  c->open = all;
  return Q3_OK;
}

extern "C" int q3_prefill_comm_set_wait_limit(void* comm, uint64_t wait_ns) {
  using namespace q3;
  Q3_REQUIRE(comm, "q3_prefill_comm_set_wait_limit: null pointer");
  Q3_REQUIRE(wait_ns >= kMinWaitNs && wait_ns <= kMaxWaitNs,
             "q3_prefill_comm_set_wait_limit: %llu ns outside [%llu, %llu]",
             (unsigned long long)wait_ns, (unsigned long long)kMinWaitNs,
             (unsigned long long)kMaxWaitNs);
  static_cast<PrefillComm*>(comm)->wait_ns = wait_ns;
  return Q3_OK;
}

extern "C" int q3_prefill_comm_destroy(void* comm) {
  using namespace q3;
  if (!comm) return Q3_OK;
  PrefillComm* c = static_cast<PrefillComm*>(comm);
  cudaDeviceSynchronize();
  for (int r = 0; r < kMaxRanks; ++r)
    if (c->peers[r] && !c->attached[r]) cudaIpcCloseMemHandle(c->peers[r]);
  if (c->local) cudaFree(c->local);
  delete c;
  return Q3_OK;
}

extern "C" int q3_gemm_allreduce(const void* A, const void* W, void* C, int64_t M, int64_t N,
                                 int64_t K, const void* residual, void* comm,
                                 q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(A && W && C && comm, "q3_gemm_allreduce: null pointer");
  PrefillComm* c = static_cast<PrefillComm*>(comm);
  Q3_REQUIRE(c->open || c->world == 1, "q3_gemm_allreduce: communicator peers not opened");
  Q3_REQUIRE(M > 16 && M <= c->max_rows,
             "q3_gemm_allreduce: M=%lld outside (16, max_rows=%lld] (decode shapes use "
             "q3_gemm_ar)",
             (long long)M, (long long)c->max_rows);
  Q3_REQUIRE(N > 0 && N % 32 == 0 && N <= c->max_cols,
             "q3_gemm_allreduce: N=%lld must be a multiple of 32 and <= %lld", (long long)N,
             (long long)c->max_cols);
  Q3_REQUIRE(K > 0 && K % 32 == 0 && K < (1ll << 31),
             "q3_gemm_allreduce: K=%lld must be a multiple of 32", (long long)K);
  Q3_REQUIRE(aligned(A, 16) && aligned(W, 16) && aligned(C, 16) &&
                 (!residual || aligned(residual, 16)),
             "q3_gemm_allreduce: pointers must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  const uint32_t call = ++c->calls;
  const int par = (int)(call & 1u);
  const int world = c->world;
  const int stripe = (int)(((M + world - 1) / world + kPTile - 1) / kPTile * kPTile);
  __nv_bfloat16* recv[kMaxRanks] = {nullptr};
  uint32_t* flags[kMaxRanks] = {nullptr};
  RsParams rp{};
  for (int o = 0; o < world; ++o) {
    // where this rank's partial rows for owner o go
    recv[o] = reinterpret_cast<__nv_bfloat16*>(c->base(o) + c->recv_at(par, c->rank));
    flags[o] = reinterpret_cast<uint32_t*>(c->base(o) + c->pflag_at(par, c->rank));
    // what this rank reads: every source's partial of its stripe, every
    // owner's reduced stripe
    rp.recv[o] = reinterpret_cast<const __nv_bfloat16*>(c->local + c->recv_at(par, o));
    rp.pflag[o] = reinterpret_cast<const uint32_t*>(c->local + c->pflag_at(par, o));
    rp.red_peer[o] = reinterpret_cast<const __nv_bfloat16*>(c->base(o) + c->red_at(par));
    rp.rflag_peer[o] = reinterpret_cast<const uint32_t*>(c->base(o) + c->rflag_at(par));
  }
  rp.red_own = reinterpret_cast<__nv_bfloat16*>(c->local + c->red_at(par));
  rp.rflag_own = reinterpret_cast<uint32_t*>(c->local + c->rflag_at(par));
  rp.C = static_cast<__nv_bfloat16*>(C);
  rp.R = static_cast<const __nv_bfloat16*>(residual);
  rp.M = (int)M;
  rp.N = (int)N;
  rp.stripe = stripe;
  rp.n_tiles = (int)((N + kPTileN - 1) / kPTileN);
  rp.world = world;
  rp.rank = c->rank;
  rp.call = call;
  rp.wait_ns = c->wait_ns;
  rp.err = device_error_word();
  int rc = launch_gemm_push(A, W, (int)M, (int)N, (int)K, recv, flags, world, stripe, call, s);
  if (rc) return rc;
  return launch_ex(rs_ag_kernel, dim3(num_sms()), dim3(kRsThreads), 0, s, 1, rp);
}
