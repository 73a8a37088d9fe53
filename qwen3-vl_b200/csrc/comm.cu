// Peer-memory communicator (CUDA IPC) and the fused row-parallel projection +
// all-reduce entry point.  See comm.h for the buffer layout.
#include <string.h>

#include "comm.h"
#include "common.cuh"

namespace q3 {

CommDev Comm::dev() const {
  CommDev d{};
  const size_t data_bytes = comm_data_bytes(max_tiles);
  for (int r = 0; r < kMaxRanks; ++r) {
    void* base = (r == rank) ? local : peers[r];
    d.inbox[r] = base ? reinterpret_cast<uint2*>(base) : nullptr;
  }
  d.counters = reinterpret_cast<uint32_t*>(static_cast<char*>(local) + data_bytes);
  d.rank = rank;
  d.world = world;
  d.max_tiles = max_tiles;
  d.wait_ns = wait_ns;
  return d;
}

// Decode-shaped projection with the all-reduce fused in (gemv.cu).
int launch_gemv_ar(const void* A, const void* W, void* C, const void* R, int M, int N, int K,
                   float* ss_out, const CommDev& comm, cudaStream_t s);

}  // namespace q3

extern "C" int q3_comm_create(int rank, int world, int64_t max_cols, void** comm_out,
                              void* ipc_handle_out) {
  using namespace q3;
  Q3_REQUIRE(comm_out && ipc_handle_out, "q3_comm_create: null pointer");
  Q3_REQUIRE(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world,
             "q3_comm_create: rank %d / world %d unsupported (max %d ranks)", rank, world,
             kMaxRanks);
  Q3_REQUIRE(max_cols > 0 && max_cols <= (1 << 20), "q3_comm_create: bad max_cols");
  Comm* c = new Comm();
  c->rank = rank;
  c->world = world;
  c->max_tiles = (int)((max_cols + kArCols - 1) / kArCols);
  c->bytes = comm_bytes(c->max_tiles);
  cudaGetDevice(&c->device);
  cudaError_t e = cudaMalloc(&c->local, c->bytes);
  if (e != cudaSuccess) {
    delete c;
    return fail(Q3_ERR_CUDA, "q3_comm_create: cudaMalloc(%zu) failed: %s", comm_bytes(0),
                cudaGetErrorString(e));
  }
  e = cudaMemset(c->local, 0, c->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->local);
  if (e != cudaSuccess) {
    cudaFree(c->local);
    delete c;
    return fail(Q3_ERR_CUDA, "q3_comm_create: %s", cudaGetErrorString(e));
  }
  memcpy(ipc_handle_out, &h, sizeof(h));
  *comm_out = c;
  return Q3_OK;
}

extern "C" int q3_comm_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int q3_comm_open_peers(void* comm, const void* all_handles) {
  using namespace q3;
  Q3_REQUIRE(comm && all_handles, "q3_comm_open_peers: null pointer");
  Comm* c = static_cast<Comm*>(comm);
  Q3_REQUIRE(!c->open, "q3_comm_open_peers: already open");
  const char* hs = static_cast<const char*>(all_handles);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hs + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (c->peers[q]) { cudaIpcCloseMemHandle(c->peers[q]); c->peers[q] = nullptr; }
      return fail(Q3_ERR_COMM, "q3_comm_open_peers: opening rank %d's buffer failed: %s", r,
                  cudaGetErrorString(e));
    }
    c->peers[r] = p;
  }
  c->open = true;
  return Q3_OK;
}

extern "C" int q3_init_comm(void* comm, int rank, int world, const void* all_handles) {
  using namespace q3;
  Q3_REQUIRE(comm && all_handles, "q3_init_comm: null pointer");
  const Comm* c = static_cast<const Comm*>(comm);
  Q3_REQUIRE(c->rank == rank && c->world == world,
             "q3_init_comm: communicator was created for rank %d of %d, not %d of %d", c->rank,
             c->world, rank, world);
  return q3_comm_open_peers(comm, all_handles);
}

extern "C" int q3_comm_buffer(const void* comm, void** buffer_out, size_t* bytes_out) {
  using namespace q3;
  Q3_REQUIRE(comm && buffer_out, "q3_comm_buffer: null pointer");
  const Comm* c = static_cast<const Comm*>(comm);
  *buffer_out = c->local;
  if (bytes_out) *bytes_out = c->bytes;
  return Q3_OK;
}

extern "C" int q3_comm_attach_peer(void* comm, int peer_rank, void* peer_buffer) {
  using namespace q3;
  Q3_REQUIRE(comm && peer_buffer, "q3_comm_attach_peer: null pointer");
  Comm* c = static_cast<Comm*>(comm);
  Q3_REQUIRE(peer_rank >= 0 && peer_rank < c->world && peer_rank != c->rank,
             "q3_comm_attach_peer: peer rank %d is not another rank of world %d", peer_rank,
             c->world);
  Q3_REQUIRE(!c->peers[peer_rank], "q3_comm_attach_peer: rank %d already has a buffer",
             peer_rank);
  Q3_REQUIRE(aligned(peer_buffer, 256), "q3_comm_attach_peer: buffer must be 256-byte aligned");
  c->peers[peer_rank] = peer_buffer;
  c->attached[peer_rank] = true;
  bool all = true;
  for (int r = 0; r < c->world; ++r)
    if (r != c->rank && !c->peers[r]) all = false;
  c->open = all;
  return Q3_OK;
}

extern "C" int q3_comm_set_wait_limit(void* comm, uint64_t wait_ns) {
  using namespace q3;
  Q3_REQUIRE(comm, "q3_comm_set_wait_limit: null pointer");
  Q3_REQUIRE(wait_ns >= kMinWaitNs && wait_ns <= kMaxWaitNs,
             "q3_comm_set_wait_limit: %llu ns outside [%llu, %llu]",
             (unsigned long long)wait_ns, (unsigned long long)kMinWaitNs,
             (unsigned long long)kMaxWaitNs);
  static_cast<Comm*>(comm)->wait_ns = wait_ns;
  return Q3_OK;
}

extern "C" int q3_comm_destroy(void* comm) {
  using namespace q3;
  if (!comm) return Q3_OK;
  Comm* c = static_cast<Comm*>(comm);
  cudaDeviceSynchronize();
  for (int r = 0; r < kMaxRanks; ++r)
    if (c->peers[r] && !c->attached[r]) cudaIpcCloseMemHandle(c->peers[r]);
  if (c->local) cudaFree(c->local);
  delete c;
  return Q3_OK;
}

extern "C" int q3_gemm_ar(const void* A, const void* W, void* C, int64_t M, int64_t N, int64_t K,
                          const void* residual, float* ss_out, void* comm, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(A && W && C && comm, "q3_gemm_ar: null pointer");
  Comm* c = static_cast<Comm*>(comm);
  Q3_REQUIRE(c->open || c->world == 1, "q3_gemm_ar: communicator peers not opened");
  Q3_REQUIRE(M >= 1 && M <= kArTokens, "q3_gemm_ar: M=%lld outside [1, %d] (decode shapes)",
             (long long)M, kArTokens);
  Q3_REQUIRE(N > 0 && N % kArCols == 0 && N / kArCols <= c->max_tiles,
             "q3_gemm_ar: N=%lld must be a multiple of %d and <= %d", (long long)N, kArCols,
             c->max_tiles * kArCols);
  Q3_REQUIRE(K > 0 && K % 32 == 0, "q3_gemm_ar: K=%lld must be a multiple of 32", (long long)K);
  Q3_REQUIRE(aligned(A, 16) && aligned(W, 16) && aligned(C, 16) &&
                 (!residual || aligned(residual, 16)),
             "q3_gemm_ar: pointers must be 16-byte aligned");
  return launch_gemv_ar(A, W, C, residual, (int)M, (int)N, (int)K, ss_out, c->dev(),
                        (cudaStream_t)stream);
}
