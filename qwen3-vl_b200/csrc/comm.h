// Peer-memory communicator for the in-kernel tensor-parallel all-reduce.
//
// Every rank owns one device buffer (allocated by q3_comm_create) that its
// peers write into over NVLink; the buffers are exchanged as CUDA IPC handles
// and opened on every rank, so kernels receive plain peer pointers.
//
// Layout of a rank's buffer (max_tiles tiles of 64 output columns):
//   inbox    [2 parities][kMaxRanks sources][max_tiles][kArWords] 8-byte words
//   counters [max_tiles] uint32   (per-tile call numbers of this rank)
// Each inbox word carries two bf16 partial values and the call number f that
// wrote them, so a receiver knows a word has arrived when its flag reads f:
// no fence, no flag store and no atomic is needed to publish a partial, and
// 8-byte stores over NVLink land whole.  Call f uses parity f & 1; flags only
// grow and start at 0, so stale words never match.  Partials travel as bf16,
// the dtype the reference all-reduces (its o_proj/down outputs are bf16
// tensors, model_fused.py:266-267, 273-274).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace q3 {

constexpr int kMaxRanks = 8;
constexpr int kArCols = 64;    // output columns per exchanged tile
constexpr int kArTokens = 16;  // token slots per tile (decode M <= 16)
constexpr int kArTileElems = kArCols * kArTokens;
constexpr int kArWords = kArTileElems / 2;  // (2 x bf16 data, uint32 flag) words per tile

struct CommDev {
  uint2* inbox[kMaxRanks];  // each rank's inbox (peer-mapped; own for rank)
  uint32_t* counters;       // this rank's per-tile call numbers
  int rank, world, max_tiles;
  uint64_t wait_ns;         // bound of every wait on a peer's words
  int early_dependents;     // let the next kernel launch once the weights are consumed
};

struct Comm {
  int rank = 0, world = 1, max_tiles = 0;
  size_t bytes = 0;
  void* local = nullptr;             // this rank's buffer (cudaMalloc)
  void* peers[kMaxRanks] = {nullptr};  // opened IPC mappings (nullptr for self)
  int device = 0;
  bool open = false;
  bool attached[kMaxRanks] = {false};  // peers set by q3_comm_attach_peer (not IPC)
  uint64_t wait_ns = 2000000000ull;    // q3_comm_set_wait_limit
  CommDev dev() const;
};

// Range accepted for a communicator's wait limit: 1 ms .. 60 s.
constexpr uint64_t kMinWaitNs = 1000000ull;
constexpr uint64_t kMaxWaitNs = 60000000000ull;

inline size_t comm_data_bytes(int max_tiles) {
  return (size_t)2 * kMaxRanks * max_tiles * kArWords * sizeof(uint2);
}
inline size_t comm_bytes(int max_tiles) {
  return comm_data_bytes(max_tiles) + (size_t)max_tiles * sizeof(uint32_t);
}

}  // namespace q3
