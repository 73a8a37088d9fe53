// Peer-memory communicator for the in-kernel tensor-parallel all-reduce.
//
// Every rank owns one device buffer (allocated by q3_comm_create) that its
// peers write into over NVLink; the buffers are exchanged as CUDA IPC handles
// and opened on every rank, so kernels receive plain peer pointers.
//
// Layout of a rank's buffer (max_tiles tiles of 64 output columns):
//   data     [2 parities][kMaxRanks sources][max_tiles][64 cols x 16 tokens] bf16
//   flags    [kMaxRanks sources][max_tiles] uint32   (written by the source rank)
//   counters [max_tiles] uint32                      (local call sequence numbers)
// A tile exchange of call number f (per tile, counted identically on every
// rank) writes parity f & 1 and raises the source's flag to f.  Partials travel
// as bf16, the dtype the reference all-reduces (its o_proj/down outputs are
// bf16 tensors, model_fused.py:266-267, 273-274).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace q3 {

constexpr int kMaxRanks = 8;
constexpr int kArCols = 64;    // output columns per exchanged tile
constexpr int kArTokens = 16;  // token slots per tile (decode M <= 16)
constexpr int kArTileElems = kArCols * kArTokens;

struct CommDev {
  __nv_bfloat16* data[kMaxRanks];  // base of each rank's data region (peer-mapped)
  uint32_t* flags[kMaxRanks];   // base of each rank's flag region (peer-mapped)
  uint32_t* counters;           // this rank's per-tile sequence numbers
  int rank, world, max_tiles;
};

struct Comm {
  int rank = 0, world = 1, max_tiles = 0;
  size_t bytes = 0;
  void* local = nullptr;             // this rank's buffer (cudaMalloc)
  void* peers[kMaxRanks] = {nullptr};  // opened IPC mappings (nullptr for self)
  int device = 0;
  bool open = false;
  CommDev dev() const;
};

inline size_t comm_data_bytes(int max_tiles) {
  return (size_t)2 * kMaxRanks * max_tiles * kArTileElems * sizeof(__nv_bfloat16);
}
inline size_t comm_bytes(int max_tiles) {
  return comm_data_bytes(max_tiles) + (size_t)kMaxRanks * max_tiles * sizeof(uint32_t) +
         (size_t)max_tiles * sizeof(uint32_t);
}

}  // namespace q3
