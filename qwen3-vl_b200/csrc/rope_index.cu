// Multimodal 3-axis position ids (M-RoPE rows) and per-sequence rope deltas,
// built on the device from the token-type map and the vision grids.
//
// Restates transformers 5.5.0 modeling_qwen3_vl.py:1031-1122
// (Qwen3VLModel.get_rope_index) with get_vision_position_ids :975-1029
// (temporal merge 1, time interval 1):
//   - a video of grid (t, h, w) is t frames of grid (1, h, w);
//   - the kept tokens of a sequence (mask != 0) are cut into maximal runs of
//     one type (0 text, 1 image, 2 video frame);
//   - a text run takes p, p+1, ... on all three axes and advances p by its
//     length;
//   - an image / frame run takes the next grid of its kind (grids are consumed
//     in batch order) and token i of the run gets t = p, h = p + i / (w' t),
//     w = p + i % w', with h' = h / merge, w' = w / merge; p advances by
//     max(h, w) / merge;
//   - masked tokens keep position 0; delta = max position + 1 - kept tokens.
//
// Layout: one CTA per sequence.  A first launch counts each sequence's image
// and frame runs (so every sequence knows the first grid it consumes); the
// second walks the sequence in chunks of kThreads x kItems tokens with three
// dependent block scans per chunk -- (1) the previous kept token's type and
// the kept-token index, (2) run starts per kind and the last run start, (3)
// the position advance -- carrying each scan's total into the next chunk.
// The work is integer and latency bound (one pass over the 4-byte types and
// mask, 24 bytes of positions out per token).
//
// Errors are per-sequence status words (0 = ok), the cases the reference
// rejects: more vision runs than grids, a run whose length differs from its
// grid's token count, a type outside {0, 1, 2}, a sequence with no kept token.
#include "common.cuh"

namespace q3 {
namespace {

constexpr int kThreads = 512;
constexpr int kItems = 8;
constexpr int kChunk = kThreads * kItems;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxVideos = 4096;

enum : int {
  kStRunsExceedGrids = 1,
  kStRunLength = 2,
  kStBadType = 3,
  kStNoKeptToken = 4,
};

struct Sum {
  __device__ int operator()(int a, int b) const { return a + b; }
};
struct Max {
  __device__ int operator()(int a, int b) const { return a > b ? a : b; }
};

// Exclusive block scan of one int per thread (commutative op); returns the
// exclusive value and the block total.  sh holds kWarps + 1 ints.
template <class Op>
__device__ int block_scan(int v, int ident, Op op, int* sh, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x = op(x, y);
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kWarps ? sh[lane] : ident;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w = op(w, y);
    }
    __syncwarp();
    if (lane < kWarps) sh[lane] = w;
  }
  __syncthreads();
  const int before_warp = warp ? sh[warp - 1] : ident;
  total = sh[kWarps - 1];
  int excl = __shfl_up_sync(0xffffffffu, x, 1);
  if (lane == 0) excl = ident;
  __syncthreads();  // sh is reused by the next scan
  return op(before_warp, excl);
}

struct Grid {
  int64_t t, h, w;
};

// Grid of the ord-th run of `kind` (image: image_thw[ord]; frame: the video
// whose frame range holds ord, as a one-frame grid).  Returns false when the
// runs outnumber the grids.
__device__ bool run_grid(int kind, int ord, const int64_t* img, int n_img, const int64_t* vid,
                         int n_vid, const int* vpre, Grid& g) {
  if (ord < 0) return false;
  if (kind == 1) {
    if (ord >= n_img) return false;
    g = {img[3 * ord], img[3 * ord + 1], img[3 * ord + 2]};
    return true;
  }
  if (ord >= vpre[n_vid]) return false;
  int lo = 0, hi = n_vid;  // largest v with vpre[v] <= ord
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (vpre[mid] <= ord) lo = mid; else hi = mid;
  }
  g = {1, vid[3 * lo + 1], vid[3 * lo + 2]};
  return true;
}

__device__ __forceinline__ int64_t grid_tokens(const Grid& g, int merge) {
  return g.t * (g.h / merge) * (g.w / merge);
}

__device__ __forceinline__ void load_chunk(const int32_t* types, const int32_t* mask, int64_t base,
                                           int64_t S, int ty[kItems], bool kp[kItems]) {
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int64_t s = base + i;
    const bool in = s < S;
    const int t = in ? types[s] : 0;
    ty[i] = (t >= 0 && t <= 2) ? t : 3;  // class 3: a type the reference does not know
    kp[i] = in && (mask == nullptr || mask[s] != 0);
  }
}

// Previous kept type for each item given the carry from earlier tokens;
// returns the last kept type of the chunk through `last` (unchanged if none).
__device__ __forceinline__ void prev_types(const int ty[kItems], const bool kp[kItems], int carry,
                                           int* sh, int pv[kItems], int& last) {
  int code = 0;  // (item index in chunk + 1) * 4 + type of the thread's last kept token
#pragma unroll
  for (int i = 0; i < kItems; ++i)
    if (kp[i]) code = ((threadIdx.x * kItems + i) + 1) * 4 + ty[i];
  int tot;
  const int before = block_scan(code, 0, Max(), sh, tot);
  int p = before ? (before & 3) : carry;
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    pv[i] = p;
    if (kp[i]) p = ty[i];
  }
  last = tot ? (tot & 3) : carry;
}

__global__ void __launch_bounds__(kThreads) rope_runs_kernel(const int32_t* __restrict__ types,
                                                            const int32_t* __restrict__ mask,
                                                            int64_t S, int* __restrict__ counts) {
  pdl_wait();
  __shared__ int sh[kWarps + 1];
  const int b = blockIdx.x;
  const int32_t* ty_row = types + (int64_t)b * S;
  const int32_t* mk_row = mask ? mask + (int64_t)b * S : nullptr;
  int carry = -1, n_img = 0, n_vid = 0;
  for (int64_t c0 = 0; c0 < S; c0 += kChunk) {
    int ty[kItems], pv[kItems];
    bool kp[kItems];
    load_chunk(ty_row, mk_row, c0 + (int64_t)threadIdx.x * kItems, S, ty, kp);
    int last;
    prev_types(ty, kp, carry, sh, pv, last);
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      if (kp[i] && pv[i] != ty[i]) {
        n_img += ty[i] == 1;
        n_vid += ty[i] == 2;
      }
    }
    carry = last;
  }
  int tot_img, tot_vid;
  block_scan(n_img, 0, Sum(), sh, tot_img);
  block_scan(n_vid, 0, Sum(), sh, tot_vid);
  if (threadIdx.x == 0) {
    counts[2 * b] = tot_img;
    counts[2 * b + 1] = tot_vid;
  }
}

struct IndexArgs {
  const int32_t* types;
  const int32_t* mask;
  int64_t S;
  const int64_t* img;
  int n_img;
  const int64_t* vid;
  int n_vid;
  int merge;
  const int* counts;
  int* status;
  int64_t* pos;    // [3, B, S]
  int64_t* delta;  // [B]
  int B;
};

__device__ __forceinline__ void flag(int* status, int code) { atomicMax(status, code); }

__global__ void __launch_bounds__(kThreads) rope_index_kernel(IndexArgs a) {
  pdl_wait();
  extern __shared__ int vpre[];  // [n_vid + 1] exclusive prefix of the videos' frame counts
  __shared__ int sh[kWarps + 1];
  const int b = blockIdx.x;
  const int tid = threadIdx.x;

  // grids consumed by earlier sequences
  int part_img = 0, part_vid = 0;
  for (int j = tid; j < b; j += kThreads) {
    part_img += a.counts[2 * j];
    part_vid += a.counts[2 * j + 1];
  }
  int img_base, vid_base;
  block_scan(part_img, 0, Sum(), sh, img_base);
  block_scan(part_vid, 0, Sum(), sh, vid_base);

  // frame prefix over the videos
  int run = 0;
  for (int v0 = 0; v0 < a.n_vid; v0 += kThreads) {
    const int v = v0 + tid;
    const int64_t tv = v < a.n_vid ? a.vid[3 * v] : 0;
    const int t = tv > 0 ? (int)tv : 0;
    int tot;
    const int ex = block_scan(t, 0, Sum(), sh, tot);
    if (v < a.n_vid) vpre[v] = run + ex;
    run += tot;
  }
  if (tid == 0) vpre[a.n_vid] = run;
  __syncthreads();

  const int32_t* ty_row = a.types + (int64_t)b * a.S;
  const int32_t* mk_row = a.mask ? a.mask + (int64_t)b * a.S : nullptr;
  const int64_t plane = (int64_t)a.B * a.S;
  int64_t* pt = a.pos + (int64_t)b * a.S;
  int* st = a.status + b;

  // carries across chunks
  int c_prev_type = -1;  // type of the last kept token so far (-1: none)
  int c_kept = 0;        // kept tokens so far
  int c_img = 0, c_vid = 0;  // image / frame runs started so far (this sequence)
  int c_start = -1;      // kept index of the last run start
  int c_p = 0;           // position advance so far
  int my_max = -1;

  for (int64_t c0 = 0; c0 < a.S; c0 += kChunk) {
    const int64_t base = c0 + (int64_t)tid * kItems;
    int ty[kItems], pv[kItems];
    bool kp[kItems];
    load_chunk(ty_row, mk_row, base, a.S, ty, kp);
    int last_type;
    prev_types(ty, kp, c_prev_type, sh, pv, last_type);

    // (1) kept-token index; run starts
    bool sf[kItems];
    int n_kept = 0, n_img = 0, n_vid = 0, last_start = -1;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      if (kp[i] && ty[i] == 3) flag(st, kStBadType);
      sf[i] = kp[i] && pv[i] != ty[i];
      n_kept += kp[i];
    }
    int tot_kept;
    const int kept_ex = c_kept + block_scan(n_kept, 0, Sum(), sh, tot_kept);
    int ci[kItems];
    {
      int k = kept_ex;
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        ci[i] = k;
        k += kp[i];
        if (sf[i]) {
          n_img += ty[i] == 1;
          n_vid += ty[i] == 2;
          last_start = ci[i];
        }
      }
    }

    // (2) run ordinals and the last run start before each token
    int tot_img, tot_vid, tot_start;
    int img_ex = c_img + block_scan(n_img, 0, Sum(), sh, tot_img);
    int vid_ex = c_vid + block_scan(n_vid, 0, Sum(), sh, tot_vid);
    int start_ex = block_scan(last_start, -1, Max(), sh, tot_start);
    if (start_ex < 0) start_ex = c_start;

    Grid g[kItems];
    int run_start[kItems];
    int w_loc = 0;
    int wv[kItems];
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      if (sf[i]) {
        // the run that ends here: a vision run must have filled its grid
        if (pv[i] == 1 || pv[i] == 2) {
          Grid pg;
          const int ord = (pv[i] == 1 ? img_base + img_ex : vid_base + vid_ex) - 1;
          if (run_grid(pv[i], ord, a.img, a.n_img, a.vid, a.n_vid, vpre, pg) &&
              grid_tokens(pg, a.merge) != (int64_t)(ci[i] - start_ex))
            flag(st, kStRunLength);
        }
        if (ty[i] == 1) ++img_ex;
        if (ty[i] == 2) ++vid_ex;
        start_ex = ci[i];
      }
      run_start[i] = start_ex;
      wv[i] = 0;
      g[i] = {0, 0, 0};
      if (kp[i]) {
        if (ty[i] == 0) {
          wv[i] = 1;
        } else if (ty[i] != 3) {
          const int ord = (ty[i] == 1 ? img_base + img_ex : vid_base + vid_ex) - 1;
          if (!run_grid(ty[i], ord, a.img, a.n_img, a.vid, a.n_vid, vpre, g[i])) {
            flag(st, kStRunsExceedGrids);
          } else if (ci[i] - run_start[i] >= grid_tokens(g[i], a.merge)) {
            flag(st, kStRunLength);
          }
          if (sf[i]) {
            const int64_t hw = g[i].h > g[i].w ? g[i].h : g[i].w;
            wv[i] = (int)(hw / a.merge);
          }
        }
      }
      w_loc += wv[i];
    }

    // (3) positions
    int tot_w;
    int p = c_p + block_scan(w_loc, 0, Sum(), sh, tot_w);
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int64_t s = base + i;
      int64_t pt_t = 0, pt_h = 0, pt_w = 0;
      if (kp[i]) {
        if (ty[i] == 0) {
          pt_t = pt_h = pt_w = p;
        } else {
          const int64_t hh = g[i].h / a.merge, ww = g[i].w / a.merge;
          const int64_t p0 = sf[i] ? p : p - (g[i].h > g[i].w ? g[i].h : g[i].w) / a.merge;
          const int64_t o = ci[i] - run_start[i];
          pt_t = p0;
          if (ww > 0 && hh > 0 && g[i].t > 0) {
            pt_h = p0 + o / (ww * g[i].t);
            pt_w = p0 + o % ww;
          }
        }
        const int64_t m = pt_h > pt_w ? pt_h : pt_w;
        const int64_t mm = m > pt_t ? m : pt_t;
        if (mm > my_max) my_max = (int)mm;
      }
      p += wv[i];
      if (s < a.S) {
        pt[s] = pt_t;
        pt[plane + s] = pt_h;
        pt[2 * plane + s] = pt_w;
      }
    }

    c_prev_type = last_type;
    c_kept += tot_kept;
    c_img += tot_img;
    c_vid += tot_vid;
    if (tot_start >= 0) c_start = tot_start;
    c_p += tot_w;
  }

  int seq_max;
  block_scan(my_max, -1, Max(), sh, seq_max);
  if (tid == 0) {
    if (c_kept == 0) {
      flag(st, kStNoKeptToken);
      a.delta[b] = 0;
    } else {
      a.delta[b] = (int64_t)seq_max + 1 - c_kept;
      // the final run must also have filled its grid
      if (c_prev_type == 1 || c_prev_type == 2) {
        Grid pg;
        const int ord = (c_prev_type == 1 ? img_base + c_img : vid_base + c_vid) - 1;
        if (run_grid(c_prev_type, ord, a.img, a.n_img, a.vid, a.n_vid, vpre, pg) &&
            grid_tokens(pg, a.merge) != (int64_t)(c_kept - c_start))
          flag(st, kStRunLength);
      }
    }
  }
}

}  // namespace
}  // namespace q3

extern "C" size_t q3_rope_index_workspace_bytes(int B) {
  return B > 0 ? (size_t)2 * B * sizeof(int) : 0;
}

extern "C" int q3_rope_index(const int32_t* types, const int32_t* mask, int B, int64_t S,
                             const int64_t* image_thw, int n_image, const int64_t* video_thw,
                             int n_video, int merge, int64_t* pos_out, int64_t* delta_out,
                             int32_t* status_out, void* workspace, size_t workspace_bytes,
                             q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(B >= 0 && S >= 0 && S < (int64_t)1 << 30, "q3_rope_index: bad shape B=%d S=%lld", B,
             (long long)S);
  if (B == 0) return Q3_OK;
  Q3_REQUIRE(types && pos_out && delta_out && status_out && workspace,
             "q3_rope_index: null pointer");
  Q3_REQUIRE(merge > 0, "q3_rope_index: merge must be positive (got %d)", merge);
  Q3_REQUIRE(n_image >= 0 && (n_image == 0 || image_thw), "q3_rope_index: image grids");
  Q3_REQUIRE(n_video >= 0 && n_video <= kMaxVideos && (n_video == 0 || video_thw),
             "q3_rope_index: video grids (at most %d videos)", kMaxVideos);
  Q3_REQUIRE(workspace_bytes >= q3_rope_index_workspace_bytes(B),
             "q3_rope_index: workspace of %zu bytes, need %zu", workspace_bytes,
             q3_rope_index_workspace_bytes(B));
  Q3_REQUIRE(aligned(types, 4) && (!mask || aligned(mask, 4)) && aligned(pos_out, 8) &&
                 aligned(delta_out, 8) && aligned(status_out, 4) && aligned(workspace, 4) &&
                 (!image_thw || aligned(image_thw, 8)) && (!video_thw || aligned(video_thw, 8)),
             "q3_rope_index: misaligned pointer");
  cudaStream_t st = (cudaStream_t)stream;
  int* counts = (int*)workspace;
  Q3_CUDA_CHECK(cudaMemsetAsync(status_out, 0, (size_t)B * sizeof(int32_t), st));
  int rc = launch_ex(rope_runs_kernel, dim3(B), dim3(kThreads), 0, st, 1, types, mask, S, counts);
  if (rc != Q3_OK) return rc;
  IndexArgs a{types, mask, S, image_thw, n_image, video_thw, n_video, merge, counts,
              (int*)status_out, pos_out, delta_out, B};
  const size_t smem = (size_t)(n_video + 1) * sizeof(int);
  return launch_ex(rope_index_kernel, dim3(B), dim3(kThreads), smem, st, 1, a);
}
