// Page allocator of a paged KV cache (host side).
//
// The reference keeps one contiguous [B, Hkv, max_seq_len, D] cache per layer,
// allocated per request (init_kv_cache, model_fused.py:224-232).  Here the K/V
// storage of every layer is a pool of fixed-size pages, [num_pages, Hkv,
// page_tokens, D] per layer and per K/V, owned by the caller.  This allocator
// only hands out page indices: a sequence slot owns an ordered list of pages,
// and its block table row maps position p to page row[p / page_tokens],
// offset p % page_tokens.
//
// Capacity is bucketed: a slot grows to the smallest configured bucket that
// covers the requested tokens, so decode graphs captured per bucket keep a
// fixed table width.  With no buckets, capacity is rounded up to whole pages.
// Allocation is all-or-nothing and deterministic (a LIFO free list that
// starts in ascending page order), so tensor-parallel ranks that issue the
// same calls hold the same tables.  The allocator calls are host-only and
// thread-safe.
//
// q3_kv_pages_write is the device side of the KV write (model_fused.py:244-246
// for a paged cache): it copies the new K/V rows, as q3_qkv_norm_rope emits
// them densely, into their pages, one warp per 256-byte row.
#include <algorithm>
#include <mutex>
#include <new>
#include <vector>

#include "common.cuh"

namespace q3 {
namespace {

struct KvPages {
  int num_pages = 0, page_tokens = 0, max_seqs = 0, max_pages_per_seq = 0;
  std::vector<int64_t> buckets;          // ascending token capacities
  std::vector<int32_t> free_pages;       // stack; back() is handed out next
  std::vector<std::vector<int32_t>> seq; // pages owned by each slot, in position order
  mutable std::mutex mu;
};

int64_t capacity_for(const KvPages& p, int64_t tokens) {
  if (tokens <= 0) return 0;
  if (p.buckets.empty())
    return (tokens + p.page_tokens - 1) / p.page_tokens * p.page_tokens;
  for (int64_t b : p.buckets)
    if (b >= tokens) return b;
  return -1;
}

constexpr int kPageHd = 128;

// One warp per (b, kv head, s, K|V) row: 32 lanes x 8 bytes.  A position past
// the table or a page index outside the pool is recorded in the device error
// word and its row skipped (no write outside the pool).
__global__ void __launch_bounds__(256) kv_page_write_kernel(
    const __nv_bfloat16* __restrict__ k_src, const __nv_bfloat16* __restrict__ v_src,
    __nv_bfloat16* __restrict__ k_pages, __nv_bfloat16* __restrict__ v_pages,
    const int32_t* __restrict__ table, int64_t stride, int page_tokens, int num_pages, int B,
    int Hkv, int S, int64_t start_pos, const int32_t* __restrict__ pos_dev, int* err) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const int64_t job = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t rows = (int64_t)B * Hkv * S;
  if (job >= 2 * rows) return;
  const bool is_v = job >= rows;
  const int64_t r = is_v ? job - rows : job;  // (b * Hkv + h) * S + s
  const int s = (int)(r % S);
  const int64_t bh = r / S;
  const int h = (int)(bh % Hkv), b = (int)(bh / Hkv);
  const int64_t t = (pos_dev ? (int64_t)(*pos_dev) : start_pos) + s;
  const int64_t slot = t / page_tokens;
  const int pg = (t >= 0 && slot < stride) ? table[(int64_t)b * stride + slot] : -1;
  if (pg < 0 || pg >= num_pages) {
    if (lane == 0) report_timeout(err, 0x403);
    return;
  }
  const uint2* src = reinterpret_cast<const uint2*>((is_v ? v_src : k_src) + r * kPageHd);
  uint2* dst = reinterpret_cast<uint2*>((is_v ? v_pages : k_pages) +
                                        (((int64_t)pg * Hkv + h) * page_tokens + t % page_tokens) *
                                            kPageHd);
  dst[lane] = src[lane];
}

}  // namespace
}  // namespace q3

extern "C" int q3_kv_pages_write(const void* k_src, const void* v_src, void* k_pages,
                                 void* v_pages, int B, int Hkv, int S, int head_dim,
                                 const int32_t* block_table, int64_t table_stride,
                                 int page_tokens, int num_pages, int64_t start_pos,
                                 const int32_t* pos_dev, q3_stream_t stream) {
  using namespace q3;
  Q3_REQUIRE(k_src && v_src && k_pages && v_pages && block_table,
             "q3_kv_pages_write: null pointer");
  Q3_REQUIRE(head_dim == kPageHd, "q3_kv_pages_write: head_dim must be 128 (got %d)", head_dim);
  Q3_REQUIRE(B > 0 && Hkv > 0 && S > 0 && table_stride > 0 && page_tokens > 0 && num_pages > 0,
             "q3_kv_pages_write: bad shape");
  Q3_REQUIRE(pos_dev || (start_pos >= 0 && start_pos + S <= table_stride * page_tokens),
             "q3_kv_pages_write: positions %lld..%lld beyond the table width",
             (long long)start_pos, (long long)(start_pos + S - 1));
  Q3_REQUIRE(aligned(k_src, 8) && aligned(v_src, 8) && aligned(k_pages, 8) &&
                 aligned(v_pages, 8) && aligned(block_table, 4),
             "q3_kv_pages_write: misaligned pointer");
  const int64_t jobs = 2 * (int64_t)B * Hkv * S;
  return launch_ex(kv_page_write_kernel, dim3((unsigned)((jobs + 7) / 8)), dim3(256), 0,
                   (cudaStream_t)stream, 1, (const __nv_bfloat16*)k_src,
                   (const __nv_bfloat16*)v_src, (__nv_bfloat16*)k_pages,
                   (__nv_bfloat16*)v_pages, block_table, table_stride, page_tokens, num_pages, B,
                   Hkv, S, start_pos, pos_dev, device_error_word());
}

extern "C" int q3_kv_pages_create(int num_pages, int page_tokens, int max_seqs,
                                  int max_pages_per_seq, const int64_t* buckets, int n_buckets,
                                  void** pool_out) {
  using namespace q3;
  Q3_REQUIRE(pool_out, "q3_kv_pages_create: null pool_out");
  *pool_out = nullptr;
  Q3_REQUIRE(num_pages > 0 && max_seqs > 0 && max_pages_per_seq > 0,
             "q3_kv_pages_create: num_pages, max_seqs and max_pages_per_seq must be positive");
  Q3_REQUIRE(page_tokens > 0 && page_tokens % 64 == 0,
             "q3_kv_pages_create: page_tokens=%d must be a positive multiple of 64 (the "
             "attention tile)", page_tokens);
  Q3_REQUIRE(n_buckets >= 0 && (n_buckets == 0 || buckets),
             "q3_kv_pages_create: bucket list");
  for (int i = 0; i < n_buckets; ++i) {
    Q3_REQUIRE(buckets[i] > 0 && buckets[i] % page_tokens == 0,
               "q3_kv_pages_create: bucket %lld is not a positive multiple of page_tokens %d",
               (long long)buckets[i], page_tokens);
    Q3_REQUIRE(i == 0 || buckets[i] > buckets[i - 1],
               "q3_kv_pages_create: buckets must be strictly ascending");
    Q3_REQUIRE(buckets[i] / page_tokens <= max_pages_per_seq,
               "q3_kv_pages_create: bucket %lld needs more than max_pages_per_seq=%d pages",
               (long long)buckets[i], max_pages_per_seq);
  }
  KvPages* p = new (std::nothrow) KvPages();
  Q3_REQUIRE(p, "q3_kv_pages_create: out of host memory");
  p->num_pages = num_pages;
  p->page_tokens = page_tokens;
  p->max_seqs = max_seqs;
  p->max_pages_per_seq = max_pages_per_seq;
  p->buckets.assign(buckets, buckets + n_buckets);
  p->free_pages.resize(num_pages);
  for (int i = 0; i < num_pages; ++i) p->free_pages[i] = num_pages - 1 - i;
  p->seq.resize(max_seqs);
  *pool_out = p;
  return Q3_OK;
}

extern "C" int q3_kv_pages_destroy(void* pool) {
  delete static_cast<q3::KvPages*>(pool);
  return Q3_OK;
}

extern "C" int q3_kv_pages_reserve(void* pool, int slot, int64_t tokens, int64_t* capacity_out) {
  using namespace q3;
  Q3_REQUIRE(pool, "q3_kv_pages_reserve: null pool");
  KvPages& p = *static_cast<KvPages*>(pool);
  std::lock_guard<std::mutex> lock(p.mu);
  Q3_REQUIRE(slot >= 0 && slot < p.max_seqs, "q3_kv_pages_reserve: slot %d outside [0, %d)", slot,
             p.max_seqs);
  Q3_REQUIRE(tokens >= 0, "q3_kv_pages_reserve: negative token count");
  std::vector<int32_t>& own = p.seq[slot];
  const int64_t have = (int64_t)own.size() * p.page_tokens;
  if (tokens <= have) {
    if (capacity_out) *capacity_out = have;
    return Q3_OK;
  }
  const int64_t cap = capacity_for(p, tokens);
  Q3_REQUIRE(cap > 0, "q3_kv_pages_reserve: %lld tokens exceed the largest bucket %lld",
             (long long)tokens, (long long)(p.buckets.empty() ? 0 : p.buckets.back()));
  const int64_t need_pages = cap / p.page_tokens;
  Q3_REQUIRE(need_pages <= p.max_pages_per_seq,
             "q3_kv_pages_reserve: %lld tokens need %lld pages, more than max_pages_per_seq=%d",
             (long long)tokens, (long long)need_pages, p.max_pages_per_seq);
  const int64_t grow = need_pages - (int64_t)own.size();
  if (grow > (int64_t)p.free_pages.size())
    return fail(Q3_ERR_NO_MEMORY, "q3_kv_pages_reserve: slot %d needs %lld more pages, %zu free",
                slot, (long long)grow, p.free_pages.size());
  for (int64_t i = 0; i < grow; ++i) {
    own.push_back(p.free_pages.back());
    p.free_pages.pop_back();
  }
  if (capacity_out) *capacity_out = cap;
  return Q3_OK;
}

extern "C" int q3_kv_pages_release(void* pool, int slot) {
  using namespace q3;
  Q3_REQUIRE(pool, "q3_kv_pages_release: null pool");
  KvPages& p = *static_cast<KvPages*>(pool);
  std::lock_guard<std::mutex> lock(p.mu);
  Q3_REQUIRE(slot >= 0 && slot < p.max_seqs, "q3_kv_pages_release: slot %d outside [0, %d)", slot,
             p.max_seqs);
  std::vector<int32_t>& own = p.seq[slot];
  // pages go back so that the next reservation takes them in the same order
  for (auto it = own.rbegin(); it != own.rend(); ++it) p.free_pages.push_back(*it);
  own.clear();
  return Q3_OK;
}

extern "C" int q3_kv_pages_table(const void* pool, const int32_t* slots, int n, int width,
                                 int32_t* table_out) {
  using namespace q3;
  Q3_REQUIRE(pool && (n == 0 || (slots && table_out)), "q3_kv_pages_table: null pointer");
  Q3_REQUIRE(n >= 0 && width > 0, "q3_kv_pages_table: bad shape n=%d width=%d", n, width);
  const KvPages& p = *static_cast<const KvPages*>(pool);
  std::lock_guard<std::mutex> lock(p.mu);
  for (int i = 0; i < n; ++i) {
    const int s = slots[i];
    Q3_REQUIRE(s >= 0 && s < p.max_seqs, "q3_kv_pages_table: slot %d outside [0, %d)", s,
               p.max_seqs);
    const std::vector<int32_t>& own = p.seq[s];
    Q3_REQUIRE((int)own.size() <= width, "q3_kv_pages_table: slot %d holds %zu pages > width %d",
               s, own.size(), width);
    int32_t* row = table_out + (int64_t)i * width;
    std::copy(own.begin(), own.end(), row);
    std::fill(row + own.size(), row + width, -1);
  }
  return Q3_OK;
}

extern "C" int q3_kv_pages_stats(const void* pool, int slot, int64_t* free_pages,
                                 int64_t* slot_pages) {
  using namespace q3;
  Q3_REQUIRE(pool, "q3_kv_pages_stats: null pool");
  const KvPages& p = *static_cast<const KvPages*>(pool);
  std::lock_guard<std::mutex> lock(p.mu);
  if (free_pages) *free_pages = (int64_t)p.free_pages.size();
  if (slot_pages) {
    Q3_REQUIRE(slot >= 0 && slot < p.max_seqs, "q3_kv_pages_stats: slot %d outside [0, %d)",
               slot, p.max_seqs);
    *slot_pages = (int64_t)p.seq[slot].size();
  }
  return Q3_OK;
}
