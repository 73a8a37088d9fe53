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
// same calls hold the same tables.  All calls are host-only and thread-safe.
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

}  // namespace
}  // namespace q3

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
