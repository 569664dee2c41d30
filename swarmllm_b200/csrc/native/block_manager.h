// Paged KV-cache block manager with reference-counted prefix sharing.
//
// The reference keeps one contiguous, 512-token-growing cache per request
// (src/inference/split/kv_cache.rs:57,529,588) and a separate BLAKE3-keyed
// prefix cache of KV snapshots (src/inference/split/prefix_cache.rs:59,190).
// Here both are one structure: KV lives in fixed 16-token pages; a sequence
// owns a block table (list of page ids); full pages are content-addressed by
// a chained 64-bit hash of (parent hash, page tokens), so a new request whose
// prompt starts with a cached prefix maps the same physical pages (refcount +1)
// instead of copying a snapshot.  Unreferenced cached pages stay resident and
// are evicted LRU when the free list runs dry.
#pragma once
#include <cstdint>
#include <list>
#include <stdexcept>
#include <unordered_map>
#include <vector>

namespace swarm_native {

class BlockManager {
 public:
  BlockManager(int num_pages, int page_size, bool enable_prefix_cache);

  int page_size() const { return page_size_; }
  int num_pages() const { return num_pages_; }
  int num_free() const;  // free + evictable cached pages

  // Create a sequence.  With prefix caching, the longest run of full cached
  // pages matching `tokens` is mapped; returns the number of tokens covered.
  // `salt` is the root of the sequence's hash chain: sequences whose KV
  // differs for the same tokens (another LoRA adapter) use another salt and
  // never share pages.  At most `cap` tokens are mapped (< 0: no cap); with
  // `exact`, a hit shorter than `cap` maps nothing (a sequence that can only
  // resume at one position: recurrent state saved there).
  int add_sequence(int64_t seq_id, const std::vector<int32_t>& tokens, uint64_t salt = 0,
                   int cap = -1, bool exact = false);
  // Chained hash of each leading full page of `tokens` (the prefix-cache keys).
  std::vector<uint64_t> chain_hashes(const std::vector<int32_t>& tokens, int n_pages,
                                     uint64_t salt = 0) const;
  bool has_sequence(int64_t seq_id) const { return seqs_.count(seq_id) != 0; }
  int seq_len(int64_t seq_id) const;
  // Reserve room for n more tokens; returns the slot ids (page*page_size+off),
  // or an empty vector if not enough pages (nothing is changed then).
  std::vector<int32_t> append_slots(int64_t seq_id, int n);
  // Can `n` more tokens be appended to these sequences (each) right now?
  bool can_append(const std::vector<int64_t>& seq_ids, int n) const;
  // Record the token ids that now occupy the sequence (for prefix hashing).
  void commit_tokens(int64_t seq_id, const std::vector<int32_t>& tokens);
  // Drop tokens beyond new_len (speculative rollback).  Pages past it are released.
  void truncate(int64_t seq_id, int new_len);
  // Copy-on-write fork: the child shares all pages; a shared partial last page is copied
  // lazily by the caller via the returned (src_page, dst_page) pair (-1,-1 if none).
  std::pair<int, int> fork(int64_t parent, int64_t child);
  void free_sequence(int64_t seq_id);
  const std::vector<int32_t>& pages(int64_t seq_id) const;
  // Row-major [n, max_pages] int32 table (padded with 0).
  void fill_block_table(const std::vector<int64_t>& seq_ids, int max_pages, int32_t* out) const;

  int64_t prefix_hits() const { return prefix_hit_tokens_; }
  // Prefix snapshots (export / import of cached KV pages, e.g. across nodes).
  // Pages of the longest cached chain of full pages of `tokens` (no
  // references are taken: copy them out before scheduling more work).
  std::vector<int32_t> cached_prefix_pages(const std::vector<int32_t>& tokens,
                                           uint64_t salt = 0) const;
  // Make the first n_pages full pages of `tokens` cached: for each page of
  // the chain not already cached, take a free (or evict an LRU) page and
  // register its hash; it is left unreferenced in the LRU, as if a finished
  // request had produced it.  Returns one entry per page: the page to fill
  // with the KV data, or -1 where the page was already cached (or no page
  // was available; the chain stops there).
  std::vector<int32_t> import_prefix_pages(const std::vector<int32_t>& tokens, int n_pages,
                                           uint64_t salt = 0);
  int num_cached_pages() const { return (int)hash_to_page_.size(); }

 private:
  struct Seq {
    std::vector<int32_t> pages;
    std::vector<int32_t> tokens;  // committed tokens (for hashing)
    int len = 0;                  // reserved tokens
    int hashed_pages = 0;         // leading full pages already registered
    uint64_t last_hash = 0;
    uint64_t root = 0;            // hash-chain root (salt)
  };
  int alloc_page();
  void release_page(int p);
  void register_full_pages(Seq& s);
  static uint64_t hash_page(uint64_t parent, const int32_t* toks, int n);

  int num_pages_, page_size_;
  bool prefix_;
  std::vector<int32_t> free_;
  std::vector<int32_t> ref_;
  std::vector<uint64_t> page_hash_;  // 0 = not cached
  std::unordered_map<uint64_t, int32_t> hash_to_page_;
  std::list<int32_t> lru_;  // cached pages with ref 0, front = oldest
  std::unordered_map<int32_t, std::list<int32_t>::iterator> lru_pos_;
  std::unordered_map<int64_t, Seq> seqs_;
  int64_t prefix_hit_tokens_ = 0;
};

}  // namespace swarm_native
