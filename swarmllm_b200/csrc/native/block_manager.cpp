#include "block_manager.h"

#include <algorithm>

namespace swarm_native {

BlockManager::BlockManager(int num_pages, int page_size, bool enable_prefix_cache)
    : num_pages_(num_pages), page_size_(page_size), prefix_(enable_prefix_cache) {
  if (num_pages <= 0 || page_size <= 0) throw std::invalid_argument("bad block manager size");
  free_.reserve(num_pages);
  // Page 0 is handed out last so a zero-padded block table rarely aliases live data.
  for (int p = num_pages - 1; p >= 0; --p) free_.push_back(p);
  ref_.assign(num_pages, 0);
  page_hash_.assign(num_pages, 0);
}

int BlockManager::num_free() const { return (int)free_.size() + (int)lru_.size(); }

// 64-bit chained hash (splitmix64 finaliser over a multiply-xor fold).
uint64_t BlockManager::hash_page(uint64_t parent, const int32_t* toks, int n) {
  uint64_t h = parent ^ 0x9E3779B97F4A7C15ull;
  for (int i = 0; i < n; ++i) {
    h ^= (uint64_t)(uint32_t)toks[i] + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    h *= 0xBF58476D1CE4E5B9ull;
  }
  h ^= h >> 31;
  h *= 0x94D049BB133111EBull;
  h ^= h >> 29;
  return h ? h : 1;
}

int BlockManager::alloc_page() {
  if (!free_.empty()) {
    int p = free_.back();
    free_.pop_back();
    ref_[p] = 1;
    return p;
  }
  if (!lru_.empty()) {  // evict the oldest unreferenced cached page
    int p = lru_.front();
    lru_.pop_front();
    lru_pos_.erase(p);
    hash_to_page_.erase(page_hash_[p]);
    page_hash_[p] = 0;
    ref_[p] = 1;
    return p;
  }
  return -1;
}

void BlockManager::release_page(int p) {
  if (--ref_[p] > 0) return;
  if (page_hash_[p] != 0) {
    lru_.push_back(p);
    lru_pos_[p] = std::prev(lru_.end());
  } else {
    free_.push_back(p);
  }
}

std::vector<uint64_t> BlockManager::chain_hashes(const std::vector<int32_t>& tokens, int n_pages,
                                                 uint64_t salt) const {
  std::vector<uint64_t> out;
  n_pages = std::min(n_pages, (int)tokens.size() / page_size_);
  uint64_t h = salt;
  for (int i = 0; i < n_pages; ++i) {
    h = hash_page(h, tokens.data() + (size_t)i * page_size_, page_size_);
    out.push_back(h);
  }
  return out;
}

int BlockManager::add_sequence(int64_t seq_id, const std::vector<int32_t>& tokens,
                               uint64_t salt, int cap, bool exact) {
  if (seqs_.count(seq_id)) throw std::invalid_argument("sequence exists");
  Seq s;
  s.root = salt;
  s.last_hash = salt;
  int covered = 0;
  if (prefix_) {
    uint64_t h = salt;
    // Never map the whole prompt: the last token must be recomputed for logits.
    int full = ((int)tokens.size() - 1) / page_size_;
    if (cap >= 0) full = std::min(full, cap / page_size_);
    for (int i = 0; i < full; ++i) {
      uint64_t nh = hash_page(h, tokens.data() + (size_t)i * page_size_, page_size_);
      auto it = hash_to_page_.find(nh);
      if (it == hash_to_page_.end()) break;
      int p = it->second;
      if (ref_[p] == 0) {
        auto lp = lru_pos_.find(p);
        if (lp != lru_pos_.end()) {
          lru_.erase(lp->second);
          lru_pos_.erase(lp);
        }
      }
      ++ref_[p];
      s.pages.push_back(p);
      h = nh;
      covered += page_size_;
    }
    if (exact && cap >= 0 && covered != (cap / page_size_) * page_size_) {
      for (int p : s.pages) release_page(p);   // back to the LRU / free list
      s.pages.clear();
      h = salt;
      covered = 0;
    }
    s.hashed_pages = (int)s.pages.size();
    s.last_hash = h;
    s.tokens.assign(tokens.begin(), tokens.begin() + covered);
    s.len = covered;
  }
  prefix_hit_tokens_ += covered;
  seqs_.emplace(seq_id, std::move(s));
  return covered;
}

std::vector<int32_t> BlockManager::cached_prefix_pages(const std::vector<int32_t>& tokens,
                                                       uint64_t salt) const {
  std::vector<int32_t> out;
  if (!prefix_) return out;
  uint64_t h = salt;
  const int full = (int)tokens.size() / page_size_;
  for (int i = 0; i < full; ++i) {
    const uint64_t nh = hash_page(h, tokens.data() + (size_t)i * page_size_, page_size_);
    auto it = hash_to_page_.find(nh);
    if (it == hash_to_page_.end()) break;
    out.push_back(it->second);
    h = nh;
  }
  return out;
}

std::vector<int32_t> BlockManager::import_prefix_pages(const std::vector<int32_t>& tokens,
                                                       int n_pages, uint64_t salt) {
  std::vector<int32_t> out;
  if (!prefix_) return out;
  n_pages = std::min(n_pages, (int)tokens.size() / page_size_);
  uint64_t h = salt;
  for (int i = 0; i < n_pages; ++i) {
    const uint64_t nh = hash_page(h, tokens.data() + (size_t)i * page_size_, page_size_);
    h = nh;
    if (hash_to_page_.count(nh)) {  // already cached here: keep ours
      out.push_back(-1);
      continue;
    }
    const int p = alloc_page();
    if (p < 0) {  // no room: the rest of the chain is not importable
      out.push_back(-1);
      break;
    }
    page_hash_[p] = nh;
    hash_to_page_[nh] = p;
    release_page(p);  // ref 1 -> 0: cached and evictable
    out.push_back(p);
  }
  return out;
}

int BlockManager::seq_len(int64_t seq_id) const {
  auto it = seqs_.find(seq_id);
  if (it == seqs_.end()) throw std::out_of_range("no such sequence");
  return it->second.len;
}

bool BlockManager::can_append(const std::vector<int64_t>& seq_ids, int n) const {
  int need = 0;
  for (auto id : seq_ids) {
    const Seq& s = seqs_.at(id);
    const int have = (int)s.pages.size() * page_size_;
    const int want = s.len + n;
    if (want > have) need += (want - have + page_size_ - 1) / page_size_;
  }
  return need <= num_free();
}

std::vector<int32_t> BlockManager::append_slots(int64_t seq_id, int n) {
  Seq& s = seqs_.at(seq_id);
  const int have = (int)s.pages.size() * page_size_;
  const int want = s.len + n;
  const int extra = want > have ? (want - have + page_size_ - 1) / page_size_ : 0;
  if (extra > num_free()) return {};
  for (int i = 0; i < extra; ++i) s.pages.push_back(alloc_page());
  std::vector<int32_t> slots(n);
  for (int i = 0; i < n; ++i) {
    const int pos = s.len + i;
    slots[i] = s.pages[pos / page_size_] * page_size_ + pos % page_size_;
  }
  s.len = want;
  return slots;
}

void BlockManager::register_full_pages(Seq& s) {
  if (!prefix_) return;
  const int full = (int)s.tokens.size() / page_size_;
  while (s.hashed_pages < full) {
    const int i = s.hashed_pages;
    const uint64_t nh = hash_page(s.last_hash, s.tokens.data() + (size_t)i * page_size_, page_size_);
    const int p = s.pages[i];
    if (page_hash_[p] == 0 && !hash_to_page_.count(nh)) {
      page_hash_[p] = nh;
      hash_to_page_[nh] = p;
    }
    s.last_hash = nh;
    ++s.hashed_pages;
  }
}

void BlockManager::commit_tokens(int64_t seq_id, const std::vector<int32_t>& tokens) {
  Seq& s = seqs_.at(seq_id);
  s.tokens.insert(s.tokens.end(), tokens.begin(), tokens.end());
  if ((int)s.tokens.size() > s.len) s.tokens.resize(s.len);
  register_full_pages(s);
}

void BlockManager::truncate(int64_t seq_id, int new_len) {
  Seq& s = seqs_.at(seq_id);
  if (new_len >= s.len) return;
  s.len = std::max(0, new_len);
  const int keep_pages = (s.len + page_size_ - 1) / page_size_;
  while ((int)s.pages.size() > keep_pages) {
    release_page(s.pages.back());
    s.pages.pop_back();
  }
  if ((int)s.tokens.size() > s.len) s.tokens.resize(s.len);
  if (s.hashed_pages > s.len / page_size_) {
    // Recompute the hash chain up to the surviving full pages.
    s.hashed_pages = 0;
    s.last_hash = s.root;
    const int full = s.len / page_size_;
    for (int i = 0; i < full && i * page_size_ + page_size_ <= (int)s.tokens.size(); ++i) {
      s.last_hash = hash_page(s.last_hash, s.tokens.data() + (size_t)i * page_size_, page_size_);
      ++s.hashed_pages;
    }
  }
}

std::pair<int, int> BlockManager::fork(int64_t parent, int64_t child) {
  if (seqs_.count(child)) throw std::invalid_argument("child exists");
  Seq c = seqs_.at(parent);
  for (int p : c.pages) ++ref_[p];
  std::pair<int, int> cow{-1, -1};
  if (c.len % page_size_ != 0 && !c.pages.empty()) {
    // The partially filled last page is written by both; give the child its own copy.
    int src = c.pages.back();
    int dst = alloc_page();
    if (dst < 0) {
      for (int p : c.pages) release_page(p);
      throw std::runtime_error("out of KV pages in fork");
    }
    release_page(src);
    c.pages.back() = dst;
    cow = {src, dst};
  }
  seqs_.emplace(child, std::move(c));
  return cow;
}

void BlockManager::free_sequence(int64_t seq_id) {
  auto it = seqs_.find(seq_id);
  if (it == seqs_.end()) return;
  for (int p : it->second.pages) release_page(p);
  seqs_.erase(it);
}

const std::vector<int32_t>& BlockManager::pages(int64_t seq_id) const { return seqs_.at(seq_id).pages; }

void BlockManager::fill_block_table(const std::vector<int64_t>& seq_ids, int max_pages,
                                    int32_t* out) const {
  for (size_t r = 0; r < seq_ids.size(); ++r) {
    const auto& pg = seqs_.at(seq_ids[r]).pages;
    if ((int)pg.size() > max_pages) throw std::out_of_range("block table too narrow");
    int32_t* row = out + r * (size_t)max_pages;
    std::copy(pg.begin(), pg.end(), row);
    std::fill(row + pg.size(), row + max_pages, 0);
  }
}

}  // namespace swarm_native
