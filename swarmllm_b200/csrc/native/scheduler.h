// Continuous-batching scheduler with chunked prefill.
//
// Each engine step runs ONE forward over a mixed batch: one token for every
// decoding sequence (decode first, so running requests never stall) plus
// prompt chunks for sequences still prefilling, up to a per-step token budget
// (Sarathi-style).  New requests are admitted FIFO while KV pages and the
// running-sequence cap allow.  When the KV pool runs dry the newest running
// sequence is preempted: its pages are freed and it is re-queued to recompute
// (prompt + generated so far) later.
//
// Mirrors the reference's worker slot table and tick
// (src/inference/slot_table.rs:28-270, Slot::take_prefill_chunk at :207;
// src/inference/model_worker.rs:11934 step_decode_pool), re-designed around a
// paged KV pool instead of per-request contiguous caches.
#pragma once
#include <cstdint>
#include <deque>
#include <unordered_map>
#include <vector>

#include "block_manager.h"

namespace swarm_native {

struct Request {
  int64_t id = 0;
  std::vector<int32_t> prompt;   // prompt (grows with generated tokens on preemption)
  std::vector<int32_t> output;   // generated tokens
  int max_new = 16;
  int32_t eos = -1;
  int n_computed = 0;            // tokens whose KV is in the cache
  bool running = false;
  bool finished = false;
  int64_t arrival = 0;
  int n_preempted = 0;
  uint64_t cache_salt = 0;       // prefix-cache namespace (0: base model)
  int max_cover = -1;            // prefix-cache hit cap at first admission (< 0: none)
  bool cover_exact = false;      // hit exactly max_cover tokens or none
  int split_at = -1;             // a prefill chunk ends at this position (state snapshot)
};

struct StepPlan {
  std::vector<int64_t> seq_ids;       // [B] sequences in this step (batch order)
  std::vector<int32_t> seq_start;     // [B] first token row of each sequence
  std::vector<int32_t> seq_ntok;      // [B] tokens of each sequence in this step
  std::vector<int32_t> seq_sample;    // [B] 1 if the last row's logits are sampled
  std::vector<int32_t> tokens;        // [N] token ids
  std::vector<int32_t> positions;     // [N]
  std::vector<int32_t> slots;         // [N] KV slot ids
  std::vector<int32_t> row_seq;       // [N] batch index of each row
  int n_decode = 0;                   // sequences in pure decode
  int n_prefill_tokens = 0;
};

class Scheduler {
 public:
  Scheduler(BlockManager* bm, int max_step_tokens, int max_running, int prefill_chunk);
  void add_request(int64_t id, const std::vector<int32_t>& prompt, int max_new, int32_t eos,
                   uint64_t cache_salt = 0, int max_cover = -1, bool cover_exact = false,
                   int split_at = -1);
  bool abort(int64_t id);
  StepPlan schedule();
  // Feed back the sampled token of each sequence with seq_sample == 1 (in batch
  // order).  Returns ids of requests that finished in this step.
  std::vector<int64_t> commit(const StepPlan& plan, const std::vector<int32_t>& sampled);
  const Request& request(int64_t id) const { return reqs_.at(id); }
  void release(int64_t id);  // forget a finished request
  int num_waiting() const { return (int)waiting_.size(); }
  int num_running() const { return (int)running_.size(); }
  bool has_work() const { return !waiting_.empty() || !running_.empty(); }
  int64_t num_preemptions() const { return preemptions_; }

 private:
  void preempt(int64_t id);
  BlockManager* bm_;
  int max_step_tokens_, max_running_, prefill_chunk_;
  std::unordered_map<int64_t, Request> reqs_;
  std::deque<int64_t> waiting_;
  std::vector<int64_t> running_;  // admission order
  int64_t clock_ = 0, preemptions_ = 0;
};

}  // namespace swarm_native
