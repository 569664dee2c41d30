#include "scheduler.h"

#include <algorithm>
#include <stdexcept>

namespace swarm_native {

Scheduler::Scheduler(BlockManager* bm, int max_step_tokens, int max_running, int prefill_chunk)
    : bm_(bm),
      max_step_tokens_(max_step_tokens),
      max_running_(max_running),
      prefill_chunk_(prefill_chunk) {}

void Scheduler::add_request(int64_t id, const std::vector<int32_t>& prompt, int max_new,
                            int32_t eos, uint64_t cache_salt, int max_cover, bool cover_exact,
                            int split_at) {
  if (reqs_.count(id)) throw std::invalid_argument("duplicate request id");
  if (prompt.empty()) throw std::invalid_argument("empty prompt");
  Request r;
  r.id = id;
  r.prompt = prompt;
  r.max_new = max_new;
  r.eos = eos;
  r.cache_salt = cache_salt;
  r.max_cover = max_cover;
  r.cover_exact = cover_exact;
  r.split_at = split_at;
  r.arrival = clock_++;
  reqs_.emplace(id, std::move(r));
  waiting_.push_back(id);
}

bool Scheduler::abort(int64_t id) {
  auto it = reqs_.find(id);
  if (it == reqs_.end()) return false;
  it->second.finished = true;
  bm_->free_sequence(id);
  waiting_.erase(std::remove(waiting_.begin(), waiting_.end(), id), waiting_.end());
  running_.erase(std::remove(running_.begin(), running_.end(), id), running_.end());
  return true;
}

void Scheduler::preempt(int64_t id) {
  Request& r = reqs_.at(id);
  bm_->free_sequence(id);
  // Recompute later: the generated tokens become part of the prompt.
  r.prompt.insert(r.prompt.end(), r.output.begin(), r.output.end());
  r.max_new -= (int)r.output.size();
  r.output.clear();
  r.n_computed = 0;
  r.running = false;
  ++r.n_preempted;
  ++preemptions_;
  running_.erase(std::remove(running_.begin(), running_.end(), id), running_.end());
  waiting_.push_front(id);
}

StepPlan Scheduler::schedule() {
  StepPlan plan;
  int budget = max_step_tokens_;
  // A prefill chunk stops at the request's split position.
  auto clip = [&](const Request& r, int n) {
    return (r.split_at > r.n_computed && r.n_computed + n > r.split_at) ? r.split_at - r.n_computed : n;
  };
  auto emit = [&](int64_t id, int ntok, bool sample, bool decode) {
    Request& r = reqs_.at(id);
    std::vector<int32_t> slots = bm_->append_slots(id, ntok);
    if ((int)slots.size() != ntok) return false;
    const int b = (int)plan.seq_ids.size();
    plan.seq_ids.push_back(id);
    plan.seq_start.push_back((int)plan.tokens.size());
    plan.seq_ntok.push_back(ntok);
    plan.seq_sample.push_back(sample ? 1 : 0);
    for (int i = 0; i < ntok; ++i) {
      const int pos = r.n_computed + i;
      const int32_t tok = decode ? r.output.back()
                                 : (pos < (int)r.prompt.size() ? r.prompt[pos] : r.output[pos - r.prompt.size()]);
      plan.tokens.push_back(tok);
      plan.positions.push_back(pos);
      plan.slots.push_back(slots[i]);
      plan.row_seq.push_back(b);
    }
    if (decode) ++plan.n_decode; else plan.n_prefill_tokens += ntok;
    return true;
  };

  // 1) Decode tokens for running sequences that finished their prompt.
  std::vector<int64_t> decoders;
  for (int64_t id : running_) {
    const Request& r = reqs_.at(id);
    if (r.n_computed >= (int)r.prompt.size() && !r.output.empty()) decoders.push_back(id);
  }
  for (size_t i = 0; i < decoders.size(); ++i) {
    int64_t id = decoders[i];
    if (budget <= 0) break;
    while (!bm_->can_append({id}, 1)) {
      // Preempt the newest running sequence (possibly this one).
      int64_t victim = running_.back();
      preempt(victim);
      decoders.erase(std::remove(decoders.begin(), decoders.end(), victim), decoders.end());
      if (victim == id) { id = -1; --i; break; }
    }
    if (id < 0) continue;
    if (emit(id, 1, true, true)) --budget;
  }
  // 2) Continue chunked prefill of running sequences.
  for (int64_t id : std::vector<int64_t>(running_)) {
    if (budget <= 0) break;
    Request& r = reqs_.at(id);
    const int remaining = (int)r.prompt.size() - r.n_computed;
    if (remaining <= 0) continue;
    const int n = clip(r, std::min({remaining, budget, prefill_chunk_}));
    if (!bm_->can_append({id}, n)) continue;
    if (emit(id, n, n == remaining, false)) budget -= n;
  }
  // 3) Admit waiting requests.
  while (!waiting_.empty() && budget > 0 && (int)running_.size() < max_running_) {
    const int64_t id = waiting_.front();
    Request& r = reqs_.at(id);
    const int covered = bm_->add_sequence(id, r.prompt, r.cache_salt, r.max_cover, r.cover_exact);
    r.n_computed = covered;
    const int remaining = (int)r.prompt.size() - covered;
    const int n = clip(r, std::min({remaining, budget, prefill_chunk_}));
    if (!bm_->can_append({id}, n)) {
      bm_->free_sequence(id);
      r.n_computed = 0;
      break;
    }
    waiting_.pop_front();
    // A request re-admitted after preemption recomputes from the start when
    // its hit had to be exact (the saved state belongs to the first admission).
    if (r.cover_exact) r.max_cover = 0;
    r.running = true;
    running_.push_back(id);
    if (emit(id, n, n == remaining, false)) budget -= n;
  }
  return plan;
}

std::vector<int64_t> Scheduler::commit(const StepPlan& plan, const std::vector<int32_t>& sampled) {
  std::vector<int64_t> done;
  size_t si = 0;
  for (size_t b = 0; b < plan.seq_ids.size(); ++b) {
    const int64_t id = plan.seq_ids[b];
    auto it = reqs_.find(id);
    if (it == reqs_.end() || it->second.finished) {
      if (plan.seq_sample[b]) ++si;
      continue;
    }
    Request& r = it->second;
    // Tokens fed this step are now in the cache.
    std::vector<int32_t> fed(plan.tokens.begin() + plan.seq_start[b],
                             plan.tokens.begin() + plan.seq_start[b] + plan.seq_ntok[b]);
    r.n_computed += plan.seq_ntok[b];
    bm_->commit_tokens(id, fed);
    if (plan.seq_sample[b]) {
      if (si >= sampled.size()) throw std::out_of_range("missing sampled token");
      const int32_t tok = sampled[si++];
      r.output.push_back(tok);
      if ((int)r.output.size() >= r.max_new || (r.eos >= 0 && tok == r.eos)) {
        r.finished = true;
        r.running = false;
        running_.erase(std::remove(running_.begin(), running_.end(), id), running_.end());
        bm_->free_sequence(id);
        done.push_back(id);
      }
    }
  }
  return done;
}

void Scheduler::release(int64_t id) {
  auto it = reqs_.find(id);
  if (it != reqs_.end() && it->second.finished) reqs_.erase(it);
}

}  // namespace swarm_native
