// Draft trees for tree speculative decoding.
//
// A tree is grown level by level from a drafter's top-k proposals: every
// frontier node offers its k best next tokens, and the `width` children with
// the highest cumulative log-probability survive (the reference grows and
// prunes the same way: DraftTree / GrownTree / worth_checking,
// src/inference/draft_tree.rs:92,617,866).  Node 0 is the root: the last
// committed token, whose KV is written during verification.  Each node gets
// an ancestor bitmask (self included) used as the attention visibility mask
// of its verification row, so at most 64 nodes.
//
// Verification walks from the root: the target model's token at the current
// node is accepted if some child carries it, and the walk continues there.
// The result is the accepted node path plus the bonus token drawn at the last
// accepted node (walk_verified_tree, src/inference/sampling.rs:496).
#pragma once
#include <cstdint>
#include <vector>

namespace pybind11 {
class module_;
}

namespace swarm_native {

struct TreeNode {
  int32_t token = 0;
  int32_t parent = -1;
  int32_t depth = 0;
  double logp = 0.0;  // cumulative
  uint64_t mask = 0;  // ancestors including self
};

class DraftTree {
 public:
  explicit DraftTree(int32_t root_token, int max_nodes = 64);
  int size() const { return (int)nodes_.size(); }
  const std::vector<TreeNode>& nodes() const { return nodes_; }
  std::vector<int32_t> frontier() const { return frontier_; }
  // Expand: for frontier node i (in frontier order) candidates cand_tok[i*k+j],
  // cand_logp[i*k+j].  Keeps the best `width` children (subject to the node
  // budget).  Returns the new frontier (node indices).
  std::vector<int32_t> expand(const std::vector<int32_t>& cand_tok,
                              const std::vector<float>& cand_logp, int k, int width);
  // target[i] = the target model's chosen token at node i.  Returns the
  // accepted path (node indices, root first) and the bonus token.
  std::pair<std::vector<int32_t>, int32_t> walk(const std::vector<int32_t>& target) const;
  std::vector<int32_t> tokens() const;
  std::vector<int32_t> depths() const;
  std::vector<int32_t> parents() const;
  std::vector<uint64_t> masks() const;

 private:
  int max_nodes_;
  std::vector<TreeNode> nodes_;
  std::vector<int32_t> frontier_;
};

void bind_tree(pybind11::module_& m);

}  // namespace swarm_native
