// Batched PUCT search over the evaluator (include/marina_search.h).
#include <math.h>
#include <string.h>

#include <atomic>
#include <chrono>
#include <thread>
#include <vector>

#include "marina_search.h"

namespace {

constexpr int kMaxLegal = 224;

enum : uint8_t { kLeaf = 0, kPending = 1, kExpanded = 2, kTerminal = 3 };

struct Node {
  double value_sum = 0.0;  // from the side to move at this node
  float prior = 0.f;
  float explored = 0.f;  // prior mass of the children visited at least once
  float terminal_value = 0.f;
  uint32_t visits = 0;
  uint32_t virtual_visits = 0;
  uint32_t first = 0;
  uint16_t count = 0;
  uint8_t state = kLeaf;
  mrc_move mv{};
  float mean() const { return visits ? static_cast<float>(value_sum / visits) : 0.f; }
};

struct Search {
  mrc_position root{};
  std::vector<Node> nodes;
  mrs_summary sum{};
  uint64_t in_flight = 0;
  bool finished = false;
};

// Bare kings, or a single knight or bishop beside them: no mate is possible.
bool insufficient_material(const mrc_position& p) {
  int minors = 0;
  for (int s = 0; s < 64; ++s) {
    const int t = p.board[s] < 0 ? -p.board[s] : p.board[s];
    if (t == 0 || t == 6) continue;
    if (t == 2 || t == 3) {
      ++minors;
      continue;
    }
    return false;
  }
  return minors <= 1;
}

struct Worker {
  const mrs_params* params;
  uint64_t limit;
  mrs_eval_fn eval;
  void* ctx;
  std::vector<Search*> searches;

  // Per round: the positions sent to the network and, per leaf, its search and path.
  std::vector<uint8_t> boards;
  std::vector<int32_t> legal;
  std::vector<float> priors, wdl;
  struct Leaf {
    Search* s;
    uint32_t path_start, path_len;
    int32_t count;
    mrc_move moves[kMaxLegal];
  };
  std::vector<Leaf> leaves;
  std::vector<uint32_t> paths;
  struct Reserved {
    Search* s;
    uint32_t path_start, path_len;
  };
  std::vector<Reserved> reserved;
  std::vector<uint32_t> reserved_paths;

  static void backup(Search& s, const std::vector<uint32_t>& path, float value) {
    for (size_t i = path.size(); i-- > 0;) {
      Node& n = s.nodes[path[i]];
      if (n.visits == 0 && i > 0) s.nodes[path[i - 1]].explored += n.prior;
      n.visits += 1;
      n.value_sum += value;
      value = -value;
    }
    s.sum.nodes += 1;
  }

  // One descent from the root holding a virtual visit on the way; returns 1 when it placed a
  // leaf, 0 when it backed up a terminal, -1 on a collision.
  int descend(Search& s, std::vector<uint32_t>& path) {
    mrc_position pos = s.root;
    path.clear();
    uint32_t node = 0;
    path.push_back(0);
    for (;;) {
      Node& n = s.nodes[node];
      if (n.state == kPending) {
        reserve(s, path);
        s.sum.collisions += 1;
        return -1;
      }
      if (n.state == kTerminal) {
        backup(s, path, n.terminal_value);
        return 0;
      }
      if (n.state == kLeaf) {
        if (path.size() - 1 > s.sum.max_depth) s.sum.max_depth = path.size() - 1;
        Leaf leaf;
        leaf.count = mrc_legal_moves(&pos, leaf.moves);
        if (leaf.count == 0 || pos.halfmove >= 100 || insufficient_material(pos)) {
          n.state = kTerminal;
          n.terminal_value = (leaf.count == 0 && mrc_in_check(&pos)) ? -1.f : 0.f;
          backup(s, path, n.terminal_value);
          return 0;
        }
        n.state = kPending;
        reserve(s, path);
        leaf.s = &s;
        leaf.path_start = static_cast<uint32_t>(paths.size());
        leaf.path_len = static_cast<uint32_t>(path.size());
        paths.insert(paths.end(), path.begin(), path.end());
        const size_t at = leaves.size();
        boards.resize((at + 1) * 66);
        legal.resize((at + 1) * kMaxLegal);
        mrc_encode_board(&pos, boards.data() + at * 66);
        int32_t* slots = legal.data() + at * kMaxLegal;
        for (int i = 0; i < kMaxLegal; ++i) slots[i] = i < leaf.count ? mrc_encode_move(&pos, leaf.moves[i]) : -1;
        leaves.push_back(leaf);
        return 1;
      }
      // Expanded: PUCT selection (src/search/tree.rs:290-320).
      const float parent_n = static_cast<float>(n.visits + n.virtual_visits);
      const float scale = params->cpuct * sqrtf(parent_n > 1.f ? parent_n : 1.f);
      const float unvisited_q = n.mean() - params->fpu_reduction * sqrtf(n.explored);
      uint32_t best = n.first;
      float best_score = -INFINITY;
      for (uint32_t c = n.first; c < n.first + n.count; ++c) {
        const Node& ch = s.nodes[c];
        const float q = ch.visits > 0 ? -ch.mean() : unvisited_q;
        const float score = q + scale * ch.prior / (1.f + static_cast<float>(ch.visits + ch.virtual_visits));
        if (score > best_score) {
          best_score = score;
          best = c;
        }
      }
      mrc_play(&pos, s.nodes[best].mv);
      node = best;
      path.push_back(node);
    }
  }

  void reserve(Search& s, const std::vector<uint32_t>& path) {
    for (uint32_t i : path) s.nodes[i].virtual_visits += 1;
  }

  void release(Search& s, const uint32_t* path, uint32_t len) {
    for (uint32_t i = 0; i < len; ++i) s.nodes[path[i]].virtual_visits -= 1;
  }

  uint64_t want(const Search& s) const {
    const uint64_t batch = static_cast<uint64_t>(params->batch);
    if (params->batch_ramp <= 0) return batch;
    const Node& root = s.nodes[0];
    uint64_t w = (root.visits + root.virtual_visits) / static_cast<uint64_t>(params->batch_ramp);
    if (w < 8) w = 8;
    return w < batch ? w : batch;
  }

  // Gather one batch for `s` (src/search/mod.rs:972-1021).
  void gather(Search& s, std::vector<uint32_t>& path) {
    const uint64_t w = want(s);
    const uint64_t lost_limit = params->collision_budget_pct <= 0
                                    ? UINT64_MAX
                                    : w * static_cast<uint64_t>(params->collision_budget_pct) / 100;
    const uint64_t lost_before = s.sum.collisions;
    uint64_t placed = 0;
    while (placed < w && s.sum.nodes + placed < limit) {
      if (s.sum.collisions - lost_before > lost_limit) break;
      const size_t res_before = reserved.size();
      const int r = descend(s, path);
      if (r == 1) ++placed;
      if (r == -1) {
        // keep the collision's reservation until the batch is applied
        reserved.push_back({&s, static_cast<uint32_t>(reserved_paths.size()), static_cast<uint32_t>(path.size())});
        reserved_paths.insert(reserved_paths.end(), path.begin(), path.end());
      }
      (void)res_before;
    }
  }

  int run() {
    std::vector<uint32_t> path;
    path.reserve(256);
    for (;;) {
      boards.clear(), legal.clear(), leaves.clear(), paths.clear(), reserved.clear(), reserved_paths.clear();
      bool any = false;
      for (Search* s : searches) {
        if (s->finished) continue;
        if (s->sum.nodes >= limit) {
          s->finished = true;
          continue;
        }
        any = true;
        gather(*s, path);
      }
      if (!any) return 0;
      const int n = static_cast<int>(leaves.size());
      if (n > 0) {
        priors.resize(static_cast<size_t>(n) * kMaxLegal);
        wdl.resize(static_cast<size_t>(n) * 3);
        const int rc = eval(ctx, n, boards.data(), legal.data(), priors.data(), wdl.data());
        if (rc != 0) {
          for (Search* s : searches) s->sum.error = rc;
          return rc;
        }
      }
      // Expand and back up every leaf (src/search/mod.rs:1131-1155), then release.
      for (int i = 0; i < n; ++i) {
        Leaf& leaf = leaves[i];
        Search& s = *leaf.s;
        const uint32_t* lp = paths.data() + leaf.path_start;
        const uint32_t index = lp[leaf.path_len - 1];
        const uint32_t first = static_cast<uint32_t>(s.nodes.size());
        for (int c = 0; c < leaf.count; ++c) {
          Node ch;
          const float pr = priors[static_cast<size_t>(i) * kMaxLegal + c];
          ch.prior = pr > 0.f ? pr : 0.f;
          ch.mv = leaf.moves[c];
          s.nodes.push_back(ch);
        }
        Node& leaf_node = s.nodes[index];
        leaf_node.first = first;
        leaf_node.count = static_cast<uint16_t>(leaf.count);
        leaf_node.state = kExpanded;
        const float* w3 = wdl.data() + static_cast<size_t>(i) * 3;
        float value = w3[0] - w3[2];
        if (!isfinite(value)) value = 0.f;
        path.assign(lp, lp + leaf.path_len);
        backup(s, path, value);
        release(s, lp, leaf.path_len);
        s.sum.network_evals += 1;
      }
      for (const Reserved& r : reserved) release(*r.s, reserved_paths.data() + r.path_start, r.path_len);
      for (Search* s : searches)
        if (!s->finished) s->sum.batches += 1;
    }
  }
};

}  // namespace

namespace {

int search_all(const mrc_position* roots, int n_roots, uint64_t node_limit, const mrs_params* params, mrs_eval_fn eval,
               void* const* contexts, int n_evaluators, int workers_per_evaluator, mrs_summary* per_root,
               mrs_summary* total, int32_t* root_actions, uint32_t* root_visits) {
  if (!roots || n_roots <= 0 || !params || !eval || !contexts || n_evaluators <= 0 || workers_per_evaluator <= 0 ||
      params->batch <= 0 || params->batch > 4096)
    return -1;
  std::vector<Search> searches(n_roots);
  for (int i = 0; i < n_roots; ++i) {
    searches[i].root = roots[i];
    searches[i].nodes.reserve(node_limit < (1u << 20) ? 40 * node_limit : 1u << 22);
    searches[i].nodes.emplace_back();
  }
  const int n_workers = n_evaluators * workers_per_evaluator;
  std::vector<Worker> workers(n_workers);
  for (int w = 0; w < n_workers; ++w) {
    workers[w].params = params;
    workers[w].limit = node_limit;
    workers[w].eval = eval;
    workers[w].ctx = contexts[w / workers_per_evaluator];
  }
  for (int i = 0; i < n_roots; ++i) workers[i % n_workers].searches.push_back(&searches[i]);
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<int> rcs(n_workers, 0);
  std::vector<std::thread> threads;
  for (int w = 0; w < n_workers; ++w) threads.emplace_back([&, w] { rcs[w] = workers[w].run(); });
  for (auto& t : threads) t.join();
  const double seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  int rc = 0;
  for (int r : rcs)
    if (r && !rc) rc = r;
  mrs_summary tot{};
  for (int i = 0; i < n_roots; ++i) {
    Search& s = searches[i];
    s.sum.seconds = seconds;
    s.sum.tree_nodes = s.nodes.size();
    const Node& root = s.nodes[0];
    uint32_t best = 0;
    int32_t best_action = -1;
    for (uint32_t c = root.first; c < root.first + root.count; ++c)
      if (s.nodes[c].visits > best) {
        best = s.nodes[c].visits;
        best_action = mrc_encode_move(&s.root, s.nodes[c].mv);
      }
    s.sum.best_action = best_action;
    if (root_actions && root_visits) {
      int32_t* acts = root_actions + static_cast<size_t>(i) * kMaxLegal;
      uint32_t* vis = root_visits + static_cast<size_t>(i) * kMaxLegal;
      for (int k = 0; k < kMaxLegal; ++k) acts[k] = -1, vis[k] = 0;
      for (uint32_t c = 0; c < root.count && c < static_cast<uint32_t>(kMaxLegal); ++c) {
        acts[c] = mrc_encode_move(&s.root, s.nodes[root.first + c].mv);
        vis[c] = s.nodes[root.first + c].visits;
      }
    }
    if (per_root) per_root[i] = s.sum;
    tot.nodes += s.sum.nodes;
    tot.network_evals += s.sum.network_evals;
    tot.batches += s.sum.batches;
    tot.collisions += s.sum.collisions;
    tot.tree_nodes += s.sum.tree_nodes;
    if (s.sum.max_depth > tot.max_depth) tot.max_depth = s.sum.max_depth;
  }
  tot.seconds = seconds;
  tot.error = rc;
  tot.best_action = -1;
  if (total) *total = tot;
  return rc;
}

}  // namespace

extern "C" MRC_API int mrs_search(const mrc_position* roots, int n_roots, uint64_t node_limit, const mrs_params* params,
                                  mrs_eval_fn eval, void* const* contexts, int n_evaluators, int workers_per_evaluator,
                                  mrs_summary* per_root, mrs_summary* total) {
  return search_all(roots, n_roots, node_limit, params, eval, contexts, n_evaluators, workers_per_evaluator, per_root,
                    total, nullptr, nullptr);
}

extern "C" MRC_API int mrs_search_visits(const mrc_position* roots, int n_roots, uint64_t node_limit,
                                         const mrs_params* params, mrs_eval_fn eval, void* const* contexts,
                                         int n_evaluators, int workers_per_evaluator, mrs_summary* per_root,
                                         mrs_summary* total, int32_t* root_actions, uint32_t* root_visits) {
  if (!root_actions || !root_visits) return -1;
  return search_all(roots, n_roots, node_limit, params, eval, contexts, n_evaluators, workers_per_evaluator, per_root,
                    total, root_actions, root_visits);
}
