// Host-side tree scheduler behind ta_schedule_tree: the greedy and subset-DP
// ("cube") recursions of the reference (schedule.py:96-143) over a radix
// tree, with the roofline cost model (schedule.py:41-52).
//
// The Python statement is _Planner in tree_attention/schedule.py; this file
// follows it operation for operation so that every cost is the same double and
// every tie breaks the same way, and tests hold the plans identical:
//  * job costs: integer byte/FLOP counts divided in the reference's order;
//  * sums over lists of costs use Neumaier's compensated summation (Neumaier,
//    "Rundungsfehleranalyse einiger Verfahren zur Summation endlicher Summen",
//    ZAMM 54, 1974), the algorithm CPython 3.12's built-in sum() applies to
//    floats, including its final correction step;
//  * the DP's states keep first-insertion order and a state is replaced only
//    by a strictly smaller subtotal; the final minimum is over (total, pushed
//    children as a tuple), the tuple compared lexicographically.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <map>
#include <unordered_map>
#include <utility>
#include <vector>

#include "tree_attn.h"

namespace {

using Run = std::pair<int64_t, int64_t>;   // (first position, length)
using Runs = std::vector<Run>;

struct RunsHash {
  size_t operator()(const Runs& r) const {
    uint64_t h = 1469598103934665603ull;
    for (const auto& [s, l] : r) {
      h = (h ^ uint64_t(s)) * 1099511628211ull;
      h = (h ^ uint64_t(l)) * 1099511628211ull;
    }
    return size_t(h);
  }
};

// Neumaier summation, finished the way CPython's sum() finishes it.
struct CompensatedSum {
  double total = 0.0, c = 0.0;
  void add(double x) {
    const double t = total + x;
    if (std::fabs(total) >= std::fabs(x))
      c += (total - t) + x;
    else
      c += (x - t) + total;
    total = t;
  }
  double value() const { return (c != 0.0 && std::isfinite(c)) ? total + c : total; }
};

Runs concat(const Runs& a, const Runs& b) {
  if (a.empty()) return b;
  if (b.empty()) return a;
  Runs out = a;
  if (b.front().first == out.back().first + out.back().second) {
    out.back().second += b.front().second;
    out.insert(out.end(), b.begin() + 1, b.end());
  } else {
    out.insert(out.end(), b.begin(), b.end());
  }
  return out;
}

// A pushed-children chain: (last child, index of the earlier chain), -1 = empty.
struct ChainNode {
  int child, prev;
};

class Planner {
 public:
  Planner(const int32_t* child_offsets, const int32_t* children, const int32_t* node_requests,
          std::vector<Runs> node_runs, const ta_cost_model& m, int qheads, int kvheads, int dim)
      : child_offsets_(child_offsets), children_(children), size_(node_requests), runs_(std::move(node_runs)),
        m_(m), qheads_(qheads), kvheads_(kvheads), dim_(dim) {
    req_tile_ = std::max(1, m.max_query_rows / (qheads / kvheads));
  }

  // solve(method, node, inherited): (cost, pushed children chain)
  std::pair<double, int> solve(bool cube, int node, const Runs& inherited) {
    auto& memo = solve_memo_[node];
    auto hit = memo.find(inherited);
    if (hit != memo.end()) return hit->second;
    const Runs runs = concat(inherited, runs_[node]);
    std::pair<double, int> result;
    if (child_offsets_[node] == child_offsets_[node + 1])
      result = {count_cost(size_[node], runs), -1};
    else if (!cube)
      result = solve_greedy(node, runs);
    else
      result = solve_subsets(node, runs);
    memo.emplace(inherited, result);
    return result;
  }

  std::vector<int> chain_children(int chain) const {
    std::vector<int> out;
    for (; chain >= 0; chain = chains_[chain].prev) out.push_back(chains_[chain].child);
    std::reverse(out.begin(), out.end());
    return out;
  }

  const Runs& node_runs(int node) const { return runs_[node]; }
  int first_child(int node) const { return child_offsets_[node]; }
  int last_child(int node) const { return child_offsets_[node + 1]; }
  int child(int i) const { return children_[i]; }

 private:
  double piece_cost(int64_t nreq, int64_t ntok) {
    const auto key = std::make_pair(nreq, ntok);
    auto it = piece_memo_.find(key);
    if (it != piece_memo_.end()) return it->second;
    double value = 0.0;
    if (nreq > 0 && ntok > 0) {
      const int64_t groups = qheads_ / kvheads_;
      const int64_t rows = nreq * groups;
      const bool small = rows <= m_.cube_rows;
      const int64_t row_tile = small ? m_.cube_rows : m_.max_query_rows;
      const int64_t col_tile = small ? m_.key_tile : m_.key_tile / 2;
      const int64_t qtiles = (rows + row_tile - 1) / row_tile;
      const int64_t ktiles = (ntok + col_tile - 1) / col_tile;
      const int64_t flops = 4 * qtiles * row_tile * ktiles * col_tile * dim_ * kvheads_;
      const int64_t reads = 4 * ntok * dim_ * kvheads_ * qtiles;
      const int64_t partial = 4 * nreq * qheads_ * (dim_ + 1);
      const double compute = double(flops) / m_.cube_flops, memory = double(reads) / m_.bandwidth;
      value = (memory > compute ? memory : compute) + m_.task_us * double(qtiles) * double(kvheads_) +
              double(partial) / m_.bandwidth + m_.merge_us * double(nreq);
    }
    piece_memo_.emplace(key, value);
    return value;
  }

  // Lengths of the physical jobs of every kv_split chunk of `runs`: a chunk
  // stays whole when last - first + 1 == its length, else it is cut into runs.
  const std::vector<int64_t>& chunk_pieces(const Runs& runs) {
    auto it = pieces_memo_.find(runs);
    if (it != pieces_memo_.end()) return it->second;
    std::vector<std::vector<Run>> chunks;
    std::vector<Run> current;
    int64_t used = 0;
    for (auto [start, length] : runs) {
      while (length) {
        const int64_t take = std::min<int64_t>(length, m_.kv_split - used);
        current.push_back({start, take});
        start += take;
        used += take;
        length -= take;
        if (used == m_.kv_split) {
          chunks.push_back(std::move(current));
          current.clear();
          used = 0;
        }
      }
    }
    if (!current.empty()) chunks.push_back(std::move(current));
    std::vector<int64_t> pieces;
    for (const auto& chunk : chunks) {
      int64_t total = 0;
      for (const auto& r : chunk) total += r.second;
      const int64_t first = chunk.front().first, last = chunk.back().first + chunk.back().second - 1;
      if (last - first + 1 == total)
        pieces.push_back(total);
      else
        for (const auto& r : chunk) pieces.push_back(r.second);
    }
    return pieces_memo_.emplace(runs, std::move(pieces)).first->second;
  }

  double count_cost(int64_t count, const Runs& runs) {
    auto& memo = count_memo_[runs];
    auto it = memo.find(count);
    if (it != memo.end()) return it->second;
    const std::vector<int64_t>& pieces = chunk_pieces(runs);
    CompensatedSum sum;
    for (int64_t q = 0; q < count; q += req_tile_) {
      const int64_t nreq = std::min<int64_t>(req_tile_, count - q);
      for (int64_t take : pieces) sum.add(piece_cost(nreq, take));
    }
    const double value = sum.value();
    memo.emplace(count, value);
    return value;
  }

  std::pair<double, int> solve_greedy(int node, const Runs& runs) {
    int64_t remaining = size_[node];
    std::vector<char> pushed(child_offsets_[node + 1] - child_offsets_[node], 0);
    int chain = -1;
    for (int i = child_offsets_[node]; i < child_offsets_[node + 1]; ++i) {
      const int c = children_[i];
      const int64_t count = size_[c];
      const Runs& child_runs = runs_[c];
      const double keep_apart = count_cost(remaining, runs) + count_cost(count, child_runs);
      const double push_down = count_cost(remaining - count, runs) + count_cost(count, concat(runs, child_runs));
      if (push_down < keep_apart) {
        pushed[i - child_offsets_[node]] = 1;
        chains_.push_back({c, chain});
        chain = int(chains_.size()) - 1;
        remaining -= count;
      }
    }
    double total = count_cost(remaining, runs);
    CompensatedSum sum;
    static const Runs kNone;
    for (int i = child_offsets_[node]; i < child_offsets_[node + 1]; ++i)
      sum.add(solve(false, children_[i], pushed[i - child_offsets_[node]] ? runs : kNone).first);
    total += sum.value();
    return {total, chain};
  }

  std::pair<double, int> solve_subsets(int node, const Runs& runs) {
    // states in first-insertion order: removed count -> (subtotal, chain)
    struct State {
      int64_t removed;
      double subtotal;
      int chain;
    };
    std::vector<State> states{{0, 0.0, -1}}, updated;
    std::vector<int> where(size_t(size_[node]) + 1, -1);   // removed -> index in `updated`
    static const Runs kNone;
    for (int i = child_offsets_[node]; i < child_offsets_[node + 1]; ++i) {
      const int c = children_[i];
      const int64_t count = size_[c];
      const double apart = solve(true, c, kNone).first;
      const double together = solve(true, c, runs).first;
      updated.clear();
      auto offer = [&](int64_t slot, double value, int chain) {
        if (slot >= int64_t(where.size())) where.resize(size_t(slot) + 1, -1);
        const int at = where[slot];
        if (at < 0) {
          where[slot] = int(updated.size());
          updated.push_back({slot, value, chain});
        } else if (value < updated[at].subtotal) {
          updated[at].subtotal = value;
          updated[at].chain = chain;
        }
      };
      for (const State& s : states) {
        offer(s.removed, s.subtotal + apart, s.chain);
        chains_.push_back({c, s.chain});
        offer(s.removed + count, s.subtotal + together, int(chains_.size()) - 1);
      }
      for (const State& s : updated) where[s.removed] = -1;
      std::swap(states, updated);
    }
    const int64_t size = size_[node];
    // min over (total, pushed tuple): the tuples are compared only among the
    // states whose totals tie with the smallest
    double best = 0.0;
    bool first = true;
    std::vector<double> totals(states.size());
    for (size_t k = 0; k < states.size(); ++k) {
      totals[k] = states[k].subtotal + count_cost(size - states[k].removed, runs);
      if (first || totals[k] < best) {
        best = totals[k];
        first = false;
      }
    }
    int chosen = -1;
    std::vector<int> chosen_tuple;
    for (size_t k = 0; k < states.size(); ++k) {
      if (!(totals[k] == best)) continue;
      std::vector<int> tuple = chain_children(states[k].chain);
      if (chosen < 0 || tuple < chosen_tuple) {
        chosen = int(k);
        chosen_tuple = std::move(tuple);
      }
    }
    return {best, states[chosen].chain};
  }

  const int32_t* child_offsets_;
  const int32_t* children_;
  const int32_t* size_;
  std::vector<Runs> runs_;
  ta_cost_model m_;
  int64_t qheads_, kvheads_, dim_;
  int req_tile_;
  std::vector<ChainNode> chains_;
  std::map<std::pair<int64_t, int64_t>, double> piece_memo_;
  std::unordered_map<Runs, std::vector<int64_t>, RunsHash> pieces_memo_;
  std::unordered_map<Runs, std::unordered_map<int64_t, double>, RunsHash> count_memo_;
  std::unordered_map<int, std::map<Runs, std::pair<double, int>>> solve_memo_;
};

}  // namespace

extern "C" int ta_schedule_tree(const int32_t* child_offsets, const int32_t* children, const int32_t* node_requests,
                                const int32_t* run_offsets, const int64_t* runs, int32_t num_nodes, int32_t method,
                                const ta_cost_model* model, int32_t num_q_heads, int32_t num_kv_heads,
                                int32_t head_dim, uint8_t* pushed, double* root_cost) {
  if (!child_offsets || !children || !node_requests || !run_offsets || !runs || !model || !pushed) return TA_ERR_ARG;
  if (num_nodes <= 0 || (method != TA_SCHEDULE_GREEDY && method != TA_SCHEDULE_CUBE)) return TA_ERR_ARG;
  if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || head_dim <= 0) return TA_ERR_ARG;
  if (model->cube_rows <= 0 || model->key_tile < 2 || model->kv_split <= 0 || model->max_query_rows <= 0)
    return TA_ERR_ARG;
  // every node but the root is the child of exactly one earlier node.  The
  // recursion follows the tree's depth on the caller's stack, so the depth is
  // bounded (the Python statement stops at its recursion limit, about 500
  // levels, far earlier)
  constexpr int kMaxDepth = 2000;
  std::vector<char> seen(num_nodes, 0);
  std::vector<int> depth(num_nodes, 0);
  for (int n = 0; n < num_nodes; ++n) {
    if (child_offsets[n + 1] < child_offsets[n] || run_offsets[n + 1] < run_offsets[n] || node_requests[n] < 0)
      return TA_ERR_ARG;
    for (int i = child_offsets[n]; i < child_offsets[n + 1]; ++i) {
      const int c = children[i];
      if (c <= n || c >= num_nodes || seen[c]) return TA_ERR_ARG;
      seen[c] = 1;
      depth[c] = depth[n] + 1;
      if (depth[c] > kMaxDepth) return TA_ERR_UNSUPPORTED;
    }
  }
  std::vector<Runs> node_runs(num_nodes);
  for (int n = 0; n < num_nodes; ++n)
    for (int r = run_offsets[n]; r < run_offsets[n + 1]; ++r) {
      if (runs[2 * r + 1] <= 0) return TA_ERR_ARG;
      node_runs[n].push_back({runs[2 * r], runs[2 * r + 1]});
    }
  Planner planner(child_offsets, children, node_requests, std::move(node_runs), *model, num_q_heads, num_kv_heads,
                  head_dim);
  const bool cube = method == TA_SCHEDULE_CUBE;
  std::fill(pushed, pushed + num_nodes, uint8_t(0));
  // the materialisation walk: each node once, with the runs it inherits
  std::vector<std::pair<int, Runs>> stack{{0, Runs{}}};
  bool root = true;
  while (!stack.empty()) {
    auto [node, inherited] = std::move(stack.back());
    stack.pop_back();
    const auto [cost, chain] = planner.solve(cube, node, inherited);
    if (root && root_cost) *root_cost = cost;
    root = false;
    const std::vector<int> moved = planner.chain_children(chain);
    const Runs runs = concat(inherited, planner.node_runs(node));
    for (int i = planner.first_child(node); i < planner.last_child(node); ++i) {
      const int c = planner.child(i);
      const bool down = std::find(moved.begin(), moved.end(), c) != moved.end();
      pushed[c] = down ? 1 : 0;
      stack.push_back({c, down ? runs : Runs{}});
    }
  }
  return TA_OK;
}
