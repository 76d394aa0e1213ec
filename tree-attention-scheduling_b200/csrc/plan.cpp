// Host-side plan builder behind ta_plan_build: the int32 metadata of a
// physical job list (the reference's prepare arrays, kernels.py:103-141, and
// this implementation's pieces and kernel task lists).
//
// The Python statement of the same construction is build_metadata() in
// tree_attention/kernels.py; this file follows it step by step and tests hold
// the two bit-identical.  Every choice that breaks a tie (the piece split, the
// best-fit packing of short segments, the LPT assignment to persistent CTAs)
// is made in the same order as there, so the device sees the same buffer.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <functional>
#include <queue>
#include <utility>
#include <vector>

#include "tree_attn.h"

namespace {

// Routing and tiling constants (tree_attention/kernels.py).
constexpr int kKnRows = 16;         // jobs of at most this many query rows: keys-in-lanes kernel
constexpr int kTcRows = 256;        // query-tile kernel: pairs of 128-row tiles
constexpr int kSmallRows = 16;      // SIMT kernel row tile
constexpr int kKeyTile = 128;
constexpr int kKnDualRows = 8;      // classes up to this many rows run two CTAs per SM
constexpr int kKnDualCtas = 2;
constexpr int kKnTaskRows = 8;      // query rows of one keys-in-lanes segment
constexpr int kKnClassRows[5] = {4, 8, 16, 32, 64};
constexpr int kKnBox = 32;          // packed segments start on 32-key boundaries
constexpr int kKnPackRows = 8;      // query rows of a packed tile
constexpr int kKnPackSegs = 4;      // segments of a packed tile
constexpr int kGrowingBit = 30;

enum Route { kSimt, kKn, kTc };

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int tiles_of(int keys) { return std::max(1, int(cdiv(keys, kKeyTile))); }
inline int small_class(int rows) { return rows <= 4 ? 0 : (rows <= 8 ? 1 : 2); }
inline int kn_class(int rows) {
  for (int c = 0; c < 5; ++c)
    if (rows <= kKnClassRows[c]) return c;
  return -1;
}

struct PieceRec {
  int job, offset, take;
};

// One keys-in-lanes segment before packing: (head, rows, first partial row,
// first pool position, keys, job | growing << 30, first request, request offset).
struct Item {
  int32_t v[8];
  int rows() const { return v[1]; }
  int keys() const { return v[4]; }
};

// Execution pieces: kn jobs cut so no piece holds more than about half a CTA's
// share of all key tiles; query-tile jobs cut a whole level of the longest
// pieces at a time while their CTAs fit one wave.
// tc_max_ctas (<= 0: none) caps the query-tile CTAs below sms; levels, if
// given, receives (query-tile CTAs, longest piece in tiles) of every level.
void split_pieces(int njobs, const std::vector<int>& rows, const std::vector<int>& route,
                  const int32_t* keys, const std::vector<char>& splittable, int heads, int sms,
                  std::vector<PieceRec>& pieces, int64_t tc_max_ctas = 0,
                  std::vector<std::pair<int64_t, int64_t>>* levels = nullptr) {
  std::vector<int> count(njobs, 1);
  int64_t total = 0;
  bool any_kn = false;
  for (int i = 0; i < njobs; ++i)
    if (route[i] == kKn) {
      total += tiles_of(keys[i]);
      any_kn = true;
    }
  if (any_kn) {
    total *= heads;
    const int64_t cap = std::max<int64_t>(2, cdiv(total, 2 * int64_t(sms)));
    for (int i = 0; i < njobs; ++i)
      if (route[i] == kKn && splittable[i] && tiles_of(keys[i]) > cap) count[i] = int(cdiv(tiles_of(keys[i]), cap));
  }
  std::vector<int64_t> pairs(njobs, 0);
  int64_t ctas = 0;
  bool any_tc = false;
  for (int i = 0; i < njobs; ++i)
    if (route[i] == kTc) {
      pairs[i] = cdiv(rows[i], kTcRows) * heads;
      ctas += pairs[i];
      any_tc = true;
    }
  const int64_t limit = tc_max_ctas > 0 ? std::min<int64_t>(sms, tc_max_ctas) : int64_t(sms);
  while (any_tc) {
    // one level: every query-tile job whose pieces are the longest takes one
    // more piece, if all of them can and the CTAs still fit one wave
    int64_t longest = 0;
    for (int i = 0; i < njobs; ++i)
      if (route[i] == kTc) longest = std::max(longest, cdiv(tiles_of(keys[i]), count[i]));
    if (levels) levels->push_back({ctas, longest});
    bool ok = true;
    int64_t extra = 0;
    for (int i = 0; i < njobs && ok; ++i) {
      if (route[i] != kTc || cdiv(tiles_of(keys[i]), count[i]) != longest) continue;
      ok = splittable[i] && double(tiles_of(keys[i])) / double(count[i] + 1) >= 2.0;
      extra += pairs[i];
    }
    if (!ok || ctas + extra > limit) break;
    for (int i = 0; i < njobs; ++i)
      if (route[i] == kTc && cdiv(tiles_of(keys[i]), count[i]) == longest) count[i] += 1;
    ctas += extra;
  }
  for (int i = 0; i < njobs; ++i) {
    const int per = int(cdiv(tiles_of(keys[i]), count[i])) * kKeyTile;
    int offset = 0;
    while (true) {
      const int take = std::min(per, keys[i] - offset);
      pieces.push_back({i, offset, take});
      offset += take;
      if (offset >= keys[i]) break;
    }
  }
}

// Short segments packed best fit (by 32-key-rounded span) into 128-key tiles
// of at most kKnPackSegs segments and kKnPackRows rows; longer ones, and
// segments of more than half a packed tile's rows, are tasks of their own.
std::vector<std::vector<int>> pack_segments(const std::vector<Item>& items) {
  std::vector<std::vector<int>> tasks;
  struct Bin {
    std::vector<int> segs;
    int used_rows;
  };
  std::vector<Bin> open[4];            // indexed by remaining span / 32 (1..3), kept in insertion order
  std::vector<size_t> head(4, 0);      // first live bin of each list (bins leave from the front)
  std::vector<std::pair<int, int>> packable;   // (span, item)
  for (int i = 0; i < int(items.size()); ++i) {
    const int keys = items[i].keys();
    const int span = int(cdiv(keys, kKnBox)) * kKnBox;
    if (keys > kKeyTile || span >= kKeyTile || items[i].rows() > kKnPackRows / 2)
      tasks.push_back({i});
    else
      packable.push_back({span, i});
  }
  std::stable_sort(packable.begin(), packable.end(),
                   [](const std::pair<int, int>& a, const std::pair<int, int>& b) { return a.first > b.first; });
  for (const auto& [span, i] : packable) {
    const int r = items[i].rows();
    bool placed = false;
    for (int free = 32; free <= 96 && !placed; free += 32) {
      if (free < span) continue;
      auto& list = open[free / 32];
      size_t& h = head[free / 32];
      if (h == list.size()) continue;
      // only the first open bin of this size is tried
      Bin& bin = list[h];
      if (bin.used_rows + r <= kKnPackRows && int(bin.segs.size()) < kKnPackSegs) {
        Bin taken = std::move(bin);
        ++h;
        taken.segs.push_back(i);
        const int left = free - span;
        if (left && int(taken.segs.size()) < kKnPackSegs)
          open[left / 32].push_back({std::move(taken.segs), taken.used_rows + r});
        else
          tasks.push_back(std::move(taken.segs));
        placed = true;
      }
    }
    if (!placed) {
      const int left = kKeyTile - span;
      if (left)
        open[left / 32].push_back({{i}, r});
      else
        tasks.push_back({i});
    }
  }
  for (int f = 1; f <= 3; ++f)
    for (size_t b = head[f]; b < open[f].size(); ++b) tasks.push_back(std::move(open[f][b].segs));
  return tasks;
}

// Step-time model that picks how far query-tile jobs are cut (tenths of a
// microsecond, from steady-state timelines of the two kernels on one B200):
// a query-tile CTA costs kTcFixed plus kTcPerTile per K/V tile of its piece;
// a keys-in-lanes CTA costs kKnFixed plus kKnPerTask per task it runs.
constexpr int64_t kTcFixed = 70, kTcPerTile = 22, kKnFixed = 25, kKnPerTask = 35;

// Keys-in-lanes tasks per row class of a piece list (the packing below).
void kn_class_counts(const std::vector<PieceRec>& plist, const std::vector<int>& route, const std::vector<int>& rows,
                     int groups, int heads, int64_t counts[5]) {
  const int chunk = std::max(groups, kKnTaskRows / groups * groups);
  std::vector<Item> items;
  for (const PieceRec& pc : plist) {
    if (route[pc.job] != kKn) continue;
    for (int h = 0; h < heads; ++h)
      for (int r0 = 0; r0 < rows[pc.job]; r0 += chunk)
        items.push_back({{h, std::min(chunk, rows[pc.job] - r0), 0, 0, pc.take, 0, -1, 0}});
  }
  for (int c = 0; c < 5; ++c) counts[c] = 0;
  for (const auto& task : pack_segments(items)) {
    int r = 0;
    for (int idx : task) r += items[idx].rows();
    const int c = kn_class(r);
    if (c >= 0) ++counts[c];
  }
}

// Cut level of the query-tile jobs and keys-in-lanes placement with the
// lowest modelled step time: after the query tiles (each class over
// min(kKnDualCtas * sms, tasks) CTAs, the default) or, with one row class,
// beside them on the SMs they leave free.  cap: query-tile CTA cap (0: none);
// beside: query-tile CTAs the keys-in-lanes CTAs are sized against (-1: default
// placement).  Ties keep more query-tile CTAs, then the default placement.
void choose_tc_level(const std::vector<std::pair<int64_t, int64_t>>& levels, const int64_t counts[5], int sms,
                     int64_t& cap, int64_t& beside) {
  cap = 0;
  beside = -1;
  if (levels.empty()) return;
  int used = 0, last = -1;
  for (int c = 0; c < 5; ++c)
    if (counts[c] > 0) {
      ++used;
      last = c;
    }
  auto per_sm = [](int c) { return kKnClassRows[c] <= kKnDualRows ? kKnDualCtas : 1; };
  int64_t best_t = 0;
  int best_index = -1, best_mode = 0;
  auto consider = [&](int64_t t, int index, int mode) {
    // key (t, -index, mode), lexicographically smallest
    if (best_index < 0 || t < best_t || (t == best_t && (index > best_index || (index == best_index && mode < best_mode)))) {
      best_t = t;
      best_index = index;
      best_mode = mode;
    }
  };
  for (int index = 0; index < int(levels.size()); ++index) {
    const int64_t ctas = levels[index].first;
    const int64_t t_tc = kTcFixed + kTcPerTile * levels[index].second;
    if (used == 0) {
      consider(t_tc, index, 0);
      continue;
    }
    int64_t rounds = 0;
    for (int c = 0; c < 5; ++c)
      if (counts[c] > 0) rounds = std::max(rounds, cdiv(counts[c], std::min<int64_t>(int64_t(per_sm(c)) * sms, counts[c])));
    consider(t_tc + kKnFixed + kKnPerTask * rounds, index, 0);
    if (used == 1 && sms > ctas) {
      const int64_t side = std::min<int64_t>(int64_t(per_sm(last)) * (sms - ctas), counts[last]);
      consider(std::max(t_tc, kKnFixed + kKnPerTask * cdiv(counts[last], side)), index, 1);
    }
  }
  cap = best_index == int(levels.size()) - 1 ? 0 : levels[best_index].first;
  beside = best_mode ? levels[best_index].first : -1;
}

// Longest-processing-time assignment of tasks to `bins` persistent CTAs: tasks
// by decreasing cost (ties in input order), each to the least-loaded CTA (ties:
// the lowest CTA index).  offsets [bins + 1]; CTA b runs order[offsets[b]..).
void assign_lpt(const std::vector<int64_t>& costs, int bins, std::vector<int32_t>& offsets,
                std::vector<int32_t>& order) {
  std::vector<int> sorted(costs.size());
  for (size_t t = 0; t < costs.size(); ++t) sorted[t] = int(t);
  std::stable_sort(sorted.begin(), sorted.end(), [&](int a, int b) { return costs[a] > costs[b]; });
  using Load = std::pair<int64_t, int>;
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int b = 0; b < bins; ++b) heap.push({0, b});
  std::vector<std::vector<int>> lists(bins);
  for (int t : sorted) {
    const Load top = heap.top();
    heap.pop();
    lists[top.second].push_back(t);
    heap.push({top.first + costs[t], top.second});
  }
  offsets.assign(bins + 1, 0);
  order.clear();
  for (int b = 0; b < bins; ++b) {
    offsets[b + 1] = offsets[b] + int32_t(lists[b].size());
    order.insert(order.end(), lists[b].begin(), lists[b].end());
  }
}

}  // namespace

extern "C" int ta_plan_build(const int32_t* job_req_offsets, const int32_t* job_reqs, const int32_t* job_k0,
                             const int32_t* job_keys, int32_t num_jobs, int32_t num_requests, int32_t groups,
                             int32_t use_tc, int32_t num_kv_heads, int32_t sms, int64_t no_split_from,
                             int32_t* meta, int64_t meta_capacity, int64_t* meta_size, ta_plan_layout* layout) {
  if (!job_req_offsets || !job_reqs || !job_k0 || !job_keys || !meta_size || !layout) return TA_ERR_ARG;
  if (num_jobs <= 0 || num_requests <= 0 || groups <= 0 || num_kv_heads <= 0 || sms <= 0 || meta_capacity < 0)
    return TA_ERR_ARG;
  const int njobs = num_jobs, nreq = num_requests;
  if (job_req_offsets[0] != 0) return TA_ERR_ARG;
  int maxr = 0;
  for (int i = 0; i < njobs; ++i) {
    const int n = job_req_offsets[i + 1] - job_req_offsets[i];
    if (n <= 0 || job_keys[i] <= 0 || job_k0[i] < 0) return TA_ERR_ARG;
    maxr = std::max(maxr, n);
    for (int j = job_req_offsets[i]; j < job_req_offsets[i + 1]; ++j)
      if (job_reqs[j] < 0 || job_reqs[j] >= nreq) return TA_ERR_ARG;
  }
  auto reqs_of = [&](int i) { return job_reqs + job_req_offsets[i]; };
  auto nreq_of = [&](int i) { return job_req_offsets[i + 1] - job_req_offsets[i]; };

  // ---- the reference's arrays: qids, kids, qlen, klen, slots, counts ----
  std::vector<int> counts(nreq, 0);
  for (int i = 0; i < njobs; ++i)
    for (int j = 0; j < nreq_of(i); ++j) ++counts[reqs_of(i)[j]];
  const int maxs = *std::max_element(counts.begin(), counts.end());

  // ---- pieces ----
  std::vector<int> rows(njobs), route(njobs);
  std::vector<char> splittable(njobs);
  for (int i = 0; i < njobs; ++i) {
    rows[i] = nreq_of(i) * groups;
    route[i] = !use_tc ? kSimt : (rows[i] <= kKnRows ? kKn : kTc);
    splittable[i] = no_split_from < 0 || job_k0[i] < no_split_from;
  }
  std::vector<PieceRec> plist;
  std::vector<std::pair<int64_t, int64_t>> levels;
  split_pieces(njobs, rows, route, job_keys, splittable, num_kv_heads, sms, plist, 0, &levels);
  int64_t kn_counts[5];
  kn_class_counts(plist, route, rows, groups, num_kv_heads, kn_counts);
  int64_t tc_cap = 0, kn_beside = -1;
  choose_tc_level(levels, kn_counts, sms, tc_cap, kn_beside);
  if (tc_cap > 0) {
    plist.clear();
    split_pieces(njobs, rows, route, job_keys, splittable, num_kv_heads, sms, plist, tc_cap);
  }
  const int npieces = int(plist.size());
  std::vector<int32_t> piece_slot(npieces);
  std::vector<int> pcounts(nreq, 0);
  int64_t slot = 0;
  for (int p = 0; p < npieces; ++p) {
    piece_slot[p] = int32_t(slot);
    const int i = plist[p].job;
    for (int j = 0; j < nreq_of(i); ++j) ++pcounts[reqs_of(i)[j]];
    slot += nreq_of(i);
  }
  if (slot > INT32_MAX / std::max(1, groups)) return TA_ERR_ARG;
  const int maxp = *std::max_element(pcounts.begin(), pcounts.end());

  // ---- kernel task lists ----
  std::vector<std::pair<int, int>> small[3];
  std::vector<int32_t> tc;   // [n, 4]
  std::vector<Item> items;
  for (int p = 0; p < npieces; ++p) {
    const int i = plist[p].job, offset = plist[p].offset, take = plist[p].take;
    const int32_t* rq = reqs_of(i);
    const int n = nreq_of(i);
    const int q0 = rq[n - 1] - rq[0] + 1 == n ? rq[0] : -1;
    if (route[i] == kKn) {
      const int growing = no_split_from >= 0 && job_k0[i] >= no_split_from ? 1 : 0;
      const int chunk = std::max(groups, kKnTaskRows / groups * groups);
      for (int h = 0; h < num_kv_heads; ++h)
        for (int r0 = 0; r0 < rows[i]; r0 += chunk) {
          const int c0 = r0 / groups;
          items.push_back({{h, std::min(chunk, rows[i] - r0), piece_slot[p] * groups + r0, job_k0[i] + offset, take,
                            i | (growing << kGrowingBit), q0 >= 0 ? q0 + c0 : -1, c0}});
        }
    } else if (route[i] == kTc) {
      for (int t = 0; t < int(cdiv(rows[i], kTcRows)); ++t) tc.insert(tc.end(), {p, t, q0, 0});
    } else {
      for (int t = 0; t < int(cdiv(rows[i], kSmallRows)); ++t)
        small[small_class(std::min(kSmallRows, rows[i] - t * kSmallRows))].push_back({p, t});
    }
  }
  int small_max_keys = 0;
  for (const auto& c : small)
    for (const auto& st : c) small_max_keys = std::max(small_max_keys, plist[st.first].take);

  const std::vector<std::vector<int>> tasks = pack_segments(items);
  std::vector<int32_t> segs;   // [n, 12]
  std::vector<std::pair<int, int64_t>> by_class[5];   // (task, cost) per row class
  std::vector<int32_t> headers;                       // [n, 4] in task order
  for (int t = 0; t < int(tasks.size()); ++t) {
    const auto& task = tasks[t];
    headers.insert(headers.end(), {int32_t(segs.size() / 12), int32_t(task.size()), 0, 0});
    int row0 = 0, kt = 0, max_keys = 0;
    for (int idx : task) {
      const Item& it = items[idx];
      segs.insert(segs.end(), {it.v[0], row0, it.v[1], it.v[2], it.v[3], task.size() > 1 ? kt : 0, it.v[4], it.v[5],
                               it.v[6], it.v[7], 0, 0});
      row0 += it.v[1];
      kt += int(cdiv(it.v[4], kKnBox)) * kKnBox;
      max_keys = std::max(max_keys, it.v[4]);
    }
    const int c = kn_class(row0);
    if (c < 0) return TA_ERR_UNSUPPORTED;
    by_class[c].push_back({t, int64_t(tiles_of(max_keys)) + 1});
  }
  int32_t class_ctas[5] = {0, 0, 0, 0, 0};
  std::vector<int32_t> kn_offsets{0}, kn_tasks;
  {
    std::vector<int32_t> offs, order;
    std::vector<int64_t> costs;
    int32_t base = 0;
    for (int c = 0; c < 5; ++c) {
      const auto& entries = by_class[c];
      if (entries.empty()) continue;
      // beside the query tiles (kn_beside >= 0): on the SMs they leave free
      const int64_t free_sms = kn_beside >= 0 ? int64_t(sms) - kn_beside : int64_t(sms);
      const int ctas = int(std::min<int64_t>(free_sms * (kKnClassRows[c] <= kKnDualRows ? kKnDualCtas : 1),
                                             int64_t(entries.size())));
      costs.clear();
      for (const auto& e : entries) costs.push_back(e.second);
      assign_lpt(costs, ctas, offs, order);
      for (int b = 1; b <= ctas; ++b) kn_offsets.push_back(offs[b] + base);
      for (int o : order) {
        const int t = entries[o].first;
        kn_tasks.insert(kn_tasks.end(), headers.begin() + 4 * t, headers.begin() + 4 * t + 4);
      }
      base += int32_t(order.size());
      class_ctas[c] = ctas;
    }
  }

  // ---- layout: the arrays in order, each on a 4-int32 boundary ----
  const int64_t sizes[14] = {int64_t(njobs) * maxr, njobs, njobs, njobs, int64_t(nreq) * maxs, nreq,
                             int64_t(npieces) * 4, nreq, int64_t(nreq) * maxp,
                             int64_t(small[0].size() + small[1].size() + small[2].size()) * 2,
                             int64_t(tc.size()), int64_t(kn_offsets.size()), int64_t(kn_tasks.size()),
                             int64_t(segs.size())};
  int64_t offs[14];
  int64_t total = 0;
  for (int a = 0; a < 14; ++a) {
    total += (4 - total % 4) % 4;
    offs[a] = total;
    total += sizes[a];
  }
  if (total > INT32_MAX) return TA_ERR_ARG;
  *meta_size = total;
  ta_plan_layout L;
  std::memset(&L, 0, sizeof(L));
  L.num_jobs = njobs;
  L.max_requests = maxr;
  L.max_slots = maxs;
  L.num_requests = nreq;
  L.num_pieces = npieces;
  L.num_partials = int32_t(slot);
  L.max_pslots = maxp;
  L.num_small_tasks = int32_t(small[0].size() + small[1].size() + small[2].size());
  L.num_tc_tasks = int32_t(tc.size() / 4);
  L.num_kn_tasks = int32_t(kn_tasks.size() / 4);
  L.num_kn_segs = int32_t(segs.size() / 12);
  L.kn_ctas = int32_t(kn_offsets.size() - 1);
  for (int c = 0; c < 5; ++c) L.kn_class_ctas[c] = class_ctas[c];
  L.small_class_end[0] = int32_t(small[0].size());
  L.small_class_end[1] = int32_t(small[0].size() + small[1].size());
  L.small_class_end[2] = L.num_small_tasks;
  L.small_max_keys = small_max_keys;
  L.kstart_stride = 1;
  int32_t* const off_fields[14] = {&L.off_qids, &L.off_kstart, &L.off_qlen, &L.off_klen, &L.off_slots,
                                   &L.off_counts, &L.off_pieces, &L.off_pcounts, &L.off_cslots,
                                   &L.off_small_tasks, &L.off_tc_tasks, &L.off_kn_offsets, &L.off_kn_tasks,
                                   &L.off_kn_segs};
  for (int a = 0; a < 14; ++a) *off_fields[a] = int32_t(offs[a]);
  *layout = L;
  if (!meta || meta_capacity < total) return TA_ERR_TOO_LARGE;

  std::memset(meta, 0, size_t(total) * sizeof(int32_t));
  int32_t* qids = meta + offs[0];
  int32_t* kids = meta + offs[1];
  int32_t* qlen = meta + offs[2];
  int32_t* klen = meta + offs[3];
  int32_t* slots = meta + offs[4];
  int32_t* cnt = meta + offs[5];
  std::vector<int> fill(nreq, 0);
  for (int i = 0; i < njobs; ++i) {
    const int n = nreq_of(i);
    for (int j = 0; j < n; ++j) {
      const int r = reqs_of(i)[j];
      qids[int64_t(i) * maxr + j] = r;
      slots[int64_t(r) * maxs + fill[r]++] = i * maxr + j;
    }
    kids[i] = job_k0[i];
    qlen[i] = n;
    klen[i] = job_keys[i];
  }
  for (int r = 0; r < nreq; ++r) cnt[r] = counts[r];
  int32_t* pieces = meta + offs[6];
  int32_t* pc = meta + offs[7];
  int32_t* cslots = meta + offs[8];
  std::fill(fill.begin(), fill.end(), 0);
  for (int p = 0; p < npieces; ++p) {
    const int i = plist[p].job;
    pieces[4 * p + 0] = i;
    pieces[4 * p + 1] = plist[p].offset;
    pieces[4 * p + 2] = plist[p].take;
    pieces[4 * p + 3] = piece_slot[p];
    for (int j = 0; j < nreq_of(i); ++j) {
      const int r = reqs_of(i)[j];
      cslots[int64_t(r) * maxp + fill[r]++] = piece_slot[p] + j;
    }
  }
  for (int r = 0; r < nreq; ++r) pc[r] = pcounts[r];
  int32_t* st = meta + offs[9];
  for (const auto& c : small)
    for (const auto& e : c) {
      *st++ = e.first;
      *st++ = e.second;
    }
  std::copy(tc.begin(), tc.end(), meta + offs[10]);
  std::copy(kn_offsets.begin(), kn_offsets.end(), meta + offs[11]);
  std::copy(kn_tasks.begin(), kn_tasks.end(), meta + offs[12]);
  std::copy(segs.begin(), segs.end(), meta + offs[13]);
  return TA_OK;
}
