// Host-side list scheduling of a dependency DAG (no device work): the start order in which the
// persistent dataflow kernels take their rows.
//
// The dataflow kernels start a row when its dependencies are done.  Taking ready rows first come,
// first served leaves the rows of the longest remaining chains to start late, and the pass ends
// with a tail in which few SMs have work.  This simulates the classic critical-path list schedule
// on n_workers identical workers with a per-row cost model -- a ready row with the largest
// "level" (its cost plus the largest level among the rows that wait on it) starts first -- and
// returns the order in which rows START in it.  That order lists every row after the rows it
// depends on, so CTAs that take rows in it, each waiting until its row's dependencies are done,
// always make progress (the row of the earliest unfinished position has all its dependencies done).

#include <algorithm>
#include <functional>
#include <queue>
#include <utility>
#include <vector>

#include "kb_common.cuh"
#include "kb_solver.h"

extern "C" int kb_list_schedule(int n, const long long* pred_ptr, const int* pred_idx, const long long* succ_ptr,
                                const int* succ_idx, const double* cost, int n_workers, int* order_out,
                                double* makespan_out) {
  if (n < 0 || n_workers < 1 || (n > 0 && (!pred_ptr || !pred_idx || !succ_ptr || !succ_idx || !cost || !order_out)))
    return KB_ERR_ARG;
  if (n == 0) {
    if (makespan_out) *makespan_out = 0.0;
    return KB_OK;
  }
  // topological order (Kahn, sources first), then levels from the sinks back
  std::vector<long long> rem(n);
  std::vector<int> topo;
  topo.reserve(n);
  for (int i = 0; i < n; ++i) {
    rem[i] = pred_ptr[i + 1] - pred_ptr[i];
    if (rem[i] < 0) return KB_ERR_ARG;
    if (rem[i] == 0) topo.push_back(i);
  }
  for (size_t h = 0; h < topo.size(); ++h) {
    const int r = topo[h];
    for (long long j = succ_ptr[r]; j < succ_ptr[r + 1]; ++j) {
      const int s = succ_idx[j];
      if (s < 0 || s >= n) return KB_ERR_ARG;
      if (--rem[s] == 0) topo.push_back(s);
    }
  }
  if ((int)topo.size() != n) return KB_ERR_ARG;  // a cycle, or counts that do not match the edges
  std::vector<double> level(n);
  for (int h = n - 1; h >= 0; --h) {
    const int r = topo[h];
    double m = 0.0;
    for (long long j = succ_ptr[r]; j < succ_ptr[r + 1]; ++j) m = std::max(m, level[succ_idx[j]]);
    level[r] = cost[r] + m;
  }
  // the list schedule: ready rows by decreasing level (then increasing index), workers by finish time
  auto lower = [&](int a, int b) { return level[a] < level[b] || (level[a] == level[b] && a > b); };
  std::priority_queue<int, std::vector<int>, decltype(lower)> ready(lower);
  typedef std::pair<double, int> Busy;
  std::priority_queue<Busy, std::vector<Busy>, std::greater<Busy>> busy;
  for (int i = 0; i < n; ++i) {
    rem[i] = pred_ptr[i + 1] - pred_ptr[i];
    if (rem[i] == 0) ready.push(i);
  }
  double t = 0.0;
  int free_workers = n_workers, started = 0, done = 0;
  while (done < n) {
    while (free_workers > 0 && !ready.empty()) {
      const int r = ready.top();
      ready.pop();
      order_out[started++] = r;
      busy.push(Busy(t + cost[r], r));
      --free_workers;
    }
    const Busy b = busy.top();
    busy.pop();
    t = b.first;
    ++free_workers;
    ++done;
    for (long long j = succ_ptr[b.second]; j < succ_ptr[b.second + 1]; ++j)
      if (--rem[succ_idx[j]] == 0) ready.push(succ_idx[j]);
  }
  if (makespan_out) *makespan_out = t;
  return KB_OK;
}
