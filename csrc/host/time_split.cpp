// Adaptive time splitting of an event stream (the batching scheme of the
// reference's chunk pipeline, vendor/bts_sampler/split/time_split.cpp:22-410):
// a window is cut when its accumulated staleness exceeds a threshold derived
// from fixed-size base batches (mean + graph_feature * (max - mean)). Staleness
// of a repeated node visit = (alpha + 2 beta) (exp(clamp((t_last - t_batch) /
// (t_now - t_batch))) + exp(min(0.01 * visits, 100))); a repeated endpoint also
// adds the aggregation loss ``aggl``. Optional edge dropping keeps the
// (1 - drop_rate) fraction of events with the lowest per-window staleness.
#include <cmath>
#include <numeric>
#include <unordered_map>

#include "native.h"

namespace sun {
namespace {

double staleness(double tlast, double tnow, double tbatch, int visits, double alpha, double beta) {
  if (tnow - tlast == 0.0) return 0.0;
  double diff = tnow - tbatch;
  if (std::abs(diff) < 1e-6) diff = 1e-6;
  const double a0 = std::clamp((tlast - tbatch) / diff, -100.0, 100.0);
  const double d0 = std::min(1e-2 * visits, 100.0);
  const double coeff = alpha + 2.0 * beta;
  return coeff * std::exp(a0) + coeff * std::exp(d0);
}

struct Window {
  // per node: time of its last counted visit and the number of counted visits
  std::unordered_map<int64_t, std::pair<double, int>> seen;
  std::unordered_map<int64_t, double> last_time;
};

// Adds event (s, d, t) to the window and returns the staleness it contributes.
double visit(Window& w, const std::unordered_map<int64_t, double>& tbatch, int64_t s, int64_t d, double t, double alpha,
             double beta, double aggl) {
  double st = 0.0;
  w.last_time[s] = t;
  w.last_time[d] = t;
  const bool hs = w.seen.count(s), hd = w.seen.count(d);
  st += (hs ? aggl : 0.0) + (hd ? aggl : 0.0);
  auto touch = [&](int64_t node) {
    auto& e = w.seen[node];
    if (t - e.first != 0.0) {
      st += staleness(e.first, t, tbatch.at(node), e.second, alpha, beta);
      e.first = t;
      e.second += 1;
    }
  };
  if (!hs && !hd) {
    w.seen[s] = {t, 1};
    w.seen[d] = {t, s == d ? 2 : 1};
  } else if (!hs) {
    touch(d);
    w.seen[s] = {t, 1};
  } else if (!hd) {
    touch(s);
    w.seen[d] = {t, 1};
  } else if (s == d) {
    touch(s);
  } else {
    touch(s);
    touch(d);
  }
  return st;
}

std::unordered_map<int64_t, double> initial_times(const int64_t* s, const int64_t* d, const double* t, int64_t n) {
  std::unordered_map<int64_t, double> m;
  for (int64_t i = 0; i < n; ++i) {
    m.emplace(s[i], t[0]);
    m.emplace(d[i], t[0]);
  }
  return m;
}

}  // namespace

static double threshold_of(const int64_t* s, const int64_t* d, const double* t, int64_t n, int64_t bs, double gf,
                           double alpha, double beta, double aggl) {
  auto tb = initial_times(s, d, t, n);
  std::vector<double> per;
  for (int64_t a = 0; a < n; a += std::max<int64_t>(1, bs)) {
    const int64_t b = std::min(n, a + std::max<int64_t>(1, bs));
    Window w;
    double st = 0.0;
    for (int64_t i = a; i < b; ++i) st += visit(w, tb, s[i], d[i], t[i], alpha, beta, aggl);
    for (auto& kv : w.last_time) tb[kv.first] = kv.second;
    per.push_back(st);
  }
  if (per.empty()) return 0.0;
  const double mean = std::accumulate(per.begin(), per.end(), 0.0) / per.size();
  const double mx = *std::max_element(per.begin(), per.end());
  return mean + gf * (mx - mean);
}

static std::vector<int64_t> drop_edges(const int64_t* s, const int64_t* d, const double* t, int64_t n, int64_t win,
                                       double alpha, double beta, double drop_rate) {
  auto tb = initial_times(s, d, t, n);
  std::vector<double> score(n);
  for (int64_t a = 0; a < n; a += std::max<int64_t>(1, win)) {
    const int64_t b = std::min(n, a + std::max<int64_t>(1, win));
    Window w;
    for (int64_t i = a; i < b; ++i) score[i] = -visit(w, tb, s[i], d[i], t[i], alpha, beta, 0.0);
    for (auto& kv : w.last_time) tb[kv.first] = kv.second;
  }
  std::vector<double> sorted = score;
  std::sort(sorted.begin(), sorted.end());
  const int64_t keep = std::max<int64_t>(1, static_cast<int64_t>((1.0 - drop_rate) * n));
  const double thr = sorted[keep - 1];
  std::vector<int64_t> idx;
  for (int64_t i = 0; i < n; ++i)
    if (score[i] <= thr) idx.push_back(i);
  return idx;
}

static std::vector<int64_t> split(const int64_t* s, const int64_t* d, const double* t, int64_t n, double thr,
                                  double alpha, double beta, double aggl) {
  std::vector<int64_t> group(n, 0);
  auto tb = initial_times(s, d, t, n);
  std::vector<int64_t> cuts{0};
  int64_t start = 0;
  while (start < n - 1) {
    Window w;
    double st = 0.0;
    for (int64_t i = start; i < n; ++i) {
      st += visit(w, tb, s[i], d[i], t[i], alpha, beta, aggl);
      if (st > thr || i == n - 1) {
        cuts.push_back(i);
        start = i;
        for (auto& kv : w.last_time) tb[kv.first] = kv.second;
        break;
      }
    }
  }
  cuts.back() = n;
  for (size_t g = 0; g + 1 < cuts.size(); ++g)
    for (int64_t j = cuts[g]; j < cuts[g + 1]; ++j) group[j] = static_cast<int64_t>(g);
  return group;
}

SplitResult adaptive_split(torch::Tensor src, torch::Tensor dst, torch::Tensor ts, int64_t base_batch_size,
                           double graph_feature, double alpha, double beta, double aggl, bool enable_drop,
                           double drop_rate, int64_t window_size) {
  TORCH_CHECK(src.dim() == 1 && dst.dim() == 1 && ts.dim() == 1, "inputs must be 1-D");
  TORCH_CHECK(src.numel() == dst.numel() && src.numel() == ts.numel(), "size mismatch");
  auto s = src.to(torch::kInt64).contiguous(), d = dst.to(torch::kInt64).contiguous();
  auto t = ts.to(torch::kFloat64).contiguous();
  const int64_t n = s.numel();
  SplitResult r;
  if (n == 0) {
    r.group_index = torch::zeros({0}, torch::kInt64);
    r.keep_indices = torch::zeros({0}, torch::kInt64);
    return r;
  }
  if (enable_drop) {
    auto keep = drop_edges(s.data_ptr<int64_t>(), d.data_ptr<int64_t>(), t.data_ptr<double>(), n, window_size, alpha,
                           beta, drop_rate);
    r.keep_indices = torch::tensor(keep, torch::kInt64);
    r.drop_proportion = 1.0 - static_cast<double>(keep.size()) / n;
    s = s.index({r.keep_indices}).contiguous();
    d = d.index({r.keep_indices}).contiguous();
    t = t.index({r.keep_indices}).contiguous();
  } else {
    r.keep_indices = torch::arange(n, torch::kInt64);
  }
  const int64_t m = s.numel();
  const double thr = threshold_of(s.data_ptr<int64_t>(), d.data_ptr<int64_t>(), t.data_ptr<double>(), m,
                                  base_batch_size, graph_feature, alpha, beta, aggl);
  auto g = split(s.data_ptr<int64_t>(), d.data_ptr<int64_t>(), t.data_ptr<double>(), m, thr, alpha, beta, aggl);
  r.group_index = torch::tensor(g, torch::kInt64);
  return r;
}

}  // namespace sun
