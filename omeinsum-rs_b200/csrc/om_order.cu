// Contraction-order optimiser: simulated annealing over binary contraction
// trees (host code).
//
// Replaces the reference's call into omeco's TreeSA
// (src/einsum/engine.rs:84-91, optimize_treesa; omeco 0.2.4, an external
// crate absent from the reference tree).  This is this library's own
// restatement of the published tree-annealing idea (Kalachev, Panteleev,
// Zhou, Zhang, "Multi-tensor contraction for XEB verification of quantum
// circuits", 2021; the TreeSA method of OMEinsumContractionOrders.jl):
//   * state: a binary tree over the input tensors;
//   * move: a rotation at an internal node X = (A, Y) with Y = (B, C)
//     internal -- X becomes ((A, C), B) or ((A, B), C) -- which changes the
//     labels of one intermediate only;
//   * cost: log2(sum over nodes of 2^tc(node)) + sc_weight * sum over nodes
//     of max(0, log2 size(node) - sc_target) + rw_weight * log2(sum of the
//     nodes' read-write sizes), tc(node) = log2 of the product of the
//     extents of every label the node touches;
//   * kept: the best tree seen at the end of a beta level by log2 tc +
//     sc_weight * max(0, largest log2 intermediate - sc_target);
//   * Metropolis acceptance exp(-beta * delta) on the local change of the
//     two nodes a move touches (log2-sum of their tc, their sizes above
//     sc_target, their read-write volume), beta swept from beta_start
//     to beta_end in beta_step increments, niters sweeps (one move attempt
//     per internal node) per beta; the best of ntrials independent runs.
// Trials without a given start begin from a randomised greedy tree.
// Labels of an intermediate: a label of a child is kept unless every one of
// its occurrences (among the inputs) lies under the node and it is not an
// output label, so hyper-edges (labels on three or more tensors) are exact.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdint>
#include <map>
#include <random>
#include <vector>

#include "om_internal.h"

namespace om {
namespace {

struct LabelCount {
  int32_t label;
  int32_t count;  // occurrences among the inputs under the node
};

struct Optimiser {
  int n;                      // inputs
  std::vector<double> lsize;  // log2 extent per dense label id
  std::vector<int32_t> total; // occurrences of each label among the inputs
  std::vector<char> in_out;   // label is an output label
  // tree: nodes 0..n-1 leaves, n..2n-2 internal
  std::vector<int> left, right, parent;
  std::vector<std::vector<LabelCount>> out;  // labels of each node's tensor (sorted)
  std::vector<double> tc, sc, rw;            // log2 per internal node
  double sc_target, sc_weight, rw_weight;

  // labels of (a, b) combined, contracted labels dropped
  void combine(const std::vector<LabelCount>& a, const std::vector<LabelCount>& b,
               std::vector<LabelCount>& o, double* all_log2) const {
    o.clear();
    double all = 0.0;
    size_t i = 0, j = 0;
    while (i < a.size() || j < b.size()) {
      LabelCount x;
      if (j == b.size() || (i < a.size() && a[i].label < b[j].label)) {
        x = a[i++];
      } else if (i == a.size() || b[j].label < a[i].label) {
        x = b[j++];
      } else {
        x = {a[i].label, a[i].count + b[j].count};
        ++i;
        ++j;
      }
      all += lsize[x.label];
      if (x.count < total[x.label] || in_out[x.label]) o.push_back(x);
    }
    *all_log2 = all;
  }
  static double size_of(const std::vector<double>& ls, const std::vector<LabelCount>& v) {
    double s = 0;
    for (auto& x : v) s += ls[x.label];
    return s;
  }
  void eval(int x) {
    double all;
    combine(out[left[x]], out[right[x]], out[x], &all);
    tc[x] = all;
    sc[x] = size_of(lsize, out[x]);
    // read-write: both operands and the result
    rw[x] = log2sum3(size_of(lsize, out[left[x]]), size_of(lsize, out[right[x]]), sc[x]);
  }
  static double log2sum3(double a, double b, double c) {
    const double m = std::max(a, std::max(b, c));
    return m + std::log2(std::exp2(a - m) + std::exp2(b - m) + std::exp2(c - m));
  }
  double penalty(double s) const { return s > sc_target ? s - sc_target : 0.0; }
};

}  // namespace
}  // namespace om

using namespace om;

extern "C" int om_b200_optimize_tree(int ntensors, const int32_t* ndims, const int32_t* ixs,
                                     int niy, const int32_t* iy, int nsizes,
                                     const int32_t* size_labels, const int64_t* size_values,
                                     const int32_t* init_children, double sc_target,
                                     double sc_weight, double rw_weight, int ntrials, int niters,
                                     double beta_start, double beta_end, double beta_step,
                                     uint64_t seed, int32_t* children_out, double* tc_out,
                                     double* sc_out) {
  if (ntensors < 2 || !ndims || !ixs || !children_out || (niy && !iy) || (nsizes && (!size_labels || !size_values)))
    return set_error(OM_ERR_INVALID, "om_b200_optimize_tree: bad argument");
  if (ntrials < 1 || niters < 1 || !(beta_step > 0) || beta_end < beta_start)
    return set_error(OM_ERR_INVALID, "om_b200_optimize_tree: bad annealing schedule");
  const int n = ntensors, nn = 2 * n - 1;
  // dense label ids
  std::map<int32_t, int32_t> id;
  std::map<int32_t, int64_t> ext;
  for (int q = 0; q < nsizes; ++q) ext[size_labels[q]] = size_values[q];
  auto dense = [&](int32_t l) {
    auto it = id.find(l);
    if (it != id.end()) return it->second;
    const int32_t d = (int32_t)id.size();
    id[l] = d;
    return d;
  };
  std::vector<std::vector<int32_t>> leaf_labels(n);
  int64_t off = 0;
  for (int t = 0; t < n; ++t) {
    for (int d = 0; d < ndims[t]; ++d) leaf_labels[t].push_back(dense(ixs[off + d]));
    off += ndims[t];
  }
  for (int q = 0; q < niy; ++q) dense(iy[q]);
  Optimiser O;
  O.n = n;
  const int nl = (int)id.size();
  O.lsize.assign(nl, 0.0);
  O.total.assign(nl, 0);
  O.in_out.assign(nl, 0);
  for (auto& kv : id) {
    auto e = ext.find(kv.first);
    if (e == ext.end()) return set_error(OM_ERR_SHAPE, "om_b200_optimize_tree: a label has no size");
    O.lsize[kv.second] = std::log2((double)std::max<int64_t>(1, e->second));
  }
  for (int q = 0; q < niy; ++q) O.in_out[id[iy[q]]] = 1;
  std::vector<std::vector<LabelCount>> leaf_out(n);
  for (int t = 0; t < n; ++t) {
    std::map<int32_t, int32_t> c;
    for (auto l : leaf_labels[t]) c[l]++;
    for (auto& kv : c) {
      O.total[kv.first] += kv.second;
      leaf_out[t].push_back({kv.first, kv.second});
    }
  }
  O.sc_target = sc_target;
  O.sc_weight = sc_weight;
  O.rw_weight = rw_weight;

  std::mt19937_64 rng(seed);
  std::uniform_real_distribution<double> U(0.0, 1.0);
  double best_cost = INFINITY;
  std::vector<int> best_left, best_right;
  int best_root = -1;

  for (int trial = 0; trial < ntrials; ++trial) {
    O.left.assign(nn, -1);
    O.right.assign(nn, -1);
    O.parent.assign(nn, -1);
    O.out.assign(nn, {});
    O.tc.assign(nn, 0.0);
    O.sc.assign(nn, 0.0);
    O.rw.assign(nn, 0.0);
    for (int t = 0; t < n; ++t) O.out[t] = leaf_out[t];
    int root;
    if (init_children && trial == 0) {
      for (int i = 0; i < n - 1; ++i) {
        const int a = init_children[2 * i], b = init_children[2 * i + 1];
        if (a < 0 || b < 0 || a >= n + i || b >= n + i)
          return set_error(OM_ERR_INVALID, "om_b200_optimize_tree: init tree refers to a later node");
        O.left[n + i] = a;
        O.right[n + i] = b;
        O.parent[a] = n + i;
        O.parent[b] = n + i;
      }
      root = nn - 1;
    } else {
      // randomised greedy start: repeatedly join the pair of current tensors
      // sharing a label with the smallest log2 size(out) - log2(size(a) +
      // size(b)) plus uniform noise in [0, 1); unconnected parts are joined
      // smallest first at the end
      std::vector<int> alive(n);
      for (int t = 0; t < n; ++t) alive[t] = t;
      std::vector<LabelCount> o;
      int next = n;
      std::vector<std::vector<int>> holders(nl);
      for (int t = 0; t < n; ++t)
        for (auto& lc : leaf_out[t]) holders[lc.label].push_back(t);
      std::vector<char> live(nn, 0);
      for (int t = 0; t < n; ++t) live[t] = 1;
      while (next < nn) {
        double best = INFINITY;
        int ba = -1, bb = -1;
        for (int l = 0; l < nl; ++l) {
          auto& h = holders[l];
          for (size_t i = 0; i < h.size(); ++i)
            for (size_t j = i + 1; j < h.size(); ++j) {
              double all;
              O.combine(O.out[h[i]], O.out[h[j]], o, &all);
              const double sa = Optimiser::size_of(O.lsize, O.out[h[i]]);
              const double sb = Optimiser::size_of(O.lsize, O.out[h[j]]);
              const double m = std::max(sa, sb);
              const double key = Optimiser::size_of(O.lsize, o) -
                                 (m + std::log2(std::exp2(sa - m) + std::exp2(sb - m))) + U(rng);
              if (key < best) {
                best = key;
                ba = h[i];
                bb = h[j];
              }
            }
        }
        if (ba < 0) {  // no shared label left: join the two smallest tensors
          std::vector<std::pair<double, int>> by;
          for (int x = 0; x < next; ++x)
            if (live[x]) by.push_back({Optimiser::size_of(O.lsize, O.out[x]), x});
          std::sort(by.begin(), by.end());
          ba = by[0].second;
          bb = by[1].second;
        }
        const int x = next++;
        O.left[x] = ba;
        O.right[x] = bb;
        O.parent[ba] = O.parent[bb] = x;
        double all;
        O.combine(O.out[ba], O.out[bb], O.out[x], &all);
        live[ba] = live[bb] = 0;
        live[x] = 1;
        for (auto* y : {&ba, &bb})
          for (auto& lc : O.out[*y]) {
            auto& h = holders[lc.label];
            h.erase(std::remove(h.begin(), h.end(), *y), h.end());
          }
        for (auto& lc : O.out[x]) holders[lc.label].push_back(x);
      }
      root = nn - 1;
    }
    // post-order evaluation
    {
      std::vector<int> st{root}, order;
      while (!st.empty()) {
        const int x = st.back();
        st.pop_back();
        if (x < n) continue;
        order.push_back(x);
        st.push_back(O.left[x]);
        st.push_back(O.right[x]);
      }
      for (auto it = order.rbegin(); it != order.rend(); ++it) O.eval(*it);
    }
    // totals
    auto totals = [&](double* T, double* P, double* R) {
      double m = -INFINITY, mr = -INFINITY;
      for (int x = n; x < nn; ++x) {
        m = std::max(m, O.tc[x]);
        mr = std::max(mr, O.rw[x]);
      }
      double s = 0, sr = 0, p = 0;
      for (int x = n; x < nn; ++x) {
        s += std::exp2(O.tc[x] - m);
        sr += std::exp2(O.rw[x] - mr);
        p += O.penalty(O.sc[x]);
      }
      *T = m + std::log2(s);
      *R = mr + std::log2(sr);
      *P = p;
    };
    double T, P, R;
    totals(&T, &P, &R);
    // running sums in linear scale relative to a fixed reference exponent
    double ref = T, refr = R;
    double lin = std::exp2(T - ref), linr = std::exp2(R - refr);
    auto cost = [&](double l, double lr, double p) {
      return (ref + std::log2(std::max(l, 1e-300))) + O.sc_weight * p +
             O.rw_weight * (refr + std::log2(std::max(lr, 1e-300)));
    };
    double cur = cost(lin, linr, P);
    std::vector<int> internal;
    for (int x = n; x < nn; ++x) internal.push_back(x);
    std::vector<LabelCount> tmp;
    // the best state of this trial, judged at the end of every beta level
    // by log2 tc + sc_weight * max(0, largest log2 size - sc_target)
    auto score = [&]() {
      double m = -INFINITY, msc = 0;
      for (int x = n; x < nn; ++x) {
        m = std::max(m, O.tc[x]);
        msc = std::max(msc, O.sc[x]);
      }
      double sum = 0;
      for (int x = n; x < nn; ++x) sum += std::exp2(O.tc[x] - m);
      return m + std::log2(sum) + O.sc_weight * std::max(0.0, msc - O.sc_target);
    };
    double trial_best = score();
    std::vector<int> tb_left = O.left, tb_right = O.right;
    auto keep_if_best = [&]() {
      const double sc_now = score();
      if (sc_now < trial_best - 1e-9) {
        trial_best = sc_now;
        tb_left = O.left;
        tb_right = O.right;
      }
    };
    for (double beta = beta_start; beta <= beta_end + 1e-12; beta += beta_step) {
      for (int it = 0; it < niters; ++it) {
        for (size_t mv = 0; mv < internal.size(); ++mv) {
          const int X = internal[rng() % internal.size()];
          // pick an internal child Y of X and the other child A
          int side = (int)(rng() & 1);
          int Y = side ? O.right[X] : O.left[X];
          if (Y < n) {
            side ^= 1;
            Y = side ? O.right[X] : O.left[X];
            if (Y < n) continue;
          }
          const int A = side ? O.left[X] : O.right[X];
          // swap A with one of Y's children (the other, K, stays in Y)
          const int pick = (int)(rng() & 1);
          const int S = pick ? O.right[Y] : O.left[Y];  // goes up to X
          const int K = pick ? O.left[Y] : O.right[Y];  // stays under Y, joined by A
          // new Y' = (K, A); X' = (Y', S)
          double all_y;
          O.combine(O.out[K], O.out[A], tmp, &all_y);
          const double sc_y = Optimiser::size_of(O.lsize, tmp);
          const double rw_y = Optimiser::log2sum3(Optimiser::size_of(O.lsize, O.out[K]),
                                                  Optimiser::size_of(O.lsize, O.out[A]), sc_y);
          // X's touched labels: out(Y') u out(S)
          double all_x = 0;
          {
            size_t i = 0, j = 0;
            const auto& a = tmp;
            const auto& b = O.out[S];
            while (i < a.size() || j < b.size()) {
              int32_t l;
              if (j == b.size() || (i < a.size() && a[i].label < b[j].label)) l = a[i++].label;
              else if (i == a.size() || b[j].label < a[i].label) l = b[j++].label;
              else {
                l = a[i].label;
                ++i;
                ++j;
              }
              all_x += O.lsize[l];
            }
          }
          const double rw_x = Optimiser::log2sum3(sc_y, Optimiser::size_of(O.lsize, O.out[S]), O.sc[X]);
          const double nlin = lin - std::exp2(O.tc[X] - ref) - std::exp2(O.tc[Y] - ref) +
                              std::exp2(all_x - ref) + std::exp2(all_y - ref);
          const double nlinr = linr - std::exp2(O.rw[X] - refr) - std::exp2(O.rw[Y] - refr) +
                               std::exp2(rw_x - refr) + std::exp2(rw_y - refr);
          const double nP = P - O.penalty(O.sc[Y]) + O.penalty(sc_y);
          const double nc = cost(nlin, nlinr, nP);
          const double d = nc - cur;
          // acceptance on the local change of the two nodes the move touches
          // (a global log-sum hides changes at small nodes, so they would
          // drift freely)
          auto lse2 = [](double a, double b) {
            const double m = std::max(a, b);
            return m + std::log2(std::exp2(a - m) + std::exp2(b - m));
          };
          const double dloc = lse2(all_x, all_y) - lse2(O.tc[X], O.tc[Y]) +
                              O.sc_weight * (std::max(sc_y, O.sc_target) - std::max(O.sc[Y], O.sc_target)) +
                              O.rw_weight * (lse2(rw_x, rw_y) - lse2(O.rw[X], O.rw[Y]));
          if (dloc <= 0 || U(rng) < std::exp(-beta * dloc)) {
            // apply: Y = (K, A), X = (Y, S)
            O.left[Y] = K;
            O.right[Y] = A;
            O.parent[A] = Y;
            if (side) {
              O.left[X] = S;
            } else {
              O.right[X] = S;
            }
            O.parent[S] = X;
            O.out[Y] = tmp;
            O.tc[Y] = all_y;
            O.sc[Y] = sc_y;
            O.rw[Y] = rw_y;
            O.tc[X] = all_x;
            O.rw[X] = rw_x;
            lin = nlin;
            linr = nlinr;
            P = nP;
            cur = nc;
            (void)d;
          }
        }
      }
      keep_if_best();
      if (trace_on())
        fprintf(stderr, "[om trace] treesa trial %d beta %.3f score %.3f best %.3f\n", trial, beta,
                score(), trial_best);
      // re-anchor the running sums (rounding drift)
      totals(&T, &P, &R);
      ref = T;
      refr = R;
      lin = 1.0;
      linr = 1.0;
      cur = cost(lin, linr, P);
    }
    if (trial_best < best_cost) {
      best_cost = trial_best;
      best_left = tb_left;
      best_right = tb_right;
      best_root = root;
    }
  }
  // post-order encoding of the best tree; report its tc and sc
  std::vector<int> order, st{best_root};
  while (!st.empty()) {
    const int x = st.back();
    st.pop_back();
    if (x < n) continue;
    order.push_back(x);
    st.push_back(best_left[x]);
    st.push_back(best_right[x]);
  }
  std::reverse(order.begin(), order.end());  // children before parents
  std::vector<int> slot(nn, -1);
  for (int t = 0; t < n; ++t) slot[t] = t;
  for (size_t i = 0; i < order.size(); ++i) {
    const int x = order[i];
    slot[x] = n + (int)i;
    children_out[2 * i] = slot[best_left[x]];
    children_out[2 * i + 1] = slot[best_right[x]];
  }
  if (tc_out || sc_out) {
    O.left = best_left;
    O.right = best_right;
    for (int t = 0; t < n; ++t) O.out[t] = leaf_out[t];
    double mx = -INFINITY, s = 0, msc = 0;
    for (int x : order) O.eval(x);
    for (int x : order) mx = std::max(mx, O.tc[x]);
    for (int x : order) {
      s += std::exp2(O.tc[x] - mx);
      msc = std::max(msc, O.sc[x]);
    }
    if (tc_out) *tc_out = mx + std::log2(s);
    if (sc_out) *sc_out = msc;
  }
  return OM_OK;
}
