// Binary contraction planner and the om_b200_contract entry point.
//
// Semantics follow Backend::contract / contract_with_argmax of the reference
// CPU backend (tensor4all/omeinsum-rs src/backend/cpu/contract.rs:467-671,
// 752-859): modes are classified as batch / left / right / contracted
// (classify_modes, contract.rs:11-45), labels present in one input only and
// absent from the output are reduced first (reduce_trace_modes, :309-363),
// and the result is contiguous column-major in modes_c order.  The argmax is
// the column-major linear index over the contracted modes in modes_a order.
//
// The layout plan is B200-specific rather than the reference's
// NoCopy/Permute/MakeContiguous choice (contract.rs:149-297): each mode group
// (left, right, contracted, batch) is flattened to ONE affine stride per
// operand whenever the strides allow it, in any physical order, so the GEMM
// kernels read strided views in place; only an operand whose group cannot be
// flattened is gathered (K1) into the GEMM's preferred layout, and only an
// output whose groups cannot be flattened goes through a scratch buffer and a
// permuting gather.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <set>
#include <string>
#include <vector>

#include "om_internal.h"

namespace om {
namespace {

struct Operand {
  std::vector<int32_t> modes;
  std::vector<int64_t> shape, strides;
  int pos(int32_t m) const {
    for (size_t i = 0; i < modes.size(); ++i)
      if (modes[i] == m) return (int)i;
    return -1;
  }
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

// stride of `group` flattened in `op` in the given order, or -1
int64_t flat_stride(const Operand& op, const std::vector<int32_t>& group) {
  int64_t base = -1, expect = 0;
  for (int32_t m : group) {
    int p = op.pos(m);
    if (op.shape[p] == 1) continue;
    if (base < 0) {
      base = op.strides[p];
      expect = base * op.shape[p];
      continue;
    }
    if (op.strides[p] != expect) return -1;
    expect *= op.shape[p];
  }
  return base < 0 ? 0 : base;
}

std::vector<int32_t> sorted_by_stride(const Operand& op, std::vector<int32_t> g) {
  std::stable_sort(g.begin(), g.end(), [&](int32_t x, int32_t y) {
    return op.strides[op.pos(x)] < op.strides[op.pos(y)];
  });
  return g;
}

// Picks the order of a mode group that flattens in as many of `ops` as
// possible, weighting failures by the operand's size (the cost of gathering
// it).  With `fixed`, the given order is kept.
std::vector<int32_t> choose_order(const std::vector<int32_t>& g,
                                  const std::vector<const Operand*>& ops, bool fixed) {
  if (fixed || g.size() < 2) return g;
  std::vector<std::vector<int32_t>> cands{g};
  for (auto* op : ops) cands.push_back(sorted_by_stride(*op, g));
  int64_t best_cost = -1;
  std::vector<int32_t> best = g;
  for (auto& c : cands) {
    int64_t cost = 0;
    for (auto* op : ops)
      if (flat_stride(*op, c) < 0) cost += op->numel();
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = c;
    }
  }
  return best;
}

int64_t group_size(const Operand& op, const std::vector<int32_t>& g) {
  int64_t s = 1;
  for (int32_t m : g) s *= op.shape[op.pos(m)];
  return s;
}

// A group that does not flatten in `op` but splits into two flattening runs
// (an inner run of k1 elements at stride s1, then the rest at stride s2),
// with k1 a multiple of 32 (a 32-wide k tile never straddles the two runs).
bool two_level(const Operand& op, const std::vector<int32_t>& g, int64_t& k1, int64_t& s1,
               int64_t& s2) {
  for (size_t p = g.size() - 1; p >= 1; --p) {
    std::vector<int32_t> in(g.begin(), g.begin() + p), out(g.begin() + p, g.end());
    const int64_t a = flat_stride(op, in), b = flat_stride(op, out);
    if (a < 0 || b < 0) continue;
    k1 = group_size(op, in);
    s1 = a;
    s2 = b;
    return k1 % 32 == 0;
  }
  return false;
}

std::vector<int64_t> contiguous_strides(const std::vector<int64_t>& shape) {
  std::vector<int64_t> st(shape.size());
  int64_t s = 1;
  for (size_t i = 0; i < shape.size(); ++i) {
    st[i] = s;
    s *= shape[i];
  }
  return st;
}

// Gathers `op` into a new contiguous buffer with axis order g0 ++ g1 ++ g2.
int gather_operand(om_backend* be, size_t es, const void* src, const Operand& op,
                   const std::vector<int32_t>& g0, const std::vector<int32_t>& g1,
                   const std::vector<int32_t>& g2, Scratch& buf, Operand& out) {
  std::vector<int32_t> order(g0);
  order.insert(order.end(), g1.begin(), g1.end());
  order.insert(order.end(), g2.begin(), g2.end());
  std::vector<int64_t> shape, strides;
  for (int32_t m : order) {
    int p = op.pos(m);
    shape.push_back(op.shape[p]);
    strides.push_back(op.strides[p]);
  }
  OM_TRY(buf.alloc(be, es * (size_t)std::max<int64_t>(op.numel(), 1)));
  OM_TRY(launch_gather(be, es, src, (int)order.size(), shape.data(), strides.data(), 0, buf.ptr));
  out.modes = order;
  out.shape = shape;
  out.strides = contiguous_strides(shape);
  return OM_OK;
}

uint64_t zero_pattern(om_algebra alg, om_dtype dt) {
  if (dt == OM_F64) {
    double v = alg == OM_MAXPLUS ? -1.7976931348623157e308 : (alg == OM_MINPLUS ? 1.7976931348623157e308 : 0.0);
    uint64_t u;
    memcpy(&u, &v, 8);
    return u;
  }
  float v = alg == OM_MAXPLUS ? -3.40282347e38f : (alg == OM_MINPLUS ? 3.40282347e38f : 0.f);
  uint32_t u;
  memcpy(&u, &v, 4);
  return u;
}

// Plans gemm_node: output modes in C's memory order (C is contiguous), the
// contracted ones in `contr` order; adjacent modes contiguous in both A and
// B merge.  False when the node exceeds the kernel's limits.
bool plan_node(const Operand& A, const Operand& B, const Operand& C,
               const std::vector<int32_t>& contr, NodeArgs& g);
bool node_fits(const Operand& A, const Operand& B, const Operand& C,
               const std::vector<int32_t>& contr) {
  NodeArgs g;
  return plan_node(A, B, C, contr, g);
}

bool plan_node(const Operand& A, const Operand& B, const Operand& C,
               const std::vector<int32_t>& contr, NodeArgs& g) {
  struct M3 {
    int64_t ext, sa, sb;
  };
  auto stride_in = [](const Operand& op, int32_t m) -> int64_t {
    int p = op.pos(m);
    return p >= 0 ? op.strides[p] : 0;
  };
  auto build = [&](const std::vector<int32_t>& modes, const Operand& ref, std::vector<M3>& out) {
    for (int32_t m : modes) {
      const int64_t e = ref.shape[ref.pos(m)];
      if (e == 1) continue;
      const int64_t sa = stride_in(A, m), sb = stride_in(B, m);
      if (!out.empty() && out.back().sa * out.back().ext == sa &&
          out.back().sb * out.back().ext == sb && out.back().ext * e < (int64_t(1) << 32)) {
        out.back().ext *= e;
        continue;
      }
      out.push_back({e, sa, sb});
    }
  };
  std::vector<M3> om, km;
  build(C.modes, C, om);
  build(contr, A, km);
  // split a long leading mode so that the tile has a row of several blocks
  if (!om.empty() && om[0].ext > 1024 && om[0].ext % 256 == 0) {
    M3 rest{om[0].ext / 256, om[0].sa * 256, om[0].sb * 256};
    om[0].ext = 256;
    om.insert(om.begin() + 1, rest);
  }
  if (om.size() > (size_t)kMaxNodeModes || km.size() > (size_t)kMaxNodeModes) return false;
  int64_t total = 1, K = 1;
  for (auto& x : om) {
    if (x.ext >= (int64_t(1) << 32)) return false;
    total *= x.ext;
  }
  for (auto& x : km) {
    if (x.ext >= (int64_t(1) << 32)) return false;
    K *= x.ext;
  }
  int nlow = 0;
  int64_t P = 1;
  while (nlow < (int)om.size() && P * om[nlow].ext <= 1024) P *= om[nlow++].ext;
  if (K >= (int64_t(1) << 32) || total / P >= (int64_t(1) << 32)) return false;
  g = NodeArgs{};
  g.K = K;
  g.total = total;
  g.P = (int32_t)P;
  g.rows = total / P;
  g.nlow = nlow;
  g.nout = (int)om.size();
  g.nk = (int)km.size();
  for (size_t j = 0; j < om.size(); ++j)
    g.out[j] = NodeMode{make_fastdiv((uint32_t)om[j].ext), om[j].sa, om[j].sb};
  for (size_t j = 0; j < km.size(); ++j)
    g.kmodes[j] = NodeMode{make_fastdiv((uint32_t)km[j].ext), km[j].sa, km[j].sb};
  return true;
}

}  // namespace

int contract_impl(om_backend* be, om_algebra alg, om_dtype dt, const void* a, Operand A,
                  const void* b, Operand B, Operand C, void* c_out, uint32_t* argmax) {
  const size_t es = dtype_size(dt);
  // ---- validation ---------------------------------------------------------
  for (const Operand* op : {&A, &B, &C}) {
    std::set<int32_t> seen(op->modes.begin(), op->modes.end());
    if (seen.size() != op->modes.size())
      return set_error(OM_ERR_SHAPE,
                       "contract: a mode repeats within one operand; take the diagonal first "
                       "(om_b200_unary), as the einsum engine's operand normalisation does");
    for (auto s : op->shape)
      if (s < 0) return set_error(OM_ERR_SHAPE, "contract: negative extent");
  }
  auto extent_of = [&](int32_t m) -> int64_t {
    int p = A.pos(m);
    if (p >= 0) return A.shape[p];
    p = B.pos(m);
    return p >= 0 ? B.shape[p] : -1;
  };
  for (size_t i = 0; i < A.modes.size(); ++i) {
    int p = B.pos(A.modes[i]);
    if (p >= 0 && B.shape[p] != A.shape[i])
      return set_error(OM_ERR_SHAPE, "contract: mode " + std::to_string(A.modes[i]) +
                                         " has different extents in A and B");
  }
  for (size_t i = 0; i < C.modes.size(); ++i) {
    int64_t e = extent_of(C.modes[i]);
    if (e < 0)
      return set_error(OM_ERR_SHAPE, "contract: output mode " + std::to_string(C.modes[i]) +
                                         " is in neither input");
    if (e != C.shape[i])
      return set_error(OM_ERR_SHAPE, "contract: shape_c disagrees with the inputs for mode " +
                                         std::to_string(C.modes[i]));
  }
  const int64_t nc = C.numel();
  if (nc == 0) return OM_OK;
  C.strides = contiguous_strides(C.shape);

  // ---- classify (contract.rs:11-45) ----------------------------------------
  std::vector<int32_t> batch, contr, lfree, rfree, ltrace, rtrace;
  for (int32_t m : A.modes) {
    bool inb = B.pos(m) >= 0, inc = C.pos(m) >= 0;
    if (inb && inc) batch.push_back(m);
    else if (inb) contr.push_back(m);
    else if (inc) lfree.push_back(m);
    else ltrace.push_back(m);
  }
  for (int32_t m : B.modes) {
    if (A.pos(m) >= 0) continue;
    if (C.pos(m) >= 0) rfree.push_back(m);
    else rtrace.push_back(m);
  }

  // empty reductions: a zero extent on a traced or contracted mode
  if (A.numel() == 0 || B.numel() == 0) {
    OM_TRY(launch_fill(be, c_out, es, nc, zero_pattern(alg, dt)));
    if (argmax) OM_TRY(launch_fill(be, argmax, 4, nc, 0));
    return OM_OK;
  }

  // ---- trace reduction (reduce_trace_modes, contract.rs:309-363) ----------
  Scratch ta, tb;
  auto reduce = [&](const void*& ptr, Operand& op, const std::vector<int32_t>& tr,
                    Scratch& buf) -> int {
    if (tr.empty()) return OM_OK;
    Operand r;
    for (size_t i = 0; i < op.modes.size(); ++i) {
      if (std::find(tr.begin(), tr.end(), op.modes[i]) != tr.end()) continue;
      r.modes.push_back(op.modes[i]);
      r.shape.push_back(op.shape[i]);
    }
    r.strides = contiguous_strides(r.shape);
    OM_TRY(buf.alloc(be, es * (size_t)std::max<int64_t>(r.numel(), 1)));
    OM_TRY(launch_unary(be, alg, dt, ptr, (int)op.modes.size(), op.modes.data(), op.shape.data(),
                        op.strides.data(), (int)r.modes.size(), r.modes.data(), r.shape.data(),
                        buf.ptr, nullptr));
    ptr = buf.ptr;
    op = r;
    return OM_OK;
  };
  OM_TRY(reduce(a, A, ltrace, ta));
  OM_TRY(reduce(b, B, rtrace, tb));

  // ---- group orders ---------------------------------------------------------
  const bool track = argmax != nullptr;
  contr = choose_order(contr, {&A, &B}, track);  // argmax index is in modes_a order
  lfree = choose_order(lfree, {&A, &C}, false);
  rfree = choose_order(rfree, {&B, &C}, false);
  batch = choose_order(batch, {&A, &B, &C}, false);

  Scratch node_a, node_b;
  // Small or heavily batched shapes (tensor-network nodes) whose operands do
  // not flatten are contracted in place (gemm_node) instead of gathered: for
  // these memory-bound nodes a gather would cost as much as the contraction.
  {
    const int64_t M0 = group_size(A, lfree), N0 = group_size(B, rfree);
    const int64_t K0 = group_size(A, contr);
    const bool small = (M0 * N0 <= 1024) || M0 < 16 || N0 < 16 || K0 <= 8;
    const bool flat = flat_stride(A, lfree) >= 0 && flat_stride(A, contr) >= 0 &&
                      flat_stride(A, batch) >= 0 && flat_stride(B, contr) >= 0 &&
                      flat_stride(B, rfree) >= 0 && flat_stride(B, batch) >= 0 &&
                      flat_stride(C, lfree) >= 0 && flat_stride(C, rfree) >= 0 &&
                      flat_stride(C, batch) >= 0;
    if (trace_on())
      fprintf(stderr, "[om trace] contract alg=%d M=%lld N=%lld K=%lld batch=%lld flat=%d small=%d argmax=%d\n",
              (int)alg, (long long)M0, (long long)N0, (long long)K0,
              (long long)group_size(A, batch), (int)flat, (int)small, (int)track);
    // The node kernel's reads coalesce when C's leading modes (8 outputs)
    // are, together with the operand's contracted modes, the operand's
    // densest modes.  An operand that is not laid out so is first gathered
    // into C's mode order (contracted modes last); for the small operand of
    // a node this costs little, for a large one it replaces scattered reads
    // by one streaming permutation.
    auto aligned = [&](const Operand& X) {
      std::vector<int32_t> lead;
      int64_t prod = 1;
      for (size_t i = 0; i < C.modes.size() && prod < 8; ++i)
        if (C.shape[i] > 1) {
          lead.push_back(C.modes[i]);
          prod *= C.shape[i];
        }
      auto in = [](const std::vector<int32_t>& v, int32_t m) {
        return std::find(v.begin(), v.end(), m) != v.end();
      };
      int remaining = 0;
      for (int32_t m : lead) remaining += X.pos(m) >= 0;
      std::vector<int> idx;
      for (size_t i = 0; i < X.modes.size(); ++i)
        if (X.shape[i] > 1) idx.push_back((int)i);
      std::stable_sort(idx.begin(), idx.end(),
                       [&](int x, int y) { return X.strides[x] < X.strides[y]; });
      int64_t expect = 1;
      for (int i : idx) {
        if (remaining == 0) break;
        if (X.strides[i] != expect) return false;
        const bool l = in(lead, X.modes[i]);
        if (!l && !in(contr, X.modes[i])) return false;
        remaining -= l;
        expect *= X.shape[i];
      }
      return true;
    };
    auto align = [&](const void*& ptr, Operand& X, Scratch& buf) -> int {
      if (aligned(X)) return OM_OK;
      std::vector<int32_t> cm, none;
      for (int32_t m : C.modes)
        if (X.pos(m) >= 0) cm.push_back(m);
      Operand g;
      OM_TRY(gather_operand(be, es, ptr, X, cm, contr, none, buf, g));
      ptr = buf.ptr;
      X = g;
      return OM_OK;
    };
    if (small && !flat && node_fits(A, B, C, contr)) {
      OM_TRY(align(a, A, node_a));
      OM_TRY(align(b, B, node_b));
    }
    NodeArgs na;
    if (small && !flat && plan_node(A, B, C, contr, na)) {
      na.alg = alg;
      na.dtype = dt;
      na.A = a;
      na.B = b;
      na.C = c_out;
      na.argmax = argmax;
      if (trace_on()) {
        fprintf(stderr, "[om trace] node total=%lld K=%lld P=%d nlow=%d out=", (long long)na.total,
                (long long)na.K, na.P, na.nlow);
        for (int j = 0; j < na.nout; ++j)
          fprintf(stderr, "%s%u:%lld:%lld", j ? "," : "", na.out[j].div.d, (long long)na.out[j].sa,
                  (long long)na.out[j].sb);
        fprintf(stderr, " k=");
        for (int j = 0; j < na.nk; ++j)
          fprintf(stderr, "%s%u:%lld:%lld", j ? "," : "", na.kmodes[j].div.d,
                  (long long)na.kmodes[j].sa, (long long)na.kmodes[j].sb);
        fprintf(stderr, "\n");
      }
      return launch_gemm_node(be, na);
    }
  }

  // Standard f32 on the tensor cores: the split pre-pass reads its operands
  // through their strides anyway, so a group (free or contracted) that does
  // not flatten in an operand but splits into two flattening runs is decoded
  // there instead of gathered.  Group orders are chosen so that C is written
  // directly and every two-level operand is still read along a unit-stride
  // axis (its free group's or its contracted group's inner run).
  struct Lv {
    int64_t n1 = 0, s1 = 0, s2 = 0;  // n1 == 0: flat (stride s1)
  };
  Lv a_row, a_k, b_row, b_k;
  bool decoded = false;
  auto level = [&](const Operand& X, const std::vector<int32_t>& g, Lv& lv) {
    lv = Lv{};
    const int64_t f = flat_stride(X, g);
    if (f >= 0) {
      lv.s1 = f;
      return true;
    }
    return g.size() >= 2 && two_level(X, g, lv.n1, lv.s1, lv.s2);
  };
  if (!track) {
    const bool need = flat_stride(A, lfree) < 0 || flat_stride(A, contr) < 0 ||
                      flat_stride(B, rfree) < 0 || flat_stride(B, contr) < 0 ||
                      flat_stride(C, lfree) < 0 || flat_stride(C, rfree) < 0;
    if (need && flat_stride(A, batch) >= 0 && flat_stride(B, batch) >= 0 &&
        flat_stride(C, batch) >= 0 &&
        tf32_takes(be, alg, dt, false, group_size(A, lfree), group_size(B, rfree),
                   group_size(A, contr), group_size(A, batch))) {
      const std::vector<std::vector<int32_t>> lc{lfree, sorted_by_stride(C, lfree),
                                                 sorted_by_stride(A, lfree)};
      const std::vector<std::vector<int32_t>> rc{rfree, sorted_by_stride(C, rfree),
                                                 sorted_by_stride(B, rfree)};
      const std::vector<std::vector<int32_t>> kc{contr, sorted_by_stride(A, contr),
                                                 sorted_by_stride(B, contr)};
      for (size_t i = 0; i < lc.size() && !decoded; ++i)
        for (size_t j = 0; j < rc.size() && !decoded; ++j)
          for (size_t k = 0; k < kc.size() && !decoded; ++k) {
            if (flat_stride(C, lc[i]) < 0 || flat_stride(C, rc[j]) < 0) continue;
            Lv ar, ak, br, bk;
            if (!level(A, lc[i], ar) || !level(A, kc[k], ak) || !level(B, rc[j], br) ||
                !level(B, kc[k], bk))
              continue;
            if (!(ar.s1 == 1 || ak.s1 == 1) || !(br.s1 == 1 || bk.s1 == 1)) continue;
            lfree = lc[i];
            rfree = rc[j];
            contr = kc[k];
            a_row = ar;
            a_k = ak;
            b_row = br;
            b_k = bk;
            decoded = true;
            if (trace_on())
              fprintf(stderr,
                      "[om trace] tf32 split decodes two levels: A rows %lld k %lld, B cols %lld "
                      "k %lld\n",
                      (long long)ar.n1, (long long)ak.n1, (long long)br.n1, (long long)bk.n1);
          }
    }
  }

  // The f64 DFMA kernel reads k two-level as well (per 16-wide slab): a
  // contracted group that does not flatten
  // in an operand but splits into two runs is decoded there instead of
  // gathered, the free groups staying flat (C may still go through the
  // output permutation).  Without argmax the contracted order may be any
  // that makes that possible.
  if (!decoded && dt != OM_U32 && !is_complex(dt) &&
      (flat_stride(A, contr) < 0 || flat_stride(B, contr) < 0) && contr.size() >= 2 &&
      flat_stride(A, lfree) >= 0 && flat_stride(B, rfree) >= 0 && flat_stride(A, batch) >= 0 &&
      flat_stride(B, batch) >= 0 && group_size(A, batch) == 1) {
    std::vector<std::vector<int32_t>> kc{contr};
    if (!track) {
      kc.push_back(sorted_by_stride(A, contr));
      kc.push_back(sorted_by_stride(B, contr));
    }
    for (size_t k = 0; k < kc.size() && !decoded; ++k) {
      Lv ak, bk;
      if (!level(A, kc[k], ak) || !level(B, kc[k], bk)) continue;
      GemmArgs t{};
      t.alg = alg;
      t.dtype = dt;
      t.M = group_size(A, lfree);
      t.N = group_size(B, rfree);
      t.K = group_size(A, contr);
      t.batch = 1;
      t.A = a;
      t.B = b;
      t.sam = flat_stride(A, lfree);
      t.sbn = flat_stride(B, rfree);
      t.sak = ak.s1;
      t.ka1 = ak.n1;
      t.sak2 = ak.s2;
      t.sbk = bk.s1;
      t.kb1 = bk.n1;
      t.sbk2 = bk.s2;
      t.argmax = argmax;
      if (!f64_dfma_takes(be, t)) continue;
      contr = kc[k];
      a_k = ak;
      b_k = bk;
      a_row = Lv{0, t.sam, 0};
      b_row = Lv{0, t.sbn, 0};
      decoded = true;
      if (trace_on())
        fprintf(stderr, "[om trace] gemm decodes two-level k: A %lld, B %lld\n", (long long)ak.n1,
                (long long)bk.n1);
    }
  }

  Scratch ga, gb;
  if (!decoded &&
      (flat_stride(A, lfree) < 0 || flat_stride(A, contr) < 0 || flat_stride(A, batch) < 0)) {
    Operand g;
    OM_TRY(gather_operand(be, es, a, A, lfree, contr, batch, ga, g));
    a = ga.ptr;
    A = g;
  }
  if (!decoded &&
      (flat_stride(B, contr) < 0 || flat_stride(B, rfree) < 0 || flat_stride(B, batch) < 0)) {
    Operand g;
    OM_TRY(gather_operand(be, es, b, B, contr, rfree, batch, gb, g));
    b = gb.ptr;
    B = g;
  }

  GemmArgs g{};
  g.alg = alg;
  g.dtype = dt;
  g.M = group_size(A, lfree);
  g.K = group_size(A, contr);
  g.N = group_size(B, rfree);
  g.batch = group_size(A, batch);
  g.A = a;
  g.sam = decoded ? a_row.s1 : flat_stride(A, lfree);
  g.sak = decoded ? a_k.s1 : flat_stride(A, contr);
  g.sab = flat_stride(A, batch);
  g.B = b;
  g.sbk = decoded ? b_k.s1 : flat_stride(B, contr);
  g.sbn = decoded ? b_row.s1 : flat_stride(B, rfree);
  g.sbb = flat_stride(B, batch);
  if (decoded) {
    g.ka1 = a_k.n1;
    g.sak2 = a_k.s2;
    g.kb1 = b_k.n1;
    g.sbk2 = b_k.s2;
    g.ma1 = a_row.n1;
    g.sam2 = a_row.s2;
    g.nb1 = b_row.n1;
    g.sbn2 = b_row.s2;
  }

  const bool c_direct =
      flat_stride(C, lfree) >= 0 && flat_stride(C, rfree) >= 0 && flat_stride(C, batch) >= 0;
  Scratch cs, as;
  if (c_direct) {
    g.C = c_out;
    g.argmax = argmax;
    g.scm = flat_stride(C, lfree);
    g.scn = flat_stride(C, rfree);
    g.scb = flat_stride(C, batch);
  } else {
    OM_TRY(cs.alloc(be, es * (size_t)nc));
    if (argmax) OM_TRY(as.alloc(be, 4 * (size_t)nc));
    g.C = cs.ptr;
    g.argmax = argmax ? (uint32_t*)as.ptr : nullptr;
    g.scm = 1;
    g.scn = g.M;
    g.scb = g.M * g.N;
  }
  OM_TRY(launch_gemm(be, g));

  if (!c_direct) {
    // scratch holds [lfree, rfree, batch]; permute into modes_c order
    std::vector<int32_t> cur(lfree);
    cur.insert(cur.end(), rfree.begin(), rfree.end());
    cur.insert(cur.end(), batch.begin(), batch.end());
    std::vector<int64_t> cur_shape;
    for (int32_t m : cur) cur_shape.push_back(C.shape[C.pos(m)]);
    std::vector<int64_t> cur_st = contiguous_strides(cur_shape);
    std::vector<int64_t> shp, st;
    for (int32_t m : C.modes) {
      int q = (int)(std::find(cur.begin(), cur.end(), m) - cur.begin());
      shp.push_back(cur_shape[q]);
      st.push_back(cur_st[q]);
    }
    OM_TRY(launch_gather(be, es, cs.ptr, (int)shp.size(), shp.data(), st.data(), 0, c_out));
    if (argmax)
      OM_TRY(launch_gather(be, 4, as.ptr, (int)shp.size(), shp.data(), st.data(), 0, argmax));
  }
  return OM_OK;
}

}  // namespace om

namespace om {
namespace {

// C = re(T[0,0]) - T[1,1] + i (T[0,1] + T[1,0]) for every output element;
// T is [2 (A part)][2 (B part)][n] column-major
template <typename R>
__global__ void complex_combine_kernel(const R* __restrict__ t, R* __restrict__ c, int64_t n) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const R* q = t + 4 * e;
    c[2 * e] = q[0] - q[3];
    c[2 * e + 1] = q[2] + q[1];
  }
}

// A complex operand seen as a real one: a leading part mode (re, im) of
// extent 2 and stride 1, every other stride doubled.
Operand real_view(const Operand& X, int32_t part) {
  Operand R;
  R.modes.push_back(part);
  R.shape.push_back(2);
  R.strides.push_back(1);
  for (size_t i = 0; i < X.modes.size(); ++i) {
    R.modes.push_back(X.modes[i]);
    R.shape.push_back(X.shape[i]);
    R.strides.push_back(2 * X.strides[i]);
  }
  return R;
}

}  // namespace

// Standard complex contraction through the real planner: with A and B as
// real operands carrying their own part mode (pa, pb), one real contraction
// gives T[pa, pb, c...] = sum_k A_pa B_pb (all four products of parts, on
// whatever real path the shape takes -- the tensor cores for f32), and a
// combine pass forms re = T00 - T11, im = T01 + T10.
int contract_complex(om_backend* be, om_algebra alg, om_dtype dt, const void* a, const Operand& A,
                     const void* b, const Operand& B, const Operand& C, void* c_out,
                     uint32_t* argmax) {
  if (alg != OM_STANDARD)
    return set_error(OM_ERR_UNSUPPORTED, "contract: complex dtypes take the Standard algebra only");
  int32_t top = 0;
  for (const Operand* op : {&A, &B, &C})
    for (auto m : op->modes) top = std::max(top, m);
  if (top > INT32_MAX - 2) return set_error(OM_ERR_INVALID, "contract: mode labels too large");
  const int32_t pa = top + 1, pb = top + 2;
  const om_dtype rt = real_part(dt);
  const size_t rs = dtype_size(rt);
  Operand RA = real_view(A, pa), RB = real_view(B, pb), RT;
  RT.modes = {pa, pb};
  RT.shape = {2, 2};
  int64_t n = 1;
  for (size_t i = 0; i < C.modes.size(); ++i) {
    RT.modes.push_back(C.modes[i]);
    RT.shape.push_back(C.shape[i]);
    n *= C.shape[i];
  }
  if (argmax && n > 0)
    OM_CUDA(cudaMemsetAsync(argmax, 0, 4 * (size_t)n, be->stream), "argmax zero");
  if (n == 0) return OM_OK;
  Scratch t;
  OM_TRY(t.alloc(be, rs * 4 * (size_t)n));
  OM_TRY(contract_impl(be, OM_STANDARD, rt, a, RA, b, RB, RT, t.ptr, nullptr));
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)be->num_sms * 8));
  ProfScope prof(be, "complex_combine");
  if (rt == OM_F32)
    complex_combine_kernel<float><<<blocks, 256, 0, be->stream>>>((const float*)t.ptr, (float*)c_out, n);
  else
    complex_combine_kernel<double><<<blocks, 256, 0, be->stream>>>((const double*)t.ptr, (double*)c_out, n);
  note_launch();
  return check_cuda(cudaGetLastError(), "complex combine launch");
}

}  // namespace om

extern "C" int om_b200_contract(om_backend* be, om_algebra alg, om_dtype dtype, const void* a,
                                int nda, const int64_t* shape_a, const int64_t* strides_a,
                                const int32_t* modes_a, const void* b, int ndb,
                                const int64_t* shape_b, const int64_t* strides_b,
                                const int32_t* modes_b, int ndc, const int64_t* shape_c,
                                const int32_t* modes_c, void* c_out, uint32_t* argmax_out) {
  using namespace om;
  if (!be || !a || !b || !c_out) return set_error(OM_ERR_INVALID, "om_b200_contract: null pointer");
  if (nda < 0 || ndb < 0 || ndc < 0 || nda > OM_MAX_DIMS || ndb > OM_MAX_DIMS || ndc > OM_MAX_DIMS)
    return set_error(OM_ERR_INVALID, "om_b200_contract: rank out of range");
  if ((nda && (!shape_a || !strides_a || !modes_a)) || (ndb && (!shape_b || !strides_b || !modes_b)) ||
      (ndc && (!shape_c || !modes_c)))
    return set_error(OM_ERR_INVALID, "om_b200_contract: null shape/stride/mode array");
  if (dtype != OM_F32 && dtype != OM_F64 && !is_complex(dtype))
    return set_error(OM_ERR_UNSUPPORTED, "om_b200_contract: dtype must be OM_F32, OM_F64, OM_C32 or OM_C64");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  Operand A, B, C;
  A.modes.assign(modes_a, modes_a + nda);
  A.shape.assign(shape_a, shape_a + nda);
  A.strides.assign(strides_a, strides_a + nda);
  B.modes.assign(modes_b, modes_b + ndb);
  B.shape.assign(shape_b, shape_b + ndb);
  B.strides.assign(strides_b, strides_b + ndb);
  C.modes.assign(modes_c, modes_c + ndc);
  C.shape.assign(shape_c, shape_c + ndc);
  if (is_complex(dtype)) return contract_complex(be, alg, dtype, a, A, b, B, C, c_out, argmax_out);
  return contract_impl(be, alg, dtype, a, A, b, B, C, c_out, argmax_out);
}
