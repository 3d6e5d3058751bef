// Einsum engine: contraction-tree walk, operand normalisation, gradient tape
// and backward, all on the device through the library's own kernels.
//
// Restates the reference's engine (tensor4all/omeinsum-rs):
//   tree walk            src/einsum/engine.rs:392-446 (execute_tree) and the
//                        tape build of src/einsum/backward.rs:535-605
//   normalisation        compute_normalized_binary_indices / normalize_binary_operand,
//                        engine.rs:515-578; normalize_tape_operand, backward.rs:607-642
//   root finalisation    finalize_tape_node, backward.rs:644-676; engine.rs:125-166
//   backward             backprop_tape_node, backward.rs:678-728:
//                        tropical binary -> argmax scatter (backward.rs:90-166),
//                        tropical unary  -> tropical_unary_backward (:213-238),
//                        Standard binary -> two contractions (:287-332),
//                        Standard unary  -> index exchange (:183-195).
// A GEMM-shaped binary node writes its output in native order (free labels
// of the left operand, free labels of the right one, batch labels), as the
// reference's value path does (contract_binary_native_order, ops.rs:122-143),
// so the GEMM writes without a permutation; a node small or batched enough
// to run thread-per-output writes in its larger operand's memory order
// instead (node_order); the root is finalised to iy.  The tape keys every
// gradient by label, so these orders change no result.
#include <algorithm>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "om_internal.h"
#include "om_semiring.cuh"

struct om_tape;

namespace om {
namespace {

// device buffer freed on the backend's stream when the last owner goes
std::shared_ptr<void> dev_alloc(om_backend* be, size_t bytes, int* rc) {
  void* p = nullptr;
  *rc = be_alloc(be, bytes ? bytes : 16, &p);
  if (*rc != OM_OK) return nullptr;
  const uint64_t id = be->id;
  return std::shared_ptr<void>(p, [be, id](void* q) { be_free(be, id, q); });
}

struct DTensor {
  std::shared_ptr<void> owner;  // null for caller-owned inputs
  const void* ptr = nullptr;
  std::vector<int64_t> shape, strides;
  std::vector<int32_t> ix;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

std::vector<int64_t> col_strides(const std::vector<int64_t>& shape) {
  std::vector<int64_t> st(shape.size());
  int64_t s = 1;
  for (size_t i = 0; i < shape.size(); ++i) {
    st[i] = s;
    s *= shape[i];
  }
  return st;
}

enum class Op { Leaf, Unary, Binary };

struct TapeNode {
  Op op;
  DTensor content;
  std::shared_ptr<void> argmax;  // u32, shaped like content (tropical)
  const uint32_t* am = nullptr;  // argmax's address (kept when a recorded tape releases memory)
  int tensor_index = -1;         // Leaf
  std::vector<int32_t> in_ix, out_ix;        // Unary
  std::vector<int32_t> left_ix, right_ix;    // Binary (out_ix too)
  int child0 = -1, child1 = -1;
};

template <typename T>
__global__ void scatter_add_kernel(const T* __restrict__ dy, const uint32_t* __restrict__ am,
                                   T* grad, int64_t n) {
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < n;
       o += (int64_t)gridDim.x * blockDim.x)
    if (dy[o] != T(0)) atomicAdd(grad + am[o], dy[o]);  // zeros change no sum
}

// ---- sparse tropical backward: the whole tape in one launch ---------------
// A small root gradient (e.g. the scalar of an optimisation problem) is
// routed down the tape as a list of element indices, one list per node, the
// values staying those of the root entries (a tropical step only moves them).
// One block walks the tape level by level from the root: an entry of a
// binary node is decoded through the node's argmax into one element of each
// child; an entry of a unary node moves to the element its argmax names; an
// entry reaching a leaf is added to the leaf's gradient (zeros skipped, as
// in the dense form).
struct SpNode {
  int kind;  // 0 leaf, 1 unary, 2 binary
  int child0, child1;
  int nc, nk;   // binary: output and contracted modes
  int off;      // binary: first record in SpMode data (nc output modes, then nk contracted)
  const uint32_t* argmax;
  void* grad;   // leaf
  // tapes kept without argmax (om_b200_einsum_tape_values): the argmax of a
  // visited element is found from the children's values instead
  int lazy;
  const void* xa;  // binary: left child's values; unary: the input's values
  const void* xb;  // binary: right child's values
  int64_t aux;     // unary: first word of its descriptor in the aux array
  int64_t kext;    // binary: number of contracted index values
};
struct SpMode {
  int64_t ext, sa, sb;  // extent; element stride in the left / right child (0 if absent)
  int64_t da, db;       // the same in the children's memory (their value strides)
  FastDiv fd;           // division by ext (extents below 2^32)
};

template <typename T>
__global__ void __launch_bounds__(512) sparse_backward_kernel(const SpNode* __restrict__ nodes,
                                                              const SpMode* __restrict__ modes,
                                                              const int* __restrict__ level_start,
                                                              int nlevels, int root, int64_t* lists,
                                                              const T* __restrict__ val, int64_t n) {
  for (int64_t e = threadIdx.x; e < n; e += blockDim.x) lists[(int64_t)root * n + e] = e;
  __syncthreads();
  for (int L = 0; L < nlevels; ++L) {
    const int first = level_start[L];
    const int64_t items = (int64_t)(level_start[L + 1] - first) * n;
    for (int64_t it = threadIdx.x; it < items; it += blockDim.x) {
      const int id = first + (int)(it / n);
      const int64_t e = it % n;
      const SpNode nd = nodes[id];
      const int64_t o = lists[(int64_t)id * n + e];
      if (nd.kind == 0) {
        const T v = val[e];
        if (v != T(0)) atomicAdd((T*)nd.grad + o, v);
      } else if (nd.kind == 1) {  // unary, or a link into another tape (no argmax)
        lists[(int64_t)nd.child0 * n + e] = nd.argmax ? (int64_t)nd.argmax[o] : o;
      } else {
        int64_t pa = 0, pb = 0, rem = o;
        const SpMode* m = modes + nd.off;
        for (int k = 0; k < nd.nc; ++k) {
          const int64_t c = rem % m[k].ext;
          rem /= m[k].ext;
          pa += c * m[k].sa;
          pb += c * m[k].sb;
        }
        int64_t w = nd.argmax[o];
        for (int k = nd.nc; k < nd.nc + nd.nk; ++k) {
          const int64_t c = w % m[k].ext;
          w /= m[k].ext;
          pa += c * m[k].sa;
          pb += c * m[k].sb;
        }
        lists[(int64_t)nd.child0 * n + e] = pa;
        lists[(int64_t)nd.child1 * n + e] = pb;
      }
    }
    __syncthreads();
  }
}

// The same walk over tapes kept without argmax: a warp per entry.  The
// argmax of a binary node's entry is recomputed from the children's values
// with the rule of generic_gemm_with_argmax (start at zero(), replace on
// strict improvement, so the first k reaching the maximum wins); the lanes
// split k and merge (better value, then smaller k).  A NaN product breaks
// that merge (the sequential rule lets a NaN replace and be replaced), so a
// node entry that meets one is rescanned sequentially by lane 0.  A unary
// node's entry follows execute_unary_with_argmax (first inner element, then
// strict improvement; the winner's column-major position in the input).
// Unary descriptor words in aux: nx, ny, ninner, nslots, xslot[nx],
// xstride[nx], xlogical[nx], yslot[ny], ysize[ny], islot[ninner],
// isize[ninner].
// binary entries with more contracted index values than this take the whole
// block instead of one warp
constexpr int64_t kLazyBlockK = 4096;
constexpr int kLazyBigQueue = 256;  // such entries per level held in shared memory

template <typename T, int ALG>
__device__ __forceinline__ void lazy_better(T v, int64_t k, T& best, int64_t& bk) {
  if (Semi<ALG, T>::better(v, best) || (v == best && k < bk)) {
    best = v;
    bk = k;
  }
}

template <typename T, int ALG>
__global__ void __launch_bounds__(1024) sparse_backward_lazy_kernel(
    const SpNode* __restrict__ nodes, const SpMode* __restrict__ modes,
    const int64_t* __restrict__ aux, const int* __restrict__ level_start, int nlevels, int root,
    int64_t* lists, const T* __restrict__ val, int64_t n) {
  using S = Semi<ALG, T>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  __shared__ T bbest[32];
  __shared__ int64_t bkk[32];
  __shared__ bool bnan[32];
  __shared__ int64_t big[kLazyBigQueue];
  __shared__ int nbig, big_overflow;
  for (int64_t e = threadIdx.x; e < n; e += blockDim.x) lists[(int64_t)root * n + e] = e;
  __syncthreads();
  for (int L = 0; L < nlevels; ++L) {
    const int first = level_start[L];
    const int64_t items = (int64_t)(level_start[L + 1] - first) * n;
    if (threadIdx.x == 0) {
      nbig = 0;
      big_overflow = 0;
    }
    __syncthreads();
    for (int64_t it = warp; it < items; it += nwarps) {
      const int id = first + (int)(it / n);
      const int64_t e = it % n;
      const SpNode nd = nodes[id];
      const int64_t o = lists[(int64_t)id * n + e];
      if (nd.kind == 0) {
        if (lane == 0) {
          const T v = val[e];
          if (v != T(0)) atomicAdd((T*)nd.grad + o, v);
        }
      } else if (nd.kind == 1 && !nd.lazy) {
        if (lane == 0) lists[(int64_t)nd.child0 * n + e] = nd.argmax ? (int64_t)nd.argmax[o] : o;
      } else if (nd.kind == 1) {
        const int64_t* d = aux + nd.aux;
        const int nx = (int)d[0], ny = (int)d[1], ni = (int)d[2], ns = (int)d[3];
        const int64_t *xslot = d + 4, *xstride = xslot + nx, *xlog = xstride + nx;
        const int64_t *yslot = xlog + nx, *ysize = yslot + ny, *islot = ysize + ny,
                      *isize = islot + ni;
        int64_t v_[OM_MAX_DIMS];
        bool set[OM_MAX_DIMS];
        for (int q = 0; q < ns; ++q) set[q] = false;
        int64_t rem = o;
        bool skip = false;
        for (int q = 0; q < ny; ++q) {
          const int64_t c = rem % ysize[q];
          rem /= ysize[q];
          const int sl = (int)yslot[q];
          if (set[sl] && v_[sl] != c) skip = true;
          set[sl] = true;
          v_[sl] = c;
        }
        int64_t inner = 1;
        for (int q = 0; q < ni; ++q) inner *= isize[q];
        const T* X = (const T*)nd.xa;
        T best = T(0);
        int64_t bk = INT64_MAX, bpos = 0;
        bool first_nan = false;
        if (!skip) {
          for (int64_t in = lane; in < inner; in += 32) {
            int64_t r2 = in;
            for (int q = 0; q < ni; ++q) {
              v_[islot[q]] = r2 % isize[q];
              r2 /= isize[q];
            }
            int64_t off = 0, lpos = 0;
            for (int q = 0; q < nx; ++q) {
              off += v_[xslot[q]] * xstride[q];
              lpos += v_[xslot[q]] * xlog[q];
            }
            const T x = X[off];
            if (in == 0) first_nan = x != x;
            if (x == x && (bk == INT64_MAX || S::better(x, best) || (x == best && in < bk))) {
              best = x;
              bk = in;
              bpos = lpos;
            }
          }
        }
        // merge: better value, then earlier inner position; a NaN first
        // element keeps position 0 (nothing is strictly better than NaN)
        for (int sh = 16; sh; sh >>= 1) {
          const T ob = __shfl_xor_sync(0xffffffffu, best, sh);
          const int64_t ok = __shfl_xor_sync(0xffffffffu, bk, sh);
          const int64_t op = __shfl_xor_sync(0xffffffffu, bpos, sh);
          if (ok != INT64_MAX && (bk == INT64_MAX || S::better(ob, best) || (ob == best && ok < bk))) {
            best = ob;
            bk = ok;
            bpos = op;
          }
        }
        first_nan = __shfl_sync(0xffffffffu, first_nan, 0);
        if (lane == 0) lists[(int64_t)nd.child0 * n + e] = (skip || first_nan || bk == INT64_MAX) ? 0 : bpos;
      } else if (nd.lazy && !nd.argmax && nd.kext > kLazyBlockK) {
        // a long contracted range: queued for the whole block below
        if (lane == 0) {
          const int at = atomicAdd(&nbig, 1);
          if (at < kLazyBigQueue) big[at] = it;
          else big_overflow = 1;
        }
        continue;
      } else {
        const SpMode* m = modes + nd.off;
        int64_t pa = 0, pb = 0, qa = 0, qb = 0, rem = o;
        for (int k = 0; k < nd.nc; ++k) {
          const int64_t c = rem % m[k].ext;
          rem /= m[k].ext;
          pa += c * m[k].sa;
          pb += c * m[k].sb;
          qa += c * m[k].da;
          qb += c * m[k].db;
        }
        int64_t w = 0;
        if (nd.argmax) {
          w = nd.argmax[o];
        } else {
          int64_t K = 1;
          for (int k = nd.nc; k < nd.nc + nd.nk; ++k) K *= m[k].ext;
          const T* A = (const T*)nd.xa;
          const T* B = (const T*)nd.xb;
          auto prod = [&](int64_t kk) {
            int64_t ra = qa, rb = qb;
            uint32_t r = (uint32_t)kk;  // contracted ranges stay below 2^32
            for (int k = nd.nc; k < nd.nc + nd.nk; ++k) {
              const uint32_t q = fast_div(r, m[k].fd);
              const int64_t c = (int64_t)(r - q * m[k].fd.d);
              r = q;
              ra += c * m[k].da;
              rb += c * m[k].db;
            }
            return S::mul(A[ra], B[rb]);
          };
          T best = S::zero();
          int64_t bk = INT64_MAX;
          bool nan = false;
          for (int64_t kk = lane; kk < K; kk += 32) {
            const T p = prod(kk);
            nan |= p != p;
            if (S::better(p, best)) {
              best = p;
              bk = kk;
            }
          }
          for (int sh = 16; sh; sh >>= 1) {
            const T ob = __shfl_xor_sync(0xffffffffu, best, sh);
            const int64_t ok = __shfl_xor_sync(0xffffffffu, bk, sh);
            lazy_better<T, ALG>(ob, ok, best, bk);
          }
          w = bk == INT64_MAX ? 0 : bk;
          if (__any_sync(0xffffffffu, nan)) {  // the sequential rule, as in the forward
            if (lane == 0) {
              T acc = S::zero();
              int64_t idx = 0;
              for (int64_t kk = 0; kk < K; ++kk) {
                const T p = prod(kk);
                if (!S::keep(acc, p)) {
                  acc = p;
                  idx = kk;
                }
              }
              w = idx;
            }
          }
          w = __shfl_sync(0xffffffffu, w, 0);
        }
        if (lane == 0) {
          for (int k = nd.nc; k < nd.nc + nd.nk; ++k) {
            const int64_t c = w % m[k].ext;
            w /= m[k].ext;
            pa += c * m[k].sa;
            pb += c * m[k].sb;
          }
          lists[(int64_t)nd.child0 * n + e] = pa;
          lists[(int64_t)nd.child1 * n + e] = pb;
        }
      }
    }
    __syncthreads();
    // entries of binary nodes with a long contracted range: one at a time,
    // the k range split over the whole block, merged as above (the queue
    // filled above; on overflow every entry of the level is looked at)
    const int nq = big_overflow ? (int)items : min(nbig, kLazyBigQueue);
    for (int qi = 0; qi < nq; ++qi) {
      const int64_t it = big_overflow ? qi : big[qi];
      const int id = first + (int)(it / n);
      const SpNode nd = nodes[id];
      if (!(nd.kind == 2 && nd.lazy && !nd.argmax && nd.kext > kLazyBlockK)) continue;
      const int64_t e = it % n;
      const int64_t o = lists[(int64_t)id * n + e];
      const SpMode* m = modes + nd.off;
      int64_t pa = 0, pb = 0, qa = 0, qb = 0, rem = o;
      for (int k = 0; k < nd.nc; ++k) {
        const int64_t c = rem % m[k].ext;
        rem /= m[k].ext;
        pa += c * m[k].sa;
        pb += c * m[k].sb;
        qa += c * m[k].da;
        qb += c * m[k].db;
      }
      const T* A = (const T*)nd.xa;
      const T* B = (const T*)nd.xb;
      auto prod = [&](int64_t kk) {
        int64_t ra = qa, rb = qb;
        uint32_t r = (uint32_t)kk;
        for (int k = nd.nc; k < nd.nc + nd.nk; ++k) {
          const uint32_t q = fast_div(r, m[k].fd);
          const int64_t c = (int64_t)(r - q * m[k].fd.d);
          r = q;
          ra += c * m[k].da;
          rb += c * m[k].db;
        }
        return S::mul(A[ra], B[rb]);
      };
      T best = S::zero();
      int64_t bk = INT64_MAX;
      bool nan = false;
      for (int64_t kk = threadIdx.x; kk < nd.kext; kk += blockDim.x) {
        const T p = prod(kk);
        nan |= p != p;
        if (S::better(p, best)) {
          best = p;
          bk = kk;
        }
      }
      for (int sh = 16; sh; sh >>= 1) {
        const T ob = __shfl_xor_sync(0xffffffffu, best, sh);
        const int64_t ok = __shfl_xor_sync(0xffffffffu, bk, sh);
        lazy_better<T, ALG>(ob, ok, best, bk);
      }
      nan = __any_sync(0xffffffffu, nan);
      if (lane == 0) {
        bbest[warp] = best;
        bkk[warp] = bk;
        bnan[warp] = nan;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        bool any_nan = false;
        for (int q = 0; q < nwarps; ++q) {
          if (q) lazy_better<T, ALG>(bbest[q], bkk[q], best, bk);
          any_nan |= bnan[q];
        }
        int64_t w = bk == INT64_MAX ? 0 : bk;
        if (any_nan) {  // the sequential rule, as in the forward
          T acc = S::zero();
          w = 0;
          for (int64_t kk = 0; kk < nd.kext; ++kk) {
            const T p = prod(kk);
            if (!S::keep(acc, p)) {
              acc = p;
              w = kk;
            }
          }
        }
        for (int k = nd.nc; k < nd.nc + nd.nk; ++k) {
          const int64_t c = w % m[k].ext;
          w /= m[k].ext;
          pa += c * m[k].sa;
          pb += c * m[k].sb;
        }
        lists[(int64_t)nd.child0 * n + e] = pa;
        lists[(int64_t)nd.child1 * n + e] = pb;
      }
      __syncthreads();
    }
  }
}

template <typename T>
__global__ void zero_many_kernel(T* const* ptrs, const int64_t* sizes, int count) {
  for (int q = blockIdx.x; q < count; q += gridDim.x)
    for (int64_t i = threadIdx.x; i < sizes[q]; i += blockDim.x) ptrs[q][i] = T(0);
}

// Root gradients with at most this many elements take the sparse path.
constexpr int64_t kSparseGradMax = 4096;

}  // namespace

struct Engine {
  om_backend* be;
  om_algebra alg;
  om_dtype dt;
  size_t es;
  bool tropical;
  std::map<int32_t, int64_t> sizes;
  std::vector<TapeNode> nodes;
  std::vector<std::vector<int64_t>> input_shapes;
  int root = -1;
  bool keep;  // tape mode (argmax for tropical)
  bool lazy = false;  // tropical tape kept without argmax (values only)

  int64_t extent(int32_t l) const {
    auto it = sizes.find(l);
    return it == sizes.end() ? -1 : it->second;
  }

  int new_tensor(const std::vector<int32_t>& ix, DTensor& t) {
    t.ix = ix;
    t.shape.clear();
    for (auto l : ix) {
      int64_t e = extent(l);
      if (e < 0) return set_error(OM_ERR_SHAPE, "einsum: label " + std::to_string(l) + " has no size");
      t.shape.push_back(e);
    }
    t.strides = col_strides(t.shape);
    int rc;
    t.owner = dev_alloc(be, es * (size_t)std::max<int64_t>(t.numel(), 1), &rc);
    t.ptr = t.owner.get();
    return rc;
  }

  // execute_unary_naive / execute_unary_with_argmax into a new tensor
  int unary(const DTensor& x, const std::vector<int32_t>& oix, bool with_argmax, DTensor& y,
            std::shared_ptr<void>& am) {
    OM_TRY(new_tensor(oix, y));
    uint32_t* amp = nullptr;
    if (with_argmax) {
      int rc;
      am = dev_alloc(be, 4 * (size_t)std::max<int64_t>(y.numel(), 1), &rc);
      OM_TRY(rc);
      amp = (uint32_t*)am.get();
    }
    return launch_unary(be, alg, dt, x.ptr, (int)x.ix.size(), x.ix.data(), x.shape.data(),
                        x.strides.data(), (int)oix.size(), oix.data(), y.shape.data(),
                        (void*)y.ptr, amp);
  }

  int contract(const DTensor& a, const std::vector<int32_t>& ia, const DTensor& b,
               const std::vector<int32_t>& ib, const std::vector<int32_t>& iy, bool with_argmax,
               DTensor& c, std::shared_ptr<void>& am) {
    OM_TRY(new_tensor(iy, c));
    uint32_t* amp = nullptr;
    if (with_argmax) {
      int rc;
      am = dev_alloc(be, 4 * (size_t)std::max<int64_t>(c.numel(), 1), &rc);
      OM_TRY(rc);
      amp = (uint32_t*)am.get();
    }
    return om_b200_contract(be, alg, dt, a.ptr, (int)ia.size(), a.shape.data(), a.strides.data(),
                            ia.data(), b.ptr, (int)ib.size(), b.shape.data(), b.strides.data(),
                            ib.data(), (int)iy.size(), c.shape.data(), iy.data(), (void*)c.ptr, amp);
  }

  // compute_normalized_binary_indices (engine.rs:515-535)
  static std::vector<int32_t> normalized(const std::vector<int32_t>& ix,
                                         const std::vector<int32_t>& other,
                                         const std::vector<int32_t>& out) {
    std::vector<int32_t> r;
    for (auto l : ix) {
      bool keep = std::find(other.begin(), other.end(), l) != other.end() ||
                  std::find(out.begin(), out.end(), l) != out.end();
      if (keep && std::find(r.begin(), r.end(), l) == r.end()) r.push_back(l);
    }
    return r;
  }

  // native_binary_output_indices (src/tensor/ops.rs:12-35): free labels of
  // A, then free labels of B, then batch labels -- the order the GEMM writes
  // without a permutation; falls back to the node's own order if that does
  // not cover it
  static std::vector<int32_t> native_order(const std::vector<int32_t>& ia,
                                           const std::vector<int32_t>& ib,
                                           const std::vector<int32_t>& iy) {
    auto has = [](const std::vector<int32_t>& v, int32_t l) {
      return std::find(v.begin(), v.end(), l) != v.end();
    };
    std::vector<int32_t> r;
    for (auto l : ia)
      if (has(iy, l) && !has(ib, l) && !has(r, l)) r.push_back(l);
    for (auto l : ib)
      if (has(iy, l) && !has(ia, l) && !has(r, l)) r.push_back(l);
    for (auto l : ia)
      if (has(iy, l) && has(ib, l) && !has(r, l)) r.push_back(l);
    return r.size() == iy.size() ? r : iy;
  }

  // Output order of a node that runs as a thread-per-output contraction
  // (small M*N, M or N below 16, or k of at most 8): the free and batch
  // labels of the larger operand in its memory order, then the rest in the
  // other operand's memory order.  The node then streams its larger input
  // and its output in the same order, both coalesced, and the next node
  // inherits the layout.  Larger nodes keep native_order (the GEMM's).
  std::vector<int32_t> node_order(const DTensor& a, const DTensor& b,
                                  const std::vector<int32_t>& iy) const {
    auto pos = [](const std::vector<int32_t>& v, int32_t l) -> int {
      for (size_t i = 0; i < v.size(); ++i)
        if (v[i] == l) return (int)i;
      return -1;
    };
    int64_t M = 1, N = 1, K = 1;
    for (size_t i = 0; i < a.ix.size(); ++i) {
      const bool inb = pos(b.ix, a.ix[i]) >= 0, iny = pos(iy, a.ix[i]) >= 0;
      if (iny && !inb) M *= a.shape[i];
      if (inb && !iny) K *= a.shape[i];
    }
    for (size_t i = 0; i < b.ix.size(); ++i)
      if (pos(iy, b.ix[i]) >= 0 && pos(a.ix, b.ix[i]) < 0) N *= b.shape[i];
    const bool small = M * N <= 1024 || M < 16 || N < 16 || K <= 8;
    if (!small) return native_order(a.ix, b.ix, iy);
    const DTensor& big = a.numel() >= b.numel() ? a : b;
    const DTensor& other = &big == &a ? b : a;
    std::vector<int32_t> r;
    for (const DTensor* t : {&big, &other}) {
      std::vector<int> idx;
      for (size_t i = 0; i < t->ix.size(); ++i)
        if (pos(iy, t->ix[i]) >= 0 && pos(r, t->ix[i]) < 0) idx.push_back((int)i);
      std::stable_sort(idx.begin(), idx.end(),
                       [&](int x, int y) { return t->strides[x] < t->strides[y]; });
      for (int i : idx) r.push_back(t->ix[i]);
    }
    return r.size() == iy.size() ? r : native_order(a.ix, b.ix, iy);
  }

  int push_unary(int child, const std::vector<int32_t>& oix, int* out_node) {
    TapeNode n;
    n.op = Op::Unary;
    n.in_ix = nodes[child].content.ix;
    n.out_ix = oix;
    n.child0 = child;
    OM_TRY(unary(nodes[child].content, oix, keep && tropical && !lazy, n.content, n.argmax));
    n.am = (const uint32_t*)n.argmax.get();
    nodes.push_back(std::move(n));
    *out_node = (int)nodes.size() - 1;
    return OM_OK;
  }

  int normalize(int node, const std::vector<int32_t>& other, const std::vector<int32_t>& out,
                int* out_node) {
    auto nix = normalized(nodes[node].content.ix, other, out);
    if (nix == nodes[node].content.ix) {
      *out_node = node;
      return OM_OK;
    }
    return push_unary(node, nix, out_node);
  }

  // descriptor words of a unary node for the lazy backward walk (the same
  // label analysis as launch_unary: slots per distinct label, inner labels =
  // labels of x absent from the output, first occurrence order)
  static int unary_aux(const DTensor& x, const std::vector<int32_t>& oix,
                       const std::vector<int64_t>& osize, std::vector<int64_t>& aux) {
    std::vector<int32_t> slots;
    auto slot_of = [&](int32_t l) -> int64_t {
      for (size_t i = 0; i < slots.size(); ++i)
        if (slots[i] == l) return (int64_t)i;
      slots.push_back(l);
      return (int64_t)slots.size() - 1;
    };
    const int nx = (int)x.ix.size(), ny = (int)oix.size();
    std::vector<int64_t> xs, xst, xl, ys, yz, is, iz;
    int64_t lg = 1;
    for (int q = 0; q < nx; ++q) {
      xs.push_back(slot_of(x.ix[q]));
      xst.push_back(x.strides[q]);
      xl.push_back(lg);
      lg *= x.shape[q];
    }
    for (int q = 0; q < ny; ++q) {
      ys.push_back(slot_of(oix[q]));
      yz.push_back(osize[q]);
    }
    for (int q = 0; q < nx; ++q) {
      const bool in_y = std::find(oix.begin(), oix.end(), x.ix[q]) != oix.end();
      const bool seen = std::find(is.begin(), is.end(), xs[q]) != is.end();
      if (in_y || seen) continue;
      is.push_back(xs[q]);
      iz.push_back(x.shape[q]);
    }
    if ((int)slots.size() > OM_MAX_DIMS) return set_error(OM_ERR_INVALID, "lazy unary: too many labels");
    for (int64_t w : {(int64_t)nx, (int64_t)ny, (int64_t)is.size(), (int64_t)slots.size()}) aux.push_back(w);
    for (auto* v : {&xs, &xst, &xl, &ys, &yz, &is, &iz}) aux.insert(aux.end(), v->begin(), v->end());
    return OM_OK;
  }

  int backprop(int idx, const DTensor& dy, void* const* grads);
  int backprop_sparse(const void* dy, void* const* grads);
  // the same walk over this tape and, through the leaves named in `link`
  // (leaf tensor index -> tape), over further tapes whose roots are those
  // leaves' contents; grads of tape k go to egrads[k]
  int backprop_sparse_linked(const void* dy, const std::vector<const Engine*>& engines,
                             const std::vector<void* const*>& egrads,
                             const std::map<int, int>& link);
};

// Tropical backward for a small root gradient: the tape is laid out level
// by level from the root and walked by sparse_backward_kernel in one launch.
int Engine::backprop_sparse(const void* dy, void* const* grads) {
  return backprop_sparse_linked(dy, {this}, {grads}, {});
}

int Engine::backprop_sparse_linked(const void* dy, const std::vector<const Engine*>& engines,
                                   const std::vector<void* const*>& egrads,
                                   const std::map<int, int>& link) {
  const int64_t n = nodes[root].content.numel();
  // breadth-first over (tape, node) from this tape's root
  std::vector<std::pair<int, int>> order{{0, root}};
  std::vector<std::vector<int>> slots(engines.size());
  for (size_t k = 0; k < engines.size(); ++k) slots[k].assign(engines[k]->nodes.size(), -1);
  slots[0][root] = 0;
  std::vector<int> level_start{0};
  auto visit = [&](int k, int c) {
    if (c >= 0 && slots[k][c] < 0) {
      slots[k][c] = (int)order.size();
      order.push_back({k, c});
    }
  };
  for (size_t head = 0; head < order.size();) {
    const size_t end = order.size();
    level_start.push_back((int)end);
    for (; head < end; ++head) {
      const int k = order[head].first;
      const TapeNode& t = engines[k]->nodes[order[head].second];
      if (t.op == Op::Leaf) {
        auto it = k == 0 ? link.find(t.tensor_index) : link.end();
        if (it != link.end()) visit(it->second, engines[it->second]->root);
        continue;
      }
      visit(k, t.child0);
      visit(k, t.child1);
    }
    if (order.size() == end) break;
  }
  if (level_start.back() != (int)order.size()) level_start.push_back((int)order.size());
  while (level_start.size() >= 2 && level_start[level_start.size() - 2] == level_start.back())
    level_start.pop_back();
  std::vector<SpNode> recs(order.size());
  std::vector<SpMode> modes;
  std::vector<int64_t> aux;
  bool any_lazy = false;
  std::vector<void*> zptr;
  std::vector<int64_t> zsize;
  for (size_t q = 0; q < order.size(); ++q) {
    const int k = order[q].first;
    const auto& enodes = engines[k]->nodes;
    const TapeNode& t = enodes[order[q].second];
    const std::vector<int>& slot = slots[k];
    SpNode r{};
    auto lk = (k == 0 && t.op == Op::Leaf) ? link.find(t.tensor_index) : link.end();
    if (lk != link.end()) {
      r.kind = 1;  // identity into the linked tape's root
      r.child0 = slots[lk->second][engines[lk->second]->root];
      r.argmax = nullptr;
    } else if (t.op == Op::Leaf) {
      r.kind = 0;
      r.grad = egrads[k][t.tensor_index];
      zptr.push_back(r.grad);
      zsize.push_back(t.content.numel());
    } else if (t.op == Op::Unary) {
      r.kind = 1;
      r.child0 = slot[t.child0];
      r.argmax = t.am;
      if (!t.am && engines[k]->lazy) {
        r.lazy = 1;
        any_lazy = true;
        const DTensor& x = enodes[t.child0].content;
        r.xa = x.ptr;
        r.aux = (int64_t)aux.size();
        OM_TRY(unary_aux(x, t.out_ix, t.content.shape, aux));
      }
    } else {
      r.kind = 2;
      r.child0 = slot[t.child0];
      r.child1 = slot[t.child1];
      r.argmax = t.am;
      r.off = (int)modes.size();
      const DTensor& l = enodes[t.child0].content;
      const DTensor& rr = enodes[t.child1].content;
      auto stride_in = [](const std::vector<int32_t>& ix, const std::vector<int64_t>& shape,
                          int32_t lab) -> int64_t {
        int64_t s = 1;
        for (size_t i = 0; i < ix.size(); ++i) {
          if (ix[i] == lab) return s;
          s *= shape[i];
        }
        return 0;
      };
      const DTensor& c = t.content;
      // element strides of a label in a child's memory (0 if absent)
      auto data_in = [](const DTensor& x, int32_t lab) -> int64_t {
        for (size_t i = 0; i < x.ix.size(); ++i)
          if (x.ix[i] == lab) return x.strides[i];
        return 0;
      };
      if (!t.am && engines[k]->lazy) {
        r.lazy = 1;
        any_lazy = true;
        r.xa = l.ptr;
        r.xb = rr.ptr;
      }
      for (size_t k = 0; k < t.out_ix.size(); ++k)
        modes.push_back({c.shape[k], stride_in(t.left_ix, l.shape, t.out_ix[k]),
                         stride_in(t.right_ix, rr.shape, t.out_ix[k]), data_in(l, t.out_ix[k]),
                         data_in(rr, t.out_ix[k]), make_fastdiv((uint32_t)c.shape[k])});
      r.nc = (int)t.out_ix.size();
      r.kext = 1;
      // contracted labels in left_ix order: the argmax's column-major digits
      for (size_t k = 0; k < t.left_ix.size(); ++k) {
        const int32_t lab = t.left_ix[k];
        const bool in_r = std::find(t.right_ix.begin(), t.right_ix.end(), lab) != t.right_ix.end();
        const bool in_c = std::find(t.out_ix.begin(), t.out_ix.end(), lab) != t.out_ix.end();
        if (in_r && !in_c) {
          modes.push_back({l.shape[k], stride_in(t.left_ix, l.shape, lab),
                           stride_in(t.right_ix, rr.shape, lab), data_in(l, lab), data_in(rr, lab),
                           make_fastdiv((uint32_t)l.shape[k])});
          r.nk++;
          r.kext *= l.shape[k];
        }
      }
    }
    recs[q] = r;
  }
  int rc;
  for (const SpNode& r : recs)
    if (r.lazy && r.kind == 2 && r.kext >= (int64_t(1) << 32))
      return set_error(OM_ERR_UNSUPPORTED, "values-only backward: a contracted range of 2^32 or more");
  const size_t b_nodes = sizeof(SpNode) * recs.size(), b_modes = sizeof(SpMode) * modes.size();
  const size_t b_aux = 8 * aux.size();
  const size_t b_levels = sizeof(int) * level_start.size(), b_lists = 8 * order.size() * (size_t)n;
  const size_t b_z = (sizeof(void*) + 8) * zptr.size();
  auto buf = dev_alloc(be, b_nodes + b_modes + b_aux + b_levels + b_z + b_lists + 64, &rc);
  OM_TRY(rc);
  char* base = (char*)buf.get();
  SpNode* d_nodes = (SpNode*)base;
  SpMode* d_modes = (SpMode*)(base + b_nodes);
  int64_t* d_aux = (int64_t*)(base + b_nodes + b_modes);
  int* d_levels = (int*)(base + b_nodes + b_modes + b_aux);
  const size_t b_head = b_nodes + b_modes + b_aux + b_levels;
  void** d_zptr = (void**)(((uintptr_t)(base + b_head) + 15) & ~(uintptr_t)15);
  int64_t* d_zsize = (int64_t*)(d_zptr + zptr.size());
  int64_t* d_lists = (int64_t*)(((uintptr_t)(d_zsize + zsize.size()) + 15) & ~(uintptr_t)15);
  std::vector<char> host(b_head);
  memcpy(host.data(), recs.data(), b_nodes);
  if (b_modes) memcpy(host.data() + b_nodes, modes.data(), b_modes);
  if (b_aux) memcpy(host.data() + b_nodes + b_modes, aux.data(), b_aux);
  memcpy(host.data() + b_nodes + b_modes + b_aux, level_start.data(), b_levels);
  OM_CUDA(cudaMemcpyAsync(base, host.data(), host.size(), cudaMemcpyHostToDevice, be->stream),
          "sparse backward upload");
  if (!zptr.empty()) {
    OM_CUDA(cudaMemcpyAsync(d_zptr, zptr.data(), sizeof(void*) * zptr.size(), cudaMemcpyHostToDevice,
                            be->stream),
            "sparse backward upload");
    OM_CUDA(cudaMemcpyAsync(d_zsize, zsize.data(), 8 * zsize.size(), cudaMemcpyHostToDevice,
                            be->stream),
            "sparse backward upload");
  }
  auto val = dev_alloc(be, es * (size_t)std::max<int64_t>(n, 1), &rc);
  OM_TRY(rc);
  OM_CUDA(cudaMemcpyAsync(val.get(), dy, es * (size_t)n, cudaMemcpyDeviceToDevice, be->stream),
          "grad copy");
  ProfScope prof(be, any_lazy ? "sparse_backward_lazy" : "sparse_backward");
  const int nz = (int)zptr.size();
  const int nlev = (int)level_start.size() - 1;
  if (dt == OM_F32) {
    if (nz) zero_many_kernel<float><<<std::min(nz, be->num_sms * 4), 256, 0, be->stream>>>(
        (float* const*)d_zptr, d_zsize, nz);
  } else {
    if (nz) zero_many_kernel<double><<<std::min(nz, be->num_sms * 4), 256, 0, be->stream>>>(
        (double* const*)d_zptr, d_zsize, nz);
  }
#define OM_LAZY(T, A)                                                                     \
  sparse_backward_lazy_kernel<T, A><<<1, 1024, 0, be->stream>>>(d_nodes, d_modes, d_aux, d_levels, \
                                                               nlev, 0, d_lists,             \
                                                               (const T*)val.get(), n)
  if (any_lazy) {
    if (dt == OM_F32) {
      if (alg == OM_MAXPLUS) OM_LAZY(float, OM_MAXPLUS);
      else if (alg == OM_MINPLUS) OM_LAZY(float, OM_MINPLUS);
      else OM_LAZY(float, OM_MAXMUL);
    } else {
      if (alg == OM_MAXPLUS) OM_LAZY(double, OM_MAXPLUS);
      else if (alg == OM_MINPLUS) OM_LAZY(double, OM_MINPLUS);
      else OM_LAZY(double, OM_MAXMUL);
    }
  } else if (dt == OM_F32) {
    sparse_backward_kernel<float><<<1, 512, 0, be->stream>>>(d_nodes, d_modes, d_levels, nlev, 0,
                                                             d_lists, (const float*)val.get(), n);
  } else {
    sparse_backward_kernel<double><<<1, 512, 0, be->stream>>>(d_nodes, d_modes, d_levels, nlev, 0,
                                                              d_lists, (const double*)val.get(), n);
  }
#undef OM_LAZY
  note_launch(nz ? 2 : 1);
  return check_cuda(cudaGetLastError(), "sparse backward launch");
}

int Engine::backprop(int idx, const DTensor& dy, void* const* grads) {
  TapeNode& n = nodes[idx];
  if (n.op == Op::Leaf) {
    // dy is contiguous in the leaf's own label order and shape
    const int64_t cnt = dy.numel();
    OM_CUDA(cudaMemcpyAsync(grads[n.tensor_index], dy.ptr, es * (size_t)cnt,
                            cudaMemcpyDeviceToDevice, be->stream),
            "einsum grad copy");
    return OM_OK;
  }
  if (n.op == Op::Unary) {
    const DTensor& child = nodes[n.child0].content;
    DTensor g;
    if (tropical) {
      // tropical_unary_backward: zero tensor, grad[argmax[o]] += dy[o]
      OM_TRY(new_tensor(child.ix, g));
      OM_CUDA(cudaMemsetAsync((void*)g.ptr, 0, es * (size_t)g.numel(), be->stream), "memset");
      const int64_t cnt = dy.numel();
      int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((cnt + 255) / 256, (int64_t)be->num_sms * 16));
      {
        ProfScope prof(be, "unary_scatter");
        if (dt == OM_F32)
          scatter_add_kernel<float><<<blocks, 256, 0, be->stream>>>(
              (const float*)dy.ptr, n.am, (float*)g.ptr, cnt);
        else
          scatter_add_kernel<double><<<blocks, 256, 0, be->stream>>>(
              (const double*)dy.ptr, n.am, (double*)g.ptr, cnt);
        note_launch();
        OM_CUDA(cudaGetLastError(), "scatter launch");
      }
    } else {
      // contract_unary_backward: index exchange out_ix -> in_ix
      std::shared_ptr<void> none;
      OM_TRY(unary(dy, n.in_ix, false, g, none));
    }
    g.ix = child.ix;
    return backprop(n.child0, g, grads);
  }
  const DTensor& l = nodes[n.child0].content;
  const DTensor& r = nodes[n.child1].content;
  DTensor gl, gr;
  if (tropical) {
    OM_TRY(new_tensor(n.left_ix, gl));
    OM_TRY(new_tensor(n.right_ix, gr));
    OM_CUDA(cudaMemsetAsync((void*)gl.ptr, 0, es * (size_t)gl.numel(), be->stream), "memset");
    OM_CUDA(cudaMemsetAsync((void*)gr.ptr, 0, es * (size_t)gr.numel(), be->stream), "memset");
    OM_TRY(om_b200_tropical_backward(be, dt, dy.ptr, n.am,
                                     (int)n.left_ix.size(), l.shape.data(), n.left_ix.data(),
                                     (int)n.right_ix.size(), r.shape.data(), n.right_ix.data(),
                                     (int)n.out_ix.size(), dy.shape.data(), n.out_ix.data(),
                                     (void*)gl.ptr, (void*)gr.ptr));
  } else {
    // standard_backward: grad_a = dy (x) b -> ia, grad_b = a (x) dy -> ib
    std::shared_ptr<void> none;
    OM_TRY(contract(dy, n.out_ix, r, n.right_ix, n.left_ix, false, gl, none));
    OM_TRY(contract(l, n.left_ix, dy, n.out_ix, n.right_ix, false, gr, none));
  }
  OM_TRY(backprop(n.child0, gl, grads));
  return backprop(n.child1, gr, grads);
}

}  // namespace om

struct om_tape {
  om::Engine eng;
};

using namespace om;

static int einsum_impl(om_backend* be, om_algebra alg, om_dtype dtype, int ntensors,
                       const void* const* tensors, const int32_t* ndims, const int64_t* shapes,
                       const int64_t* strides, const int32_t* ixs, int niy, const int32_t* iy,
                       int nsizes, const int32_t* size_labels, const int64_t* size_values,
                       int nnodes, const int32_t* children, const int32_t* node_iy_off,
                       const int32_t* node_iy, void* out, om_tape** tape_out, bool lazy) {
  if (!be || !tensors || !ndims || !out || ntensors < 1 || niy < 0 || nnodes < 0 ||
      (nnodes > 0 && (!children || !node_iy_off)))
    return set_error(OM_ERR_INVALID, "om_b200_einsum: bad argument");
  if (dtype != OM_F32 && dtype != OM_F64 && !(is_complex(dtype) && alg == OM_STANDARD))
    return set_error(OM_ERR_UNSUPPORTED,
                     "om_b200_einsum: dtype must be f32 or f64 (complex: Standard algebra only)");
  if (nnodes == 0 && ntensors != 1)
    return set_error(OM_ERR_INVALID, "om_b200_einsum: a tree without nodes needs exactly one tensor");
  if (nnodes > 0 && nnodes != ntensors - 1)
    return set_error(OM_ERR_INVALID, "om_b200_einsum: a binary tree over n tensors has n-1 nodes");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  auto* tape = new om_tape();
  Engine& E = tape->eng;
  E.be = be;
  E.alg = alg;
  E.dt = dtype;
  E.es = dtype_size(dtype);
  E.tropical = alg != OM_STANDARD;
  E.keep = tape_out != nullptr;
  E.lazy = lazy && E.tropical;
  for (int q = 0; q < nsizes; ++q) E.sizes[size_labels[q]] = size_values[q];
  std::unique_ptr<om_tape> guard(tape);

  // leaves
  int64_t off = 0;
  std::vector<int> leaf_node(ntensors);
  for (int t = 0; t < ntensors; ++t) {
    TapeNode n;
    n.op = Op::Leaf;
    n.tensor_index = t;
    n.content.ptr = tensors[t];
    n.content.shape.assign(shapes + off, shapes + off + ndims[t]);
    n.content.strides.assign(strides + off, strides + off + ndims[t]);
    n.content.ix.assign(ixs + off, ixs + off + ndims[t]);
    for (int d = 0; d < ndims[t]; ++d) {
      auto it = E.sizes.find(ixs[off + d]);
      if (it == E.sizes.end()) E.sizes[ixs[off + d]] = shapes[off + d];
      else if (it->second != shapes[off + d])
        return set_error(OM_ERR_SHAPE, "om_b200_einsum: label " + std::to_string(ixs[off + d]) +
                                           " has two extents");
    }
    E.input_shapes.push_back(n.content.shape);
    off += ndims[t];
    E.nodes.push_back(std::move(n));
    leaf_node[t] = (int)E.nodes.size() - 1;
  }
  std::vector<int32_t> final_iy(iy, iy + niy);

  int cur = leaf_node[0];
  if (nnodes > 0) {
    std::vector<int> node_of(nnodes, -1);
    for (int i = 0; i < nnodes; ++i) {
      auto resolve = [&](int c, int* out_node) -> int {
        if (c < 0 || c >= ntensors + i)
          return set_error(OM_ERR_INVALID, "om_b200_einsum: child refers to a later node");
        *out_node = c < ntensors ? leaf_node[c] : node_of[c - ntensors];
        return OM_OK;
      };
      int l, r;
      OM_TRY(resolve(children[2 * i], &l));
      OM_TRY(resolve(children[2 * i + 1], &r));
      std::vector<int32_t> niy_(node_iy + node_iy_off[i], node_iy + node_iy_off[i + 1]);
      const std::vector<int32_t> rix0 = E.nodes[r].content.ix;
      OM_TRY(E.normalize(l, rix0, niy_, &l));
      const std::vector<int32_t> lix = E.nodes[l].content.ix;
      OM_TRY(E.normalize(r, lix, niy_, &r));
      TapeNode n;
      n.op = Op::Binary;
      n.child0 = l;
      n.child1 = r;
      n.left_ix = lix;
      n.right_ix = E.nodes[r].content.ix;
      n.out_ix = E.node_order(E.nodes[l].content, E.nodes[r].content, niy_);
      OM_TRY(E.contract(E.nodes[l].content, n.left_ix, E.nodes[r].content, n.right_ix, n.out_ix,
                        E.keep && E.tropical && !E.lazy, n.content, n.argmax));
      n.am = (const uint32_t*)n.argmax.get();
      E.nodes.push_back(std::move(n));
      node_of[i] = (int)E.nodes.size() - 1;
    }
    cur = node_of[nnodes - 1];
  }
  // finalise to iy (a leaf root is always passed through the unary einsum)
  if (nnodes == 0 || E.nodes[cur].content.ix != final_iy) OM_TRY(E.push_unary(cur, final_iy, &cur));
  E.root = cur;
  const DTensor& res = E.nodes[cur].content;
  OM_CUDA(cudaMemcpyAsync(out, res.ptr, E.es * (size_t)res.numel(), cudaMemcpyDeviceToDevice,
                          be->stream),
          "einsum result copy");
  if (tape_out) *tape_out = guard.release();
  return OM_OK;
}

extern "C" int om_b200_einsum(om_backend* be, om_algebra alg, om_dtype dtype, int ntensors,
                              const void* const* tensors, const int32_t* ndims,
                              const int64_t* shapes, const int64_t* strides, const int32_t* ixs,
                              int niy, const int32_t* iy, int nsizes, const int32_t* size_labels,
                              const int64_t* size_values, int nnodes, const int32_t* children,
                              const int32_t* node_iy_off, const int32_t* node_iy, void* out,
                              om_tape** tape_out) {
  return einsum_impl(be, alg, dtype, ntensors, tensors, ndims, shapes, strides, ixs, niy, iy,
                     nsizes, size_labels, size_values, nnodes, children, node_iy_off, node_iy, out,
                     tape_out, false);
}

extern "C" int om_b200_einsum_tape_values(om_backend* be, om_algebra alg, om_dtype dtype,
                                          int ntensors, const void* const* tensors,
                                          const int32_t* ndims, const int64_t* shapes,
                                          const int64_t* strides, const int32_t* ixs, int niy,
                                          const int32_t* iy, int nsizes,
                                          const int32_t* size_labels, const int64_t* size_values,
                                          int nnodes, const int32_t* children,
                                          const int32_t* node_iy_off, const int32_t* node_iy,
                                          void* out, om_tape** tape_out) {
  if (!tape_out) return set_error(OM_ERR_INVALID, "om_b200_einsum_tape_values: tape_out is null");
  if (alg == OM_STANDARD)
    return set_error(OM_ERR_UNSUPPORTED, "om_b200_einsum_tape_values: tropical algebras only");
  return einsum_impl(be, alg, dtype, ntensors, tensors, ndims, shapes, strides, ixs, niy, iy,
                     nsizes, size_labels, size_values, nnodes, children, node_iy_off, node_iy, out,
                     tape_out, true);
}

extern "C" int om_b200_einsum_backward(om_tape* tape, const void* dy, void* const* grads) {
  if (!tape || !dy || !grads) return set_error(OM_ERR_INVALID, "om_b200_einsum_backward: null argument");
  Engine& E = tape->eng;
  OM_CUDA(cudaSetDevice(E.be->device), "cudaSetDevice");
  DTensor d = E.nodes[E.root].content;
  d.owner.reset();
  d.ptr = dy;
  const int64_t n = d.numel();
  if (E.tropical && n <= kSparseGradMax) return E.backprop_sparse(dy, grads);
  if (E.lazy)
    return set_error(OM_ERR_UNSUPPORTED, "om_b200_einsum_backward: a values-only tape needs an "
                                         "output of at most 4096 elements");
  return E.backprop(E.root, d, grads);
}

extern "C" int om_b200_tape_free(om_tape* tape) {
  delete tape;
  return OM_OK;
}

extern "C" int om_b200_tape_release(om_tape* tape) {
  if (!tape) return set_error(OM_ERR_INVALID, "om_b200_tape_release: null tape");
  Engine& E = tape->eng;
  OM_CUDA(cudaSetDevice(E.be->device), "cudaSetDevice");
  for (auto& n : E.nodes) {
    n.content.owner.reset();  // stream-ordered free; the address is kept
    n.argmax.reset();
  }
  return OM_OK;
}

extern "C" int om_b200_einsum_backward_linked(om_tape* tape, const void* dy, void* const* grads,
                                              int nlinks, const int32_t* link_leaf,
                                              om_tape* const* link_tapes,
                                              void* const* const* link_grads) {
  if (!tape || !dy || !grads || nlinks < 0 || (nlinks && (!link_leaf || !link_tapes || !link_grads)))
    return set_error(OM_ERR_INVALID, "om_b200_einsum_backward_linked: null argument");
  Engine& E = tape->eng;
  OM_CUDA(cudaSetDevice(E.be->device), "cudaSetDevice");
  if (!E.tropical || E.nodes[E.root].content.numel() > kSparseGradMax)
    return set_error(OM_ERR_UNSUPPORTED,
                     "om_b200_einsum_backward_linked: tropical tapes with a root of at most 4096 "
                     "elements only");
  std::vector<const Engine*> engines{&E};
  std::vector<void* const*> egrads{grads};
  std::map<int, int> link;
  for (int i = 0; i < nlinks; ++i) {
    if (!link_tapes[i] || !link_grads[i])
      return set_error(OM_ERR_INVALID, "om_b200_einsum_backward_linked: null linked tape");
    const Engine& S = link_tapes[i]->eng;
    if (S.alg != E.alg || S.dt != E.dt)
      return set_error(OM_ERR_INVALID, "om_b200_einsum_backward_linked: algebra or dtype differs");
    link[link_leaf[i]] = (int)engines.size();
    engines.push_back(&S);
    egrads.push_back(link_grads[i]);
  }
  return E.backprop_sparse_linked(dy, engines, egrads, link);
}
