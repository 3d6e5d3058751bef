/*
 * oracle.c -- CPU restatement of the omeinsum-rs CPU contraction path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the B200 kernels
 * are compared against (tests/, __graft_entry__.smoke() and the cpu_baseline
 * leg of bench.py).  The product library never links, loads or calls it.
 *
 * It restates, in plain C, the semantics of the reference's own CPU backend
 * (tensor4all/omeinsum-rs, paths relative to that project):
 *
 *   semiring scalar ops        src/algebra/tropical.rs:46-143,169-263,289-384
 *                              src/algebra/standard.rs:26-116
 *   generic GEMM (+argmax)     src/backend/cpu/mod.rs:862-886, 889-920
 *   batched GEMM (+argmax)     src/backend/cpu/mod.rs:414-488
 *   mode classification        src/backend/cpu/contract.rs:11-79
 *   trace reduction            src/backend/cpu/contract.rs:309-363
 *   permute odometer           src/backend/cpu/contract.rs:709-748
 *   contract / _with_argmax    src/backend/cpu/contract.rs:467-671, 752-859
 *   copy_strided               src/backend/cpu/mod.rs:584-619
 *   unary naive / argmax       src/einsum/engine.rs:752-832, 841-926
 *
 * Semantics kept exactly (they decide bit-level parity):
 *   - MaxPlus zero = -FLT_MAX (f32::MIN), MinPlus zero = +FLT_MAX, MaxMul zero = 0
 *     (tropical.rs:47-49,170-172).
 *   - add(acc, p) = (acc >= p) ? acc : p for max algebras, (acc <= p) ? acc : p
 *     for MinPlus; a NaN accumulator is replaced by the next product.
 *   - argmax starts at 0 with acc = zero(); the first k wins on ties.
 *   - everything is column-major (first axis fastest), strides in elements.
 *
 * Standard algebra: the reference calls faer 0.24 (cpu/mod.rs:651-708), whose
 * summation order is not reproducible here.  The oracle accumulates f32 in
 * double and f64 in long double and rounds once: a high-accuracy answer that
 * tests compare against with a stated relative tolerance.
 *
 * Large tensors: the loops run in the reference's own order (j, i, kk) so the
 * single-thread timing of orc_gemm is the reference's CPU cost model; the
 * orc_gemm_omp variant splits the j loop over OpenMP threads (the "all host
 * cores" CPU baseline).
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* scalar semiring ops                                                       */
/* ------------------------------------------------------------------------ */

#define DEF_SCALAR(T, SFX, TMIN, TMAX)                                            \
  static inline T zero_##SFX(int alg) {                                        \
    switch (alg) {                                                             \
      case ORC_MAXPLUS: return TMIN;                                           \
      case ORC_MINPLUS: return TMAX;                                           \
      default: return (T)0;                                                    \
    }                                                                          \
  }                                                                            \
  static inline T mul_##SFX(int alg, T a, T b) {                               \
    return (alg == ORC_MAXPLUS || alg == ORC_MINPLUS) ? (T)(a + b) : (T)(a * b); \
  }                                                                            \
  /* returns 1 when the accumulator is kept (tropical.rs add/add_with_argmax) */ \
  static inline int keep_##SFX(int alg, T acc, T p) {                          \
    return (alg == ORC_MINPLUS) ? (acc <= p) : (acc >= p);                     \
  }                                                                            \
  static inline T add_##SFX(int alg, T acc, T p) {                             \
    if (alg == ORC_STANDARD) return (T)(acc + p);                              \
    return keep_##SFX(alg, acc, p) ? acc : p;                                  \
  }                                                                            \
  /* is_better (tropical.rs:136-143,256-263): strict */                        \
  static inline int better_##SFX(int alg, T v, T best) {                       \
    if (alg == ORC_MINPLUS) return v < best;                                   \
    if (alg == ORC_STANDARD) return 0;                                         \
    return v > best;                                                           \
  }

DEF_SCALAR(float, f32, -FLT_MAX, FLT_MAX)
DEF_SCALAR(double, f64, -DBL_MAX, DBL_MAX)

/* ------------------------------------------------------------------------ */
/* GEMM (column-major A m x k, B k x n, C m x n)                             */
/* ------------------------------------------------------------------------ */

static void gemm_f32(int alg, const float* a, int64_t m, int64_t k, const float* b,
                     int64_t n, float* c, uint32_t* am, int nthreads) {
  int64_t j;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads) if (nthreads > 1)
  for (j = 0; j < n; ++j) {
    for (int64_t i = 0; i < m; ++i) {
      if (alg == ORC_STANDARD && !am) {
        double acc = 0.0;
        for (int64_t kk = 0; kk < k; ++kk) acc += (double)a[kk * m + i] * (double)b[j * k + kk];
        c[j * m + i] = (float)acc;
        continue;
      }
      float acc = zero_f32(alg);
      uint32_t best = 0;
      for (int64_t kk = 0; kk < k; ++kk) {
        float p = mul_f32(alg, a[kk * m + i], b[j * k + kk]);
        if (alg == ORC_STANDARD) {
          acc = acc + p; /* generic_gemm_with_argmax for Standard: argmax stays 0 */
        } else if (!keep_f32(alg, acc, p)) {
          acc = p;
          best = (uint32_t)kk;
        }
      }
      c[j * m + i] = acc;
      if (am) am[j * m + i] = best;
    }
  }
}

static void gemm_f64(int alg, const double* a, int64_t m, int64_t k, const double* b,
                     int64_t n, double* c, uint32_t* am, int nthreads) {
  int64_t j;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads) if (nthreads > 1)
  for (j = 0; j < n; ++j) {
    for (int64_t i = 0; i < m; ++i) {
      if (alg == ORC_STANDARD && !am) {
        long double acc = 0.0L;
        for (int64_t kk = 0; kk < k; ++kk)
          acc += (long double)a[kk * m + i] * (long double)b[j * k + kk];
        c[j * m + i] = (double)acc;
        continue;
      }
      double acc = zero_f64(alg);
      uint32_t best = 0;
      for (int64_t kk = 0; kk < k; ++kk) {
        double p = mul_f64(alg, a[kk * m + i], b[j * k + kk]);
        if (alg == ORC_STANDARD) {
          acc = acc + p;
        } else if (!keep_f64(alg, acc, p)) {
          acc = p;
          best = (uint32_t)kk;
        }
      }
      c[j * m + i] = acc;
      if (am) am[j * m + i] = best;
    }
  }
}

int orc_gemm(int alg, int dtype, const void* a, int64_t m, int64_t k, const void* b, int64_t n,
             void* c, uint32_t* argmax, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (dtype == ORC_F32)
    gemm_f32(alg, (const float*)a, m, k, (const float*)b, n, (float*)c, argmax, nthreads);
  else if (dtype == ORC_F64)
    gemm_f64(alg, (const double*)a, m, k, (const double*)b, n, (double*)c, argmax, nthreads);
  else
    return -1;
  return 0;
}

/* cpu/mod.rs:414-488: batch is the slowest axis of the permuted operands. */
int orc_gemm_batched(int alg, int dtype, const void* a, int64_t batch, int64_t m, int64_t k,
                     const void* b, int64_t n, void* c, uint32_t* argmax) {
  size_t es = dtype == ORC_F64 ? 8 : 4;
  for (int64_t t = 0; t < batch; ++t) {
    const char* ap = (const char*)a + (size_t)(t * m * k) * es;
    const char* bp = (const char*)b + (size_t)(t * k * n) * es;
    char* cp = (char*)c + (size_t)(t * m * n) * es;
    int rc = orc_gemm(alg, dtype, ap, m, k, bp, n, cp, argmax ? argmax + t * m * n : NULL, 1);
    if (rc) return rc;
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* strided copies                                                            */
/* ------------------------------------------------------------------------ */

/* Backend::copy_strided for Cpu (cpu/mod.rs:584-619): column-major odometer. */
int orc_copy_strided(int64_t elem_size, const void* src, int ndim, const int64_t* shape,
                     const int64_t* strides, int64_t offset, void* dst) {
  int64_t numel = 1;
  for (int d = 0; d < ndim; ++d) numel *= shape[d];
  int64_t idx[ORC_MAX_DIMS] = {0};
  for (int64_t e = 0; e < numel; ++e) {
    int64_t so = offset;
    for (int d = 0; d < ndim; ++d) so += idx[d] * strides[d];
    memcpy((char*)dst + e * elem_size, (const char*)src + so * elem_size, (size_t)elem_size);
    for (int d = 0; d < ndim; ++d) {
      if (++idx[d] < shape[d]) break;
      idx[d] = 0;
    }
  }
  return 0;
}

/* materialize_with_permutation_into (contract.rs:709-748): output axis a is
 * input axis perm[a]; output is contiguous column-major. */
static void permute_into(int64_t es, const void* src, int nd, const int64_t* shape,
                         const int64_t* strides, const int* perm, void* dst) {
  int64_t nshape[ORC_MAX_DIMS], nstr[ORC_MAX_DIMS];
  for (int a = 0; a < nd; ++a) {
    nshape[a] = shape[perm[a]];
    nstr[a] = strides[perm[a]];
  }
  orc_copy_strided(es, src, nd, nshape, nstr, 0, dst);
}

static void contiguous_strides(int nd, const int64_t* shape, int64_t* st) {
  int64_t s = 1;
  for (int d = 0; d < nd; ++d) {
    st[d] = s;
    s *= shape[d];
  }
}

/* ------------------------------------------------------------------------ */
/* mode bookkeeping (contract.rs:11-79)                                      */
/* ------------------------------------------------------------------------ */

static int pos_of(const int32_t* modes, int n, int32_t m) {
  for (int i = 0; i < n; ++i)
    if (modes[i] == m) return i;
  return -1;
}

typedef struct {
  int nb, nl, nr, nc;
  int32_t batch[ORC_MAX_DIMS], left[ORC_MAX_DIMS], right[ORC_MAX_DIMS], contr[ORC_MAX_DIMS];
} modes_t;

static void classify(const int32_t* ma, int na, const int32_t* mb, int nb, const int32_t* mc,
                     int nc, modes_t* o) {
  o->nb = o->nl = o->nr = o->nc = 0;
  for (int i = 0; i < na; ++i) {
    int32_t m = ma[i];
    int inb = pos_of(mb, nb, m) >= 0, inc = pos_of(mc, nc, m) >= 0;
    if (inb && inc) {
      if (pos_of(o->batch, o->nb, m) < 0) o->batch[o->nb++] = m;
    } else if (inb) {
      if (pos_of(o->contr, o->nc, m) < 0) o->contr[o->nc++] = m;
    } else if (pos_of(o->left, o->nl, m) < 0) {
      o->left[o->nl++] = m;
    }
  }
  for (int i = 0; i < nb; ++i)
    if (pos_of(ma, na, mb[i]) < 0) o->right[o->nr++] = mb[i];
}

static int64_t prod_dims(const int32_t* sel, int nsel, const int32_t* modes, int n,
                         const int64_t* shape) {
  int64_t p = 1;
  for (int i = 0; i < nsel; ++i) p *= shape[pos_of(modes, n, sel[i])];
  return p < 1 ? 1 : p;
}

/* reduce_trace_modes (contract.rs:309-363), input contiguous. */
static void* trace_reduce(int alg, int dtype, const void* data, int nd, const int64_t* shape,
                          const int32_t* modes, const int32_t* trace, int ntr, int* out_nd,
                          int64_t* out_shape, int32_t* out_modes) {
  int is_tr[ORC_MAX_DIMS] = {0};
  for (int t = 0; t < ntr; ++t) is_tr[pos_of(modes, nd, trace[t])] = 1;
  int k = 0;
  for (int d = 0; d < nd; ++d)
    if (!is_tr[d]) {
      out_shape[k] = shape[d];
      out_modes[k] = modes[d];
      ++k;
    }
  *out_nd = k;
  int64_t nst[ORC_MAX_DIMS];
  contiguous_strides(k, out_shape, nst);
  int64_t nsize = 1, osize = 1;
  for (int d = 0; d < k; ++d) nsize *= out_shape[d];
  for (int d = 0; d < nd; ++d) osize *= shape[d];
  size_t es = dtype == ORC_F64 ? 8 : 4;
  void* res = malloc((size_t)nsize * es);
  for (int64_t i = 0; i < nsize; ++i) {
    if (dtype == ORC_F64) ((double*)res)[i] = zero_f64(alg);
    else ((float*)res)[i] = zero_f32(alg);
  }
  for (int64_t lin = 0; lin < osize; ++lin) {
    int64_t rem = lin, nl = 0;
    int nd2 = 0;
    for (int d = 0; d < nd; ++d) {
      int64_t c = rem % shape[d];
      rem /= shape[d];
      if (!is_tr[d]) nl += c * nst[nd2++];
    }
    if (dtype == ORC_F64) {
      double* r = (double*)res;
      r[nl] = add_f64(alg, r[nl], ((const double*)data)[lin]);
    } else {
      float* r = (float*)res;
      r[nl] = add_f32(alg, r[nl], ((const float*)data)[lin]);
    }
  }
  return res;
}

/* ------------------------------------------------------------------------ */
/* Backend::contract / contract_with_argmax                                  */
/* ------------------------------------------------------------------------ */

/* Follows contract_with_argmax (contract.rs:752-859) for every algebra: the
 * value-only path (contract.rs:467-671) computes the same numbers through a
 * different memory layout, and for tropical algebras the value of a max/min
 * reduction does not depend on layout. */
int orc_contract(int alg, int dtype, const void* a, int nda, const int64_t* shape_a,
                 const int64_t* strides_a, const int32_t* modes_a, const void* b, int ndb,
                 const int64_t* shape_b, const int64_t* strides_b, const int32_t* modes_b,
                 int ndc, const int64_t* shape_c, const int32_t* modes_c, void* c,
                 uint32_t* argmax) {
  if (nda > ORC_MAX_DIMS || ndb > ORC_MAX_DIMS || ndc > ORC_MAX_DIMS) return -2;
  size_t es = dtype == ORC_F64 ? 8 : 4;
  int64_t na = 1, nb = 1;
  for (int d = 0; d < nda; ++d) na *= shape_a[d];
  for (int d = 0; d < ndb; ++d) nb *= shape_b[d];
  void* ac = malloc((size_t)(na ? na : 1) * es);
  void* bc = malloc((size_t)(nb ? nb : 1) * es);
  orc_copy_strided((int64_t)es, a, nda, shape_a, strides_a, 0, ac);
  orc_copy_strided((int64_t)es, b, ndb, shape_b, strides_b, 0, bc);

  modes_t md;
  classify(modes_a, nda, modes_b, ndb, modes_c, ndc, &md);
  int32_t ltr[ORC_MAX_DIMS], rtr[ORC_MAX_DIMS], lfree[ORC_MAX_DIMS], rfree[ORC_MAX_DIMS];
  int nltr = 0, nrtr = 0, nlf = 0, nrf = 0;
  for (int i = 0; i < md.nl; ++i) {
    if (pos_of(modes_c, ndc, md.left[i]) < 0) ltr[nltr++] = md.left[i];
    else lfree[nlf++] = md.left[i];
  }
  for (int i = 0; i < md.nr; ++i) {
    if (pos_of(modes_c, ndc, md.right[i]) < 0) rtr[nrtr++] = md.right[i];
    else rfree[nrf++] = md.right[i];
  }

  int a_nd = nda, b_nd = ndb;
  int64_t a_shape[ORC_MAX_DIMS], b_shape[ORC_MAX_DIMS];
  int32_t a_modes[ORC_MAX_DIMS], b_modes[ORC_MAX_DIMS];
  memcpy(a_shape, shape_a, sizeof(int64_t) * nda);
  memcpy(b_shape, shape_b, sizeof(int64_t) * ndb);
  memcpy(a_modes, modes_a, sizeof(int32_t) * nda);
  memcpy(b_modes, modes_b, sizeof(int32_t) * ndb);
  if (nltr) {
    void* r = trace_reduce(alg, dtype, ac, nda, shape_a, modes_a, ltr, nltr, &a_nd, a_shape, a_modes);
    free(ac);
    ac = r;
  }
  if (nrtr) {
    void* r = trace_reduce(alg, dtype, bc, ndb, shape_b, modes_b, rtr, nrtr, &b_nd, b_shape, b_modes);
    free(bc);
    bc = r;
  }

  int64_t bsz = prod_dims(md.batch, md.nb, a_modes, a_nd, a_shape);
  int64_t lsz = prod_dims(lfree, nlf, a_modes, a_nd, a_shape);
  int64_t rsz = prod_dims(rfree, nrf, b_modes, b_nd, b_shape);
  int64_t ksz = prod_dims(md.contr, md.nc, a_modes, a_nd, a_shape);

  /* A -> [left, contracted, batch], B -> [contracted, right, batch] */
  int pa[ORC_MAX_DIMS], pb[ORC_MAX_DIMS], q = 0;
  for (int i = 0; i < nlf; ++i) pa[q++] = pos_of(a_modes, a_nd, lfree[i]);
  for (int i = 0; i < md.nc; ++i) pa[q++] = pos_of(a_modes, a_nd, md.contr[i]);
  for (int i = 0; i < md.nb; ++i) pa[q++] = pos_of(a_modes, a_nd, md.batch[i]);
  q = 0;
  for (int i = 0; i < md.nc; ++i) pb[q++] = pos_of(b_modes, b_nd, md.contr[i]);
  for (int i = 0; i < nrf; ++i) pb[q++] = pos_of(b_modes, b_nd, rfree[i]);
  for (int i = 0; i < md.nb; ++i) pb[q++] = pos_of(b_modes, b_nd, md.batch[i]);
  int64_t ast[ORC_MAX_DIMS], bst[ORC_MAX_DIMS];
  contiguous_strides(a_nd, a_shape, ast);
  contiguous_strides(b_nd, b_shape, bst);
  void* ap = malloc((size_t)(lsz * ksz * bsz) * es);
  void* bp = malloc((size_t)(ksz * rsz * bsz) * es);
  permute_into((int64_t)es, ac, a_nd, a_shape, ast, pa, ap);
  permute_into((int64_t)es, bc, b_nd, b_shape, bst, pb, bp);

  int64_t nout = lsz * rsz * bsz;
  void* cc = malloc((size_t)nout * es);
  uint32_t* amc = argmax ? (uint32_t*)malloc((size_t)nout * 4) : NULL;
  if (md.nb == 0) orc_gemm(alg, dtype, ap, lsz, ksz, bp, rsz, cc, amc, 1);
  else orc_gemm_batched(alg, dtype, ap, bsz, lsz, ksz, bp, rsz, cc, amc);

  /* current order [left_free, right_free, batch] -> modes_c */
  int32_t cur[ORC_MAX_DIMS];
  int ncur = 0;
  for (int i = 0; i < nlf; ++i) cur[ncur++] = lfree[i];
  for (int i = 0; i < nrf; ++i) cur[ncur++] = rfree[i];
  for (int i = 0; i < md.nb; ++i) cur[ncur++] = md.batch[i];
  int64_t cshape[ORC_MAX_DIMS], cst[ORC_MAX_DIMS];
  int operm[ORC_MAX_DIMS];
  for (int i = 0; i < ncur; ++i) cshape[i] = shape_c[pos_of(modes_c, ndc, cur[i])];
  contiguous_strides(ncur, cshape, cst);
  for (int i = 0; i < ndc; ++i) operm[i] = pos_of(cur, ncur, modes_c[i]);
  permute_into((int64_t)es, cc, ncur, cshape, cst, operm, c);
  if (argmax) permute_into(4, amc, ncur, cshape, cst, operm, argmax);

  free(ac);
  free(bc);
  free(ap);
  free(bp);
  free(cc);
  free(amc);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* execute_unary_naive / execute_unary_with_argmax (engine.rs:752-926)       */
/* ------------------------------------------------------------------------ */

/* ix (length nx) labels the input axes, may repeat (diagonal); iy (length ny)
 * labels the output axes, may repeat (embedded diagonal, off-diagonal = zero).
 * sizes[label] is the size dictionary; labels must be < ORC_MAX_LABELS.  The
 * input is read through its strides; the output is contiguous column-major.
 * argmax (optional) receives the logical column-major linear input position of
 * the winner, chosen with is_better (strict) and "first element wins". */
int orc_unary(int alg, int dtype, const void* x, int nx, const int32_t* ix, const int64_t* shape_x,
              const int64_t* strides_x, int ny, const int32_t* iy, const int64_t* sizes, void* y,
              uint32_t* argmax) {
  int32_t inner[ORC_MAX_DIMS];
  int ninner = 0;
  for (int d = 0; d < nx; ++d) {
    if (pos_of(iy, ny, ix[d]) >= 0) continue;
    if (pos_of(inner, ninner, ix[d]) < 0) inner[ninner++] = ix[d];
  }
  int64_t out_size = 1, inner_size = 1;
  for (int d = 0; d < ny; ++d) out_size *= sizes[iy[d]];
  for (int d = 0; d < ninner; ++d) inner_size *= sizes[inner[d]];
  if (out_size < 1) out_size = 1;
  if (inner_size < 1) inner_size = 1;
  int64_t val[ORC_MAX_LABELS];
  for (int64_t o = 0; o < out_size; ++o) {
    int64_t rem = o;
    int skip = 0;
    int set[ORC_MAX_LABELS];
    memset(set, 0, sizeof(set));
    for (int d = 0; d < ny; ++d) {
      int64_t s = sizes[iy[d]];
      int64_t c = rem % s;
      rem /= s;
      if (set[iy[d]] && val[iy[d]] != c) {
        skip = 1;
        break;
      }
      set[iy[d]] = 1;
      val[iy[d]] = c;
    }
    if (dtype == ORC_F64) ((double*)y)[o] = zero_f64(alg);
    else ((float*)y)[o] = zero_f32(alg);
    if (argmax) argmax[o] = 0;
    if (skip) continue;
    double best64 = 0.0;
    float best32 = 0.0f;
    long double sum = 0.0L;
    if (dtype == ORC_F64) best64 = zero_f64(alg);
    else best32 = zero_f32(alg);
    uint32_t best_pos = 0;
    for (int64_t in = 0; in < inner_size; ++in) {
      int64_t r2 = in;
      for (int d = 0; d < ninner; ++d) {
        int64_t s = sizes[inner[d]];
        val[inner[d]] = r2 % s;
        r2 /= s;
      }
      int64_t lpos = 0, st = 1, spos = 0;
      for (int d = 0; d < nx; ++d) {
        lpos += val[ix[d]] * st;
        st *= shape_x[d];
        spos += val[ix[d]] * strides_x[d];
      }
      if (dtype == ORC_F64) {
        double v = ((const double*)x)[spos];
        if (argmax) {
          if (in == 0 || better_f64(alg, v, best64)) {
            best64 = v;
            best_pos = (uint32_t)lpos;
          }
        } else if (alg == ORC_STANDARD) {
          sum += v;
        } else {
          best64 = add_f64(alg, best64, v);
        }
      } else {
        float v = ((const float*)x)[spos];
        if (argmax) {
          if (in == 0 || better_f32(alg, v, best32)) {
            best32 = v;
            best_pos = (uint32_t)lpos;
          }
        } else if (alg == ORC_STANDARD) {
          sum += v;
        } else {
          best32 = add_f32(alg, best32, v);
        }
      }
    }
    if (dtype == ORC_F64) ((double*)y)[o] = (alg == ORC_STANDARD && !argmax) ? (double)sum : best64;
    else ((float*)y)[o] = (alg == ORC_STANDARD && !argmax) ? (float)sum : best32;
    if (argmax) argmax[o] = best_pos;
  }
  return 0;
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
