// Standard f64 GEMM on the FP64 pipes (DFMA), register-tiled.
//
// Serves Standard<f64> contractions of GEMM shape (the reference's faer f64
// path, src/backend/cpu/mod.rs:621-859).  tcgen05 has no f64 kind, and on
// B200 the FP64 rate of the CUDA cores is that of the FP64 tensor path, so
// a DFMA kernel that keeps the FP64 pipes busy is the B200 form:
//   * CTA tile 128 x 128, 256 threads, 8 x 8 outputs per thread (64 f64
//     accumulators), one CTA per SM;
//   * k slabs of 16 staged through registers into shared memory as [k][m]
//     and [k][n] (any of the four unit-stride orientations of A and B), two
//     buffers, so the next slab's global loads overlap the current slab's
//     FMAs;
//   * a thread's rows are pairs 16 apart (2*lr + 16 j + t), so each
//     16-byte fragment load of the 8 lanes sharing a column group covers one
//     contiguous 128-byte line, and lanes of other groups broadcast.
// Every product is an IEEE fma in k order per output (the summation order
// differs from faer's; Standard parity is by tolerance).
#include <algorithm>

#include "om_internal.h"

namespace om {
namespace {

constexpr int DM = 128, DN = 128, DK = 16, DT = 256;
// shared-memory row lengths: two doubles of padding spread the transposed
// scalar stores of a k-contiguous operand over the banks (rows stay 16-byte
// aligned: 130 doubles = 1040 bytes)
constexpr int SM_A = DM + 2, SM_B = DN + 2;

struct F64Args {
  int64_t M, N, K, batch;
  const double* A;
  int64_t lda, sab;  // the non-unit stride of A, batch stride
  const double* B;
  int64_t ldb, sbb;
  double* C;
  int64_t scm, scn, scb;
  int64_t ka1 = 0, sak2 = 0, kb1 = 0, sbk2 = 0;  // two-level k (0: flat), multiples of DK
};

template <bool A_MC, bool B_KC>
struct F64Stager {
  double2 ra[4], rb[4];

  __device__ __forceinline__ void load(const F64Args& g, const double* Ab, const double* Bb, int64_t m0,
                                       int64_t n0, int64_t k0, int tid) {
    const double2 z = make_double2(0.0, 0.0);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int u = tid + r * DT;
      if (A_MC) {  // A[m + k*lda]: pairs along m
        const int k = u / 64, m = 2 * (u % 64);
        const int64_t gm = m0 + m, gk = k0 + k;
        if (gk < g.K && gm + 1 < g.M) {
          ra[r] = *(const double2*)(Ab + gm + kofs(gk, g.lda, g.ka1, g.sak2));
        } else {
          ra[r] = z;
          if (gk < g.K && gm < g.M) ra[r].x = Ab[gm + kofs(gk, g.lda, g.ka1, g.sak2)];
        }
      } else {  // A[m*lda + k]: pairs along k
        const int m = u / 8, k = 2 * (u % 8);
        const int64_t gm = m0 + m, gk = k0 + k;
        if (gm < g.M && gk + 1 < g.K) {
          ra[r] = *(const double2*)(Ab + gm * g.lda + kofs(gk, 1, g.ka1, g.sak2));
        } else {
          ra[r] = z;
          if (gm < g.M && gk < g.K) ra[r].x = Ab[gm * g.lda + kofs(gk, 1, g.ka1, g.sak2)];
        }
      }
      if (B_KC) {  // B[k + n*ldb]: pairs along k
        const int n = u / 8, k = 2 * (u % 8);
        const int64_t gn = n0 + n, gk = k0 + k;
        if (gn < g.N && gk + 1 < g.K) {
          rb[r] = *(const double2*)(Bb + gn * g.ldb + kofs(gk, 1, g.kb1, g.sbk2));
        } else {
          rb[r] = z;
          if (gn < g.N && gk < g.K) rb[r].x = Bb[gn * g.ldb + kofs(gk, 1, g.kb1, g.sbk2)];
        }
      } else {  // B[k*ldb + n]: pairs along n
        const int k = u / 64, n = 2 * (u % 64);
        const int64_t gn = n0 + n, gk = k0 + k;
        if (gk < g.K && gn + 1 < g.N) {
          rb[r] = *(const double2*)(Bb + gn + kofs(gk, g.ldb, g.kb1, g.sbk2));
        } else {
          rb[r] = z;
          if (gk < g.K && gn < g.N) rb[r].x = Bb[gn + kofs(gk, g.ldb, g.kb1, g.sbk2)];
        }
      }
    }
  }

  __device__ __forceinline__ void store(double* As, double* Bs, int tid) const {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int u = tid + r * DT;
      if (A_MC) {
        const int k = u / 64, m = 2 * (u % 64);
        *(double2*)(As + k * SM_A + m) = ra[r];
      } else {
        const int m = u / 8, k = 2 * (u % 8);
        As[k * SM_A + m] = ra[r].x;
        As[(k + 1) * SM_A + m] = ra[r].y;
      }
      if (B_KC) {
        const int n = u / 8, k = 2 * (u % 8);
        Bs[k * SM_B + n] = rb[r].x;
        Bs[(k + 1) * SM_B + n] = rb[r].y;
      } else {
        const int k = u / 64, n = 2 * (u % 64);
        *(double2*)(Bs + k * SM_B + n) = rb[r];
      }
    }
  }
};

template <bool A_MC, bool B_KC>
__global__ void __launch_bounds__(DT, 1) gemm_f64_kernel(F64Args g) {
  extern __shared__ __align__(16) double dsm[];
  double* As0 = dsm;                 // 2 x [DK][SM_A]
  double* Bs0 = dsm + 2 * DK * SM_A; // 2 x [DK][SM_B]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lr = lane & 7, lc = lane >> 3;
  const int rbase = 64 * (warp & 1) + 2 * lr;   // rows rbase + 16 j + t
  const int cbase = 32 * (warp >> 1) + 2 * lc;  // cols cbase + 8 j + t
  const int64_t tiles_m = (g.M + DM - 1) / DM, tiles_n = (g.N + DN - 1) / DN;
  const int64_t tiles = tiles_m * tiles_n * g.batch;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t tm = tile % tiles_m, tn = (tile / tiles_m) % tiles_n, bt = tile / (tiles_m * tiles_n);
    const int64_t m0 = tm * DM, n0 = tn * DN;
    const double* Ab = g.A + bt * g.sab;
    const double* Bb = g.B + bt * g.sbb;
    double acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.0;
    F64Stager<A_MC, B_KC> st;
    __syncthreads();  // the previous tile may still read shared memory
    st.load(g, Ab, Bb, m0, n0, 0, tid);
    st.store(As0, Bs0, tid);
    __syncthreads();
    const int64_t T = (g.K + DK - 1) / DK;
    for (int64_t t = 0; t < T; ++t) {
      const int buf = (int)(t & 1);
      if (t + 1 < T) st.load(g, Ab, Bb, m0, n0, (t + 1) * DK, tid);
      const double* As = As0 + buf * DK * SM_A;
      const double* Bs = Bs0 + buf * DK * SM_B;
#pragma unroll 4
      for (int kk = 0; kk < DK; ++kk) {
        double a[8], b[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const double2 x = *(const double2*)(As + kk * SM_A + rbase + 16 * j);
          a[2 * j] = x.x;
          a[2 * j + 1] = x.y;
          const double2 y = *(const double2*)(Bs + kk * SM_B + cbase + 8 * j);
          b[2 * j] = y.x;
          b[2 * j + 1] = y.y;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
      }
      if (t + 1 < T) st.store(As0 + (buf ^ 1) * DK * SM_A, Bs0 + (buf ^ 1) * DK * SM_B, tid);
      __syncthreads();
    }
    double* Cb = g.C + bt * g.scb;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t m = m0 + rbase + 16 * (i >> 1) + (i & 1);
      if (m >= g.M) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t n = n0 + cbase + 8 * (j >> 1) + (j & 1);
        if (n < g.N) Cb[m * g.scm + n * g.scn] = acc[i][j];
      }
    }
  }
}

template <bool A_MC, bool B_KC>
int launch_f64(om_backend* be, const F64Args& a) {
  const size_t smem = sizeof(double) * 2 * DK * (SM_A + SM_B);
  auto kern = gemm_f64_kernel<A_MC, B_KC>;
  OM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
          "cudaFuncSetAttribute");
  const int64_t tiles = ((a.M + DM - 1) / DM) * ((a.N + DN - 1) / DN) * a.batch;
  const int grid = (int)std::min<int64_t>(tiles, be->num_sms);
  ProfScope prof(be, "gemm_f64_dfma");
  kern<<<grid, DT, smem, be->stream>>>(a);
  note_launch();
  return check_cuda(cudaGetLastError(), "gemm_f64 launch");
}

}  // namespace

// orientation of the operands for 16-byte loads, or false
static bool f64_orient(const GemmArgs& g, bool* amc, int64_t* lda, bool* bkc, int64_t* ldb) {
  if (g.ma1 || g.nb1) return false;
  if ((g.ka1 || g.kb1) && g.batch != 1) return false;
  if (g.ka1 && (g.ka1 % DK || g.sak2 % 2)) return false;
  if (g.kb1 && (g.kb1 % DK || g.sbk2 % 2)) return false;
  auto ok16 = [](const void* p, int64_t n_unit, int64_t st) {
    return ((uintptr_t)p % 16) == 0 && n_unit % 2 == 0 && st % 2 == 0;
  };
  if (g.sam == 1 && ok16(g.A, g.M, g.sak) && g.sab % 2 == 0) {
    *amc = true;
    *lda = g.sak;
  } else if (g.sak == 1 && ok16(g.A, g.K, g.sam) && g.sab % 2 == 0) {
    *amc = false;
    *lda = g.sam;
  } else {
    return false;
  }
  if (g.sbk == 1 && ok16(g.B, g.K, g.sbn) && g.sbb % 2 == 0) {
    *bkc = true;
    *ldb = g.sbn;
  } else if (g.sbn == 1 && ok16(g.B, g.N, g.sbk) && g.sbb % 2 == 0) {
    *bkc = false;
    *ldb = g.sbk;
  } else {
    return false;
  }
  return true;
}

bool f64_dfma_takes(om_backend* be, const GemmArgs& g) {
  bool amc, bkc;
  int64_t lda, ldb;
  // large enough for 128 x 128 tiles to pay; smaller shapes keep the
  // generic kernels
  return g.dtype == OM_F64 && g.alg == OM_STANDARD && !g.argmax && g.M >= 64 && g.N >= 64 &&
         g.K >= 16 && g.M * g.N * g.batch >= (int64_t)be->num_sms * DM * DN / 2 &&
         f64_orient(g, &amc, &lda, &bkc, &ldb);
}

int launch_gemm_f64(om_backend* be, const GemmArgs& g, bool* handled) {
  *handled = false;
  if (!f64_dfma_takes(be, g)) return OM_OK;
  F64Args a;
  a.M = g.M;
  a.N = g.N;
  a.K = g.K;
  a.batch = g.batch;
  a.A = (const double*)g.A;
  a.sab = g.sab;
  a.B = (const double*)g.B;
  a.sbb = g.sbb;
  a.C = (double*)g.C;
  a.scm = g.scm;
  a.scn = g.scn;
  a.scb = g.scb;
  a.ka1 = g.ka1;
  a.sak2 = g.sak2;
  a.kb1 = g.kb1;
  a.sbk2 = g.sbk2;
  bool amc, bkc;
  f64_orient(g, &amc, &a.lda, &bkc, &a.ldb);
  *handled = true;
  if (amc && bkc) return launch_f64<true, true>(be, a);
  if (amc) return launch_f64<true, false>(be, a);
  if (bkc) return launch_f64<false, true>(be, a);
  return launch_f64<false, false>(be, a);
}

}  // namespace om
