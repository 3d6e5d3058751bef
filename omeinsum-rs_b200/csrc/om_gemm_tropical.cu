// K2: fast f32 tropical GEMM (MaxPlus / MinPlus / MaxMul) with fused argmax.
//
// Same result, bit for bit, as generic_gemm_with_argmax of the reference
// (tensor4all/omeinsum-rs src/backend/cpu/mod.rs:889-920, scalar rules in
// src/algebra/tropical.rs:57-63,93-104) on inputs for which no product is NaN
// or -0 (checked on the device by a special-value scan; otherwise the exact
// compare-select kernel runs, gated on the same flag word, with no host sync).
//
// Design (CUDA cores; tensor cores have no max/min).  A semiring step is one
// FADD (or FMUL) and one FMNMX; on B200 both issue at one warp-instruction per
// scheduler per clock, and the packed add.f32x2 / 3-input max.f32 forms run at
// half rate, so they save nothing.  The kernel therefore aims at the issue
// ceiling of 2 instructions per (i, j, k):
//   * CTA tile 128 x 64, 256 threads, 8 x 4 outputs per thread (2 CTAs/SM),
//     k slabs of 32 double-buffered in shared memory through registers, so any
//     of the four unit-stride orientations of A and B is read with 16-byte
//     loads; per k a thread issues 3 LDS.128 and 32 (FADD, FMNMX) pairs;
//   * argmax without a per-k compare-select: after each slab one compare per
//     output marks (in shared memory) the slab in which the running max
//     strictly improved.  The last such slab holds the first k reaching the
//     final max, because every earlier slab's max is strictly smaller.  A
//     resolve pass re-stages each slab and scans only the outputs it decides
//     for the first k with a (x) b == max, so ties go to the smallest k, and
//     outputs that never beat zero() keep argmax 0, as in the reference.
#include <algorithm>

#include "om_internal.h"
#include "om_semiring.cuh"

namespace om {
namespace {

constexpr int TB_M = 128, TB_N = 64, TB_K = 32, NT = 256, NE = 32;

template <int ALG>
__device__ __forceinline__ float tmul(float a, float b) {
  return ALG == OM_MAXMUL ? a * b : a + b;
}
template <int ALG>
__device__ __forceinline__ float tfold(float acc, float p) {
  return ALG == OM_MINPLUS ? fminf(acc, p) : fmaxf(acc, p);
}
template <int ALG>
__device__ __forceinline__ bool improved(float now, float before) {
  return ALG == OM_MINPLUS ? (now < before) : (now > before);
}
// operand padding that never wins: -inf for max-plus, +inf for min-plus,
// 0 for max-mul (0*x = 0 never beats the zero() accumulator 0)
template <int ALG>
__device__ __forceinline__ float pad_value() {
  return ALG == OM_MAXPLUS ? -__int_as_float(0x7f800000)
                           : (ALG == OM_MINPLUS ? __int_as_float(0x7f800000) : 0.f);
}

struct FastArgs {
  int M, N, K, T;  // T = number of k slabs
  const float* A;
  int64_t lda, sab;  // A non-unit stride, batch stride
  const float* B;
  int64_t ldb, sbb;
  float* C;
  int64_t scm, scn, scb;
  uint32_t* argmax;
  const uint32_t* gate;
  uint32_t* ws;  // argmax: per-CTA, per-slab, per-thread improvement bitmasks
};

// Stages one 128 x 32 slab of A into As[k][m] and one 32 x 64 slab of B into
// Bs[k][n] through registers.
template <int ALG, bool A_MC, bool B_KC>
struct Stager {
  float4 ra[4], rb[2];

  __device__ __forceinline__ void load(const FastArgs& g, const float* Ab, const float* Bb, int m0,
                                       int n0, int k0, int tid) {
    const float pad = pad_value<ALG>();
    const float4 padv = make_float4(pad, pad, pad, pad);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int u = tid + r * NT;
      if (A_MC) {  // A[m + k*lda]: unit (k, 4 m)
        const int mq = u % 32, kk = u / 32;
        const int m = m0 + mq * 4, k = k0 + kk;
        ra[r] = (m < g.M && k < g.K) ? *(const float4*)(Ab + m + (int64_t)k * g.lda) : padv;
      } else {  // A[m*lda + k]: unit (m, 4 k)
        const int mm = u % TB_M, kq = u / TB_M;
        const int m = m0 + mm, k = k0 + kq * 4;
        ra[r] = (m < g.M && k < g.K) ? *(const float4*)(Ab + (int64_t)m * g.lda + k) : padv;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int u = tid + r * NT;
      if (B_KC) {  // B[k + n*ldb]: unit (n, 4 k)
        const int nn = u % TB_N, kq = u / TB_N;
        const int n = n0 + nn, k = k0 + kq * 4;
        rb[r] = (n < g.N && k < g.K) ? *(const float4*)(Bb + (int64_t)n * g.ldb + k) : padv;
      } else {  // B[k*ldb + n]: unit (k, 4 n)
        const int nq = u % 16, kk = u / 16;
        const int n = n0 + nq * 4, k = k0 + kk;
        rb[r] = (n < g.N && k < g.K) ? *(const float4*)(Bb + n + (int64_t)k * g.ldb) : padv;
      }
    }
  }

  __device__ __forceinline__ void store(float* As, float* Bs, int tid) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int u = tid + r * NT;
      if (A_MC) {
        const int mq = u % 32, kk = u / 32;
        *(float4*)(As + kk * TB_M + mq * 4) = ra[r];
      } else {
        const int mm = u % TB_M, kq = u / TB_M;
        As[(4 * kq + 0) * TB_M + mm] = ra[r].x;
        As[(4 * kq + 1) * TB_M + mm] = ra[r].y;
        As[(4 * kq + 2) * TB_M + mm] = ra[r].z;
        As[(4 * kq + 3) * TB_M + mm] = ra[r].w;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int u = tid + r * NT;
      if (B_KC) {
        const int nn = u % TB_N, kq = u / TB_N;
        Bs[(4 * kq + 0) * TB_N + nn] = rb[r].x;
        Bs[(4 * kq + 1) * TB_N + nn] = rb[r].y;
        Bs[(4 * kq + 2) * TB_N + nn] = rb[r].z;
        Bs[(4 * kq + 3) * TB_N + nn] = rb[r].w;
      } else {
        const int nq = u % 16, kk = u / 16;
        *(float4*)(Bs + kk * TB_N + nq * 4) = rb[r];
      }
    }
  }
};

// Thread (tx, ty) owns rows m = 4*tx + (i & 3) + 64*(i >> 2) (i < 8) and
// columns n = 4*ty + j (j < 4).  A warp spans 8 consecutive tx and 4
// consecutive ty, so each of its LDS.128 fragment loads touches one 128-byte
// line of shared memory (one wavefront).
__device__ __forceinline__ int row_of(int tx, int i) { return 4 * tx + (i & 3) + 64 * (i >> 2); }

template <int ALG, bool ARGMAX, bool A_MC, bool B_KC>
__global__ void __launch_bounds__(NT, 2) tropical_fast_kernel(FastArgs g) {
  if (fast_path_ruled_out(*g.gate, ALG)) return;
  extern __shared__ __align__(16) unsigned char smem[];
  float* As0 = (float*)smem;              // 2 x [TB_K][TB_M]
  float* Bs0 = As0 + 2 * TB_K * TB_M;     // 2 x [TB_K][TB_N]
  float* vals = Bs0 + 2 * TB_K * TB_N;    // [NE][NT] final values (ARGMAX)
  uint32_t* stage = (uint32_t*)(vals + NE * NT);  // [8 warps][2 * 32] resolve items

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tx = (warp & 1) * 8 + (lane & 7), ty = (warp >> 1) * 4 + (lane >> 3);
  const int m0 = blockIdx.x * TB_M, n0 = blockIdx.y * TB_N;
  const int bt = blockIdx.z;
  const float* Ab = g.A + bt * g.sab;
  const float* Bb = g.B + bt * g.sbb;
  // per-slab "improved" bitmasks of this CTA: [T][NT]
  uint32_t* masks = g.ws + ((size_t)(bt * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) *
                               (size_t)g.T * NT;

  float acc[8][4];
  const float z = Semi<ALG, float>::zero();
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = z;

  Stager<ALG, A_MC, B_KC> st;
  st.load(g, Ab, Bb, m0, n0, 0, tid);
  st.store(As0, Bs0, tid);
  __syncthreads();

  for (int t = 0; t < g.T; ++t) {
    const int buf = t & 1;
    if (t + 1 < g.T) st.load(g, Ab, Bb, m0, n0, (t + 1) * TB_K, tid);
    const float* As = As0 + buf * TB_K * TB_M;
    const float* Bs = Bs0 + buf * TB_K * TB_N;
    float before[8][4];
    if (ARGMAX) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) before[i][j] = acc[i][j];
    }
#pragma unroll 8
    for (int kk = 0; kk < TB_K; ++kk) {
      const float4 a0 = *(const float4*)(As + kk * TB_M + 4 * tx);
      const float4 a1 = *(const float4*)(As + kk * TB_M + 64 + 4 * tx);
      const float4 b0 = *(const float4*)(Bs + kk * TB_N + 4 * ty);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = tfold<ALG>(acc[i][j], tmul<ALG>(a[i], b[j]));
    }
    if (ARGMAX) {
      uint32_t bits = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (improved<ALG>(acc[i][j], before[i][j])) bits |= 1u << (i * 4 + j);
      masks[(size_t)t * NT + tid] = bits;
    }
    if (t + 1 < g.T) st.store(As0 + (buf ^ 1) * TB_K * TB_M, Bs0 + (buf ^ 1) * TB_K * TB_N, tid);
    __syncthreads();
  }

  const int64_t cbase = (int64_t)bt * g.scb;
  uint32_t remaining = 0xffffffffu;  // outputs whose deciding slab is not found yet
  if (ARGMAX) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) vals[(i * 4 + j) * NT + tid] = acc[i][j];
    uint32_t* items = stage + warp * 64;
    // Resolve pass, last slab first: the deciding slab of an output is the
    // last one whose bit is set.  Items of a slab are compacted across the
    // warp so every lane scans at most one output per round.
    if (g.T > 0) st.load(g, Ab, Bb, m0, n0, (g.T - 1) * TB_K, tid);
    for (int t = g.T - 1; t >= 0; --t) {
      const int buf = t & 1;
      float* As = As0 + buf * TB_K * TB_M;
      float* Bs = Bs0 + buf * TB_K * TB_N;
      st.store(As, Bs, tid);
      if (t > 0) st.load(g, Ab, Bb, m0, n0, (t - 1) * TB_K, tid);
      __syncthreads();
      uint32_t mine = masks[(size_t)t * NT + tid] & remaining;
      remaining &= ~mine;
      int cnt = __popc(mine);
      int pos = cnt;  // inclusive warp scan
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        int v = __shfl_up_sync(0xffffffffu, pos, d);
        if (lane >= d) pos += v;
      }
      const int total = __shfl_sync(0xffffffffu, pos, 31);
      int wr = pos - cnt;
      for (int done = 0; done < total; done += 64) {
        // write this lane's items that fall in [done, done + 64)
        uint32_t rest = mine;
        int p = wr;
        while (rest) {
          const int e = __ffs(rest) - 1;
          rest &= rest - 1;
          if (p >= done && p < done + 64) items[p - done] = ((uint32_t)lane << 5) | (uint32_t)e;
          ++p;
        }
        __syncwarp();
        for (int q = lane; q < min(64, total - done); q += 32) {
          const uint32_t it = items[q];
          const int src = (int)(it >> 5), e = (int)(it & 31);
          const int stx = (warp & 1) * 8 + (src & 7), sty = (warp >> 1) * 4 + (src >> 3);
          const int mi = row_of(stx, e >> 2), nj = 4 * sty + (e & 3);
          const float v = vals[e * NT + warp * 32 + src];
          int kb = 0;
          for (int kk = 0; kk < TB_K; ++kk) {
            if (tmul<ALG>(As[kk * TB_M + mi], Bs[kk * TB_N + nj]) == v) {
              kb = kk;
              break;
            }
          }
          const int m = m0 + mi, n = n0 + nj;
          if (m < g.M && n < g.N)
            g.argmax[cbase + (int64_t)m * g.scm + (int64_t)n * g.scn] = (uint32_t)(t * TB_K + kb);
        }
        __syncwarp();
      }
      __syncthreads();
    }
  }

#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + row_of(tx, i), n = n0 + 4 * ty + j;
      if (m < g.M && n < g.N) {
        const int64_t off = cbase + (int64_t)m * g.scm + (int64_t)n * g.scn;
        float v = acc[i][j];
        if (ALG == OM_MAXMUL && v == 0.f) v = 0.f;  // zero() is +0; a -0 product never wins
        g.C[off] = v;
        if (ARGMAX && (remaining >> (i * 4 + j)) & 1u) g.argmax[off] = 0u;
      }
    }
}

// ---------------------------------------------------------------------------
// special-value scan over the affine operand views
// ---------------------------------------------------------------------------
// An operand of the fast path is `lines` runs of `inner` unit-stride floats
// (inner % 4 == 0, 16-byte aligned), run l starting at (l % outer) * ld +
// (l / outer) * bs.
struct ScanArgs {
  const float* p;
  int inner, outer;
  int64_t ld, bs, lines;
  uint32_t pinf_bit, ninf_bit;
};

__device__ __forceinline__ uint32_t classify_bits(uint32_t u, uint32_t pinf_bit, uint32_t ninf_bit) {
  uint32_t f = 0;
  if ((u & 0x7fffffffu) > 0x7f800000u) f |= SV_NAN;
  if (u == 0x7f800000u) f |= pinf_bit;
  if (u == 0xff800000u) f |= ninf_bit;
  if (u == 0x80000000u) f |= SV_NEGZERO;
  return f;
}

// one CTA per group of runs, float4 loads along each run
__global__ void special_scan_kernel(ScanArgs s0, ScanArgs s1, uint32_t* flags) {
  uint32_t f = 0;
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const ScanArgs& s = w ? s1 : s0;
    const int vec = s.inner / 4;
    for (int64_t l = blockIdx.x; l < s.lines; l += gridDim.x) {
      const float4* run =
          (const float4*)(s.p + (l % s.outer) * s.ld + (l / s.outer) * s.bs);
      for (int v = threadIdx.x; v < vec; v += blockDim.x) {
        float4 x = run[v];
        f |= classify_bits(__float_as_uint(x.x), s.pinf_bit, s.ninf_bit) |
             classify_bits(__float_as_uint(x.y), s.pinf_bit, s.ninf_bit) |
             classify_bits(__float_as_uint(x.z), s.pinf_bit, s.ninf_bit) |
             classify_bits(__float_as_uint(x.w), s.pinf_bit, s.ninf_bit);
      }
    }
  }
  f = __reduce_or_sync(0xffffffffu, f);
  if ((threadIdx.x & 31) == 0 && f) atomicOr(flags, f);
}

template <int ALG, bool ARGMAX, bool A_MC, bool B_KC>
int launch_fast(om_backend* be, const FastArgs& fa, int64_t batch) {
  size_t smem = sizeof(float) * 2 * TB_K * (TB_M + TB_N) +
                (ARGMAX ? NE * NT * sizeof(float) + 8 * 64 * sizeof(uint32_t) : 0);
  auto kern = tropical_fast_kernel<ALG, ARGMAX, A_MC, B_KC>;
  OM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
          "cudaFuncSetAttribute");
  dim3 grid((fa.M + TB_M - 1) / TB_M, (fa.N + TB_N - 1) / TB_N, (unsigned)batch);
  ProfScope prof(be, ARGMAX ? "tropical_fast_argmax" : "tropical_fast");
  kern<<<grid, NT, smem, be->stream>>>(fa);
  note_launch();
  return check_cuda(cudaGetLastError(), "tropical_fast launch");
}

template <int ALG>
int launch_fast_alg(om_backend* be, const FastArgs& fa, int64_t batch, bool amc, bool bkc) {
  bool am = fa.argmax != nullptr;
#define OM_FAST_CASE(X, Y, Z) \
  if (am == X && amc == Y && bkc == Z) return launch_fast<ALG, X, Y, Z>(be, fa, batch);
  OM_FAST_CASE(true, true, true)
  OM_FAST_CASE(true, true, false)
  OM_FAST_CASE(true, false, true)
  OM_FAST_CASE(true, false, false)
  OM_FAST_CASE(false, true, true)
  OM_FAST_CASE(false, true, false)
  OM_FAST_CASE(false, false, true)
  OM_FAST_CASE(false, false, false)
#undef OM_FAST_CASE
  return set_error(OM_ERR_INVALID, "unreachable fast-path case");
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace

int launch_gemm_exact(om_backend* be, const GemmArgs& g);

// Takes the GEMM when the fast kernel applies (f32 tropical, large enough,
// one unit-stride axis per operand with 16-byte aligned vectors).  It then
// issues: flag reset, special-value scan, fast kernel (skips itself when the
// scan rules it out) and the exact kernel gated on the opposite condition.
int launch_gemm_tropical_fast(om_backend* be, const GemmArgs& g, bool* handled) {
  *handled = false;
  if (g.dtype != OM_F32 || g.alg == OM_STANDARD) return OM_OK;
  if (g.M < 64 || g.N < 64 || g.K < 32) return OM_OK;
  if (g.M > (1 << 30) || g.N > (1 << 30) || g.batch > 65535) return OM_OK;
  if (g.K > (1 << 30)) return OM_OK;
  bool amc, bkc;
  int64_t lda, ldb;
  if (g.sam == 1 && g.sak % 4 == 0 && g.M % 4 == 0) {
    amc = true;
    lda = g.sak;
  } else if (g.sak == 1 && g.sam % 4 == 0 && g.K % 4 == 0) {
    amc = false;
    lda = g.sam;
  } else {
    return OM_OK;
  }
  if (g.sbk == 1 && g.sbn % 4 == 0 && g.K % 4 == 0) {
    bkc = true;
    ldb = g.sbn;
  } else if (g.sbn == 1 && g.sbk % 4 == 0 && g.N % 4 == 0) {
    bkc = false;
    ldb = g.sbk;
  } else {
    return OM_OK;
  }
  if (!aligned16(g.A) || !aligned16(g.B) || (g.batch > 1 && (g.sab % 4 || g.sbb % 4))) return OM_OK;

  // special-value scan
  OM_CUDA(cudaMemsetAsync(be->d_flags, 0, sizeof(uint32_t), be->stream), "flag reset");
  ScanArgs sa, sb;
  sa.p = (const float*)g.A;
  sa.inner = (int)(amc ? g.M : g.K);
  sa.outer = (int)(amc ? g.K : g.M);
  sa.ld = lda;
  sa.bs = g.sab;
  sa.lines = (int64_t)sa.outer * g.batch;
  sa.pinf_bit = SV_A_PINF;
  sa.ninf_bit = SV_A_NINF;
  sb.p = (const float*)g.B;
  sb.inner = (int)(bkc ? g.K : g.N);
  sb.outer = (int)(bkc ? g.N : g.K);
  sb.ld = ldb;
  sb.bs = g.sbb;
  sb.lines = (int64_t)sb.outer * g.batch;
  sb.pinf_bit = SV_B_PINF;
  sb.ninf_bit = SV_B_NINF;
  int blocks = (int)std::min<int64_t>(std::max(sa.lines, sb.lines), (int64_t)be->num_sms * 8);
  {
    ProfScope prof(be, "special_scan");
    special_scan_kernel<<<std::max(blocks, 1), 128, 0, be->stream>>>(sa, sb, be->d_flags);
    note_launch();
    OM_CUDA(cudaGetLastError(), "special_scan launch");
  }

  FastArgs fa;
  fa.M = (int)g.M;
  fa.N = (int)g.N;
  fa.K = (int)g.K;
  fa.T = (int)((g.K + TB_K - 1) / TB_K);
  fa.A = (const float*)g.A;
  fa.lda = lda;
  fa.sab = g.sab;
  fa.B = (const float*)g.B;
  fa.ldb = ldb;
  fa.sbb = g.sbb;
  fa.C = (float*)g.C;
  fa.scm = g.scm;
  fa.scn = g.scn;
  fa.scb = g.scb;
  fa.argmax = g.argmax;
  fa.gate = be->d_flags;
  fa.ws = nullptr;
  Scratch ws;
  if (g.argmax) {
    const size_t ctas = (size_t)((g.M + TB_M - 1) / TB_M) * ((g.N + TB_N - 1) / TB_N) * g.batch;
    OM_TRY(ws.alloc(be, ctas * (size_t)fa.T * NT * sizeof(uint32_t)));
    fa.ws = (uint32_t*)ws.ptr;
  }
  switch (g.alg) {
    case OM_MAXPLUS: OM_TRY(launch_fast_alg<OM_MAXPLUS>(be, fa, g.batch, amc, bkc)); break;
    case OM_MINPLUS: OM_TRY(launch_fast_alg<OM_MINPLUS>(be, fa, g.batch, amc, bkc)); break;
    case OM_MAXMUL: OM_TRY(launch_fast_alg<OM_MAXMUL>(be, fa, g.batch, amc, bkc)); break;
    default: return OM_OK;
  }
  GemmArgs gated = g;
  gated.fast_gate = be->d_flags;
  OM_TRY(launch_gemm_exact(be, gated));
  *handled = true;
  return OM_OK;
}

}  // namespace om
