// K2: fast f32 tropical GEMM (MaxPlus / MinPlus / MaxMul) with fused argmax.
//
// Same result, bit for bit, as generic_gemm_with_argmax of the reference
// (tensor4all/omeinsum-rs src/backend/cpu/mod.rs:889-920, scalar rules in
// src/algebra/tropical.rs:57-63,93-104) on inputs for which no product is NaN
// or -0 (checked on the device by a special-value scan; otherwise the exact
// compare-select kernel runs, gated on the same flag word, with no host sync).
//
// Design (CUDA cores; tensor cores have no max/min).  One semiring step is an
// add (or multiply) and a max (or min).  Shared memory holds k-PAIRS (element
// (m, k..k+1) is one float2), so one packed `add.rn.f32x2` forms two products
// and one 3-input `max.f32` folds both into the accumulator: 2 instructions
// per 2 (i, j, k).  On B200 both forms occupy their pipe for two passes, but
// they need half the issue slots of scalar FADD + FMNMX, which leaves room
// for the fragment loads; measured, this form is about 25% faster.
//   * CTA tile 128 x 64, 256 threads, 8 x 4 outputs per thread (two CTAs per
//     SM), k slabs of 32 double-buffered in shared memory through registers,
//     so any of the four unit-stride orientations of A and B is read with
//     16-byte loads;
//   * lane layouts for which every fragment LDS.128 of a warp touches one
//     128-byte shared-memory line.
//
// Argmax without a per-k compare-select: after each slab one compare per
// output sets a bit when the running max strictly improved inside the slab;
// the 32-bit mask of a thread is written to a global workspace.  The last
// slab with the bit set holds the first k reaching the final max, because
// every earlier slab's max is strictly smaller.  A resolve pass buckets the
// tile's outputs by deciding slab (a counting sort across the CTA), re-stages
// only the slabs that decide something with cp.async (two stages), and scans
// each output once, in its deciding slab, for the first k with
// a (x) b == max; ties go to the smallest k and outputs that never beat
// zero() keep argmax 0, as in the reference.
#include <algorithm>

#include "om_internal.h"
#include "om_semiring.cuh"

namespace om {
namespace {

constexpr int TB_M = 128, TB_N = 64, TB_K = 32, NT = 256, NE = 32;
constexpr int kWin = 64;  // argmax resolve: slabs bucketed per window

__device__ __forceinline__ unsigned long long pk_add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long pk_mul(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float min3f(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ void unpack(unsigned long long s, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(s));
}

template <int ALG>
__device__ __forceinline__ float tmul(float a, float b) {
  return ALG == OM_MAXMUL ? a * b : a + b;
}
template <int ALG>
__device__ __forceinline__ unsigned long long tmul2(unsigned long long a, unsigned long long b) {
  return ALG == OM_MAXMUL ? pk_mul(a, b) : pk_add(a, b);
}
template <int ALG>
__device__ __forceinline__ float tfold3(float acc, float x, float y) {
  return ALG == OM_MINPLUS ? min3f(acc, x, y) : max3f(acc, x, y);
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
  int tiles, gx, gy, max_units;  // stream-K work split
  float* part_v;                 // [2 per CTA][NE][NT] piece values
  uint32_t* part_k;              // [2 per CTA][NE][NT] piece first winning k
  uint32_t* arrivals;            // [tiles] pieces of a cut tile finished so far
};

// float index of element (row, k) in a k-pair slab of width W
template <int W>
__device__ __forceinline__ int at(int row, int k) {
  return ((k >> 1) * W + row) * 2 + (k & 1);
}

// Stages one 128 x 32 slab of A and one 32 x 64 slab of B through registers
// (16 floats of A and 8 of B per thread) into the k-pair layout.
template <int ALG, bool A_MC, bool B_KC>
struct Stager {
  float4 ra[4], rb[2];

  __device__ __forceinline__ void load(const FastArgs& g, const float* Ab, const float* Bb, int m0,
                                       int n0, int k0, int tid) {
    const float pad = pad_value<ALG>();
    const float4 padv = make_float4(pad, pad, pad, pad);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      if (A_MC) {  // A[m + k*lda]: 512 (k-pair, m-quad) units, rows 2p and 2p+1
        const int q = (r >> 1) * NT + tid;
        const int mq = q % 32, kp = q / 32;
        const int m = m0 + mq * 4, k = k0 + 2 * kp + (r & 1);
        ra[r] = (m < g.M && k < g.K) ? *(const float4*)(Ab + m + (int64_t)k * g.lda) : padv;
      } else {  // A[m*lda + k]: unit = 4 k at one m
        const int u = tid + r * NT;
        const int mm = u % TB_M, kq = u / TB_M;
        const int m = m0 + mm, k = k0 + kq * 4;
        ra[r] = (m < g.M && k < g.K) ? *(const float4*)(Ab + (int64_t)m * g.lda + k) : padv;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (B_KC) {  // B[k + n*ldb]: unit = 4 k at one n
        const int u = tid + r * NT;
        const int nn = u % TB_N, kq = u / TB_N;
        const int n = n0 + nn, k = k0 + kq * 4;
        rb[r] = (n < g.N && k < g.K) ? *(const float4*)(Bb + (int64_t)n * g.ldb + k) : padv;
      } else {  // B[k*ldb + n]: 256 (k-pair, n-quad) units, rows 2p and 2p+1
        const int nq = tid % 16, kp = tid / 16;
        const int n = n0 + nq * 4, k = k0 + 2 * kp + r;
        rb[r] = (n < g.N && k < g.K) ? *(const float4*)(Bb + n + (int64_t)k * g.ldb) : padv;
      }
    }
  }

  __device__ __forceinline__ void store(float* As, float* Bs, int tid) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      if (A_MC) {
        if (r & 1) {
          const int q = (r >> 1) * NT + tid;
          const int mq = q % 32, kp = q / 32;
          const float4 x0 = ra[r - 1], x1 = ra[r];
          float4* d = (float4*)(As + at<TB_M>(mq * 4, 2 * kp));
          d[0] = make_float4(x0.x, x1.x, x0.y, x1.y);
          d[1] = make_float4(x0.z, x1.z, x0.w, x1.w);
        }
      } else {
        const int u = tid + r * NT;
        const int mm = u % TB_M, kq = u / TB_M;
        *(float2*)(As + at<TB_M>(mm, 4 * kq)) = make_float2(ra[r].x, ra[r].y);
        *(float2*)(As + at<TB_M>(mm, 4 * kq + 2)) = make_float2(ra[r].z, ra[r].w);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (B_KC) {
        const int u = tid + r * NT;
        const int nn = u % TB_N, kq = u / TB_N;
        *(float2*)(Bs + at<TB_N>(nn, 4 * kq)) = make_float2(rb[r].x, rb[r].y);
        *(float2*)(Bs + at<TB_N>(nn, 4 * kq + 2)) = make_float2(rb[r].z, rb[r].w);
      } else if (r == 1) {
        const int nq = tid % 16, kp = tid / 16;
        const float4 x0 = rb[0], x1 = rb[1];
        float4* d = (float4*)(Bs + at<TB_N>(nq * 4, 2 * kp));
        d[0] = make_float4(x0.x, x1.x, x0.y, x1.y);
        d[1] = make_float4(x0.z, x1.z, x0.w, x1.w);
      }
    }
  }
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem),
               "r"(valid ? 16 : 0));
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

// Re-stages a slab for the argmax resolve pass in the operands' natural
// layout: A as [k][m] (m-contiguous A) or [m][k]; B as [n][k] (k-contiguous
// B) or [k][n].  k-contiguous rows are padded to 36 floats so that lanes
// scanning different rows at the same k hit different banks.  Out-of-range
// chunks are zero-filled; the scan never reads them because it stops at K and
// only visits in-range outputs.
template <bool A_MC, bool B_KC>
struct ResolveStager {
  static constexpr int LD = TB_K + 4;
  static constexpr int A_FLOATS = A_MC ? TB_K * TB_M : TB_M * LD;
  static constexpr int B_FLOATS = B_KC ? TB_N * LD : TB_K * TB_N;
  static constexpr int STAGE = A_FLOATS + B_FLOATS;
  __device__ static __forceinline__ int a_at(int m, int k) { return A_MC ? k * TB_M + m : m * LD + k; }
  __device__ static __forceinline__ int b_at(int n, int k) { return B_KC ? n * LD + k : k * TB_N + n; }

  __device__ __forceinline__ void issue(const FastArgs& g, const float* Ab, const float* Bb, int m0,
                                        int n0, int t, float* RA, float* RB, int tid) {
    const int k0 = t * TB_K;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int c = tid + r * NT;
      const int m = A_MC ? 4 * (c % 32) : c / 8;
      const int k = A_MC ? c / 32 : 4 * (c % 8);
      const bool ok = (m0 + m < g.M) && (k0 + k < g.K);
      const float* src = ok ? (A_MC ? Ab + (m0 + m) + (int64_t)(k0 + k) * g.lda
                                    : Ab + (int64_t)(m0 + m) * g.lda + (k0 + k))
                            : Ab;
      cp_async16(RA + a_at(m, k), src, ok);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int c = tid + r * NT;
      const int n = B_KC ? c / 8 : 4 * (c % 16);
      const int k = B_KC ? 4 * (c % 8) : c / 16;
      const bool ok = (n0 + n < g.N) && (k0 + k < g.K);
      const float* src = ok ? (B_KC ? Bb + (int64_t)(n0 + n) * g.ldb + (k0 + k)
                                    : Bb + (n0 + n) + (int64_t)(k0 + k) * g.ldb)
                            : Bb;
      cp_async16(RB + b_at(n, k), src, ok);
    }
    asm volatile("cp.async.commit_group;");
  }
};

// floats at the start of shared memory shared by the main-loop slabs and the
// resolve stages
template <bool A_MC, bool B_KC>
__host__ __device__ constexpr int resolve_region() {
  return 2 * ResolveStager<A_MC, B_KC>::STAGE > 2 * TB_K * (TB_M + TB_N)
             ? 2 * ResolveStager<A_MC, B_KC>::STAGE
             : 2 * TB_K * (TB_M + TB_N);
}

// Output coordinates.  Warp w covers rows 64*(w & 1) + [0, 64) and columns
// 16*(w >> 1) + [0, 16); lane l = (lx = l & 7, ly = l >> 3).  Fragment loads
// of the 8 lx lanes are consecutive 16-byte chunks (one 128-byte line).
__device__ __forceinline__ int row_of(int warp, int lane, int i) {
  return 64 * (warp & 1) + 2 * (lane & 7) + (i & 1) + 16 * (i >> 1);
}
__device__ __forceinline__ int col_of(int warp, int lane, int j) {
  return 16 * (warp >> 1) + 2 * (lane >> 3) + (j & 1) + 8 * (j >> 1);
}

constexpr uint32_t kNoK = 0xffffffffu;  // partial piece that never beat zero()

// Persistent, stream-K work split: the (tile, slab) units of the whole GEMM
// are cut into gridDim.x equal contiguous ranges, one per CTA, so every CTA
// does the same amount of work whatever the tile count (no partly empty last
// wave).  A tile cut between CTAs is computed as pieces (slab ranges); each
// piece writes its value and first winning k to a partial slot, and the CTA
// whose piece arrives last (a per-tile atomic counter; nobody waits) merges
// the pieces in k order.
__device__ __forceinline__ int64_t unit_begin(int64_t c, int64_t W, int64_t G) { return c * W / G; }

// Merges the pieces of a tile that was cut between CTAs, in k order: a later
// piece replaces the running result only when strictly better, so the first k
// reaching the maximum wins, as in generic_gemm_with_argmax.  Run by the CTA
// that finishes the tile's last piece.
template <int ALG, bool ARGMAX>
__device__ __forceinline__ void merge_tile(const FastArgs& g, int tile, int64_t G, int warp,
                                           int lane, int tid) {
  const int64_t W = (int64_t)g.tiles * g.T;
  const int64_t ua = (int64_t)tile * g.T, ub = ua + g.T - 1;
  const int64_t c_first = ((ua + 1) * G + W - 1) / W - 1;  // owner of unit ua
  const int64_t c_last = ((ub + 1) * G + W - 1) / W - 1;
  const int bx = tile % g.gx, by = (tile / g.gx) % g.gy, bt = tile / (g.gx * g.gy);
  const int m0 = bx * TB_M, n0 = by * TB_N;
  const int64_t cbase = (int64_t)bt * g.scb;
  const float z = Semi<ALG, float>::zero();
  float best[NE];
  uint32_t kbest[NE];
#pragma unroll
  for (int e = 0; e < NE; ++e) {
    best[e] = z;
    kbest[e] = kNoK;
  }
  for (int64_t cc = c_first; cc <= c_last; ++cc) {
    const size_t base = (size_t)(cc * 2 + (unit_begin(cc, W, G) < ua ? 1 : 0)) * NE * NT + tid;
#pragma unroll
    for (int e = 0; e < NE; ++e) {
      const float v = __ldcg(g.part_v + base + (size_t)e * NT);
      if (ARGMAX) {
        const uint32_t k = __ldcg(g.part_k + base + (size_t)e * NT);
        if (k != kNoK && improved<ALG>(v, best[e])) {
          best[e] = v;
          kbest[e] = k;
        }
      } else {
        best[e] = (ALG == OM_MINPLUS) ? fminf(best[e], v) : fmaxf(best[e], v);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < NE; ++e) {
    const int m = m0 + row_of(warp, lane, e >> 2), n = n0 + col_of(warp, lane, e & 3);
    if (m < g.M && n < g.N) {
      const int64_t off = cbase + (int64_t)m * g.scm + (int64_t)n * g.scn;
      float v = best[e];
      if (ALG == OM_MAXMUL && v == 0.f) v = 0.f;
      g.C[off] = v;
      if (ARGMAX) g.argmax[off] = kbest[e] == kNoK ? 0u : kbest[e];
    }
  }
}

template <int ALG, bool ARGMAX, bool A_MC, bool B_KC>
__global__ void __launch_bounds__(NT, 2) tropical_fast_kernel(FastArgs g) {
  if (fast_path_ruled_out(*g.gate, ALG)) return;
  extern __shared__ __align__(16) unsigned char smem[];
  float* As0 = (float*)smem;           // 2 x TB_K*TB_M floats
  float* Bs0 = As0 + 2 * TB_K * TB_M;  // 2 x TB_K*TB_N floats
  float* vals = (float*)smem + resolve_region<A_MC, B_KC>();  // [NE][NT] (ARGMAX)
  uint32_t* kres = (uint32_t*)vals;  // resolved k of an output overwrites its value
  // resolve bookkeeping (ARGMAX): outputs bucketed by deciding slab
  uint16_t* items = (uint16_t*)(vals + NE * NT);            // [NE * NT] (thread << 5 | e)
  int* bcount = (int*)(items + NE * NT);  // [kWin + 2]: counts, then offsets; [kWin + 1]: list size
  int* bcur = bcount + kWin + 2;                            // [kWin] scatter cursors
  int* blist = bcur + kWin;                                 // [kWin] non-empty slabs, last first

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = row_of(warp, lane, 0), c0 = col_of(warp, lane, 0);
  // Work range of this CTA.  Value only: the two CTAs an SM holds (blocks b
  // and b + G/2 when the grid is two per SM) take neighbouring ranges, which
  // measured 2.4 % faster (their tiles overlap).  With argmax they keep
  // ranges G/2 apart, in the same phase of the tile: their resolve passes
  // coincide, so neither competes with the other's main loop for the
  // shared-memory pipe (measured 1.8 % faster than out of phase).
  const int64_t G = gridDim.x;
  const int64_t c = (!ARGMAX && G % 2 == 0)
                        ? (blockIdx.x < G / 2 ? 2 * (int64_t)blockIdx.x
                                              : 2 * ((int64_t)blockIdx.x - G / 2) + 1)
                        : (int64_t)blockIdx.x;
  const int64_t W = (int64_t)g.tiles * g.T;
  const int64_t u0 = unit_begin(c, W, G), u1 = unit_begin(c + 1, W, G);
  uint32_t* masks = g.ws + (size_t)c * g.max_units * NT;
  const float z = Semi<ALG, float>::zero();
  __shared__ bool last_piece;

  for (int64_t u = u0; u < u1;) {
    const int tile = (int)(u / g.T);
    const int tb = (int)(u % g.T);
    const int64_t rem_units = u1 - u;
    const int te = (int)(tb + rem_units < g.T ? tb + rem_units : g.T);
    u += te - tb;
    const int bx = tile % g.gx, by = (tile / g.gx) % g.gy, bt = tile / (g.gx * g.gy);
    const int m0 = bx * TB_M, n0 = by * TB_N;
    const float* Ab = g.A + bt * g.sab;
    const float* Bb = g.B + bt * g.sbb;

    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = z;

    Stager<ALG, A_MC, B_KC> st;
    __syncthreads();  // the previous piece may still read shared memory
    st.load(g, Ab, Bb, m0, n0, tb * TB_K, tid);
    st.store(As0, Bs0, tid);
    __syncthreads();

    for (int t = tb; t < te; ++t) {
      const int buf = (t - tb) & 1;
      if (t + 1 < te) st.load(g, Ab, Bb, m0, n0, (t + 1) * TB_K, tid);
      const float* As = As0 + buf * TB_K * TB_M;
      const float* Bs = Bs0 + buf * TB_K * TB_N;
      float before[8][4];
      if (ARGMAX) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) before[i][j] = acc[i][j];
      }
#pragma unroll 4
      for (int kp = 0; kp < TB_K / 2; ++kp) {
        const float* arow = As + kp * TB_M * 2 + 2 * r0;
        const float* brow = Bs + kp * TB_N * 2 + 2 * c0;
        unsigned long long a[8], b[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const ulonglong2 v = *(const ulonglong2*)(arow + 32 * q);
          a[2 * q] = v.x;
          a[2 * q + 1] = v.y;
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const ulonglong2 v = *(const ulonglong2*)(brow + 16 * q);
          b[2 * q] = v.x;
          b[2 * q + 1] = v.y;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float lo, hi;
            unpack(tmul2<ALG>(a[i], b[j]), lo, hi);
            acc[i][j] = tfold3<ALG>(acc[i][j], lo, hi);
          }
      }
      if (ARGMAX) {
        uint32_t bits = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (improved<ALG>(acc[i][j], before[i][j])) bits |= 1u << (i * 4 + j);
        masks[(size_t)(t - tb) * NT + tid] = bits;
      }
      if (t + 1 < te)
        st.store(As0 + (buf ^ 1) * TB_K * TB_M, Bs0 + (buf ^ 1) * TB_K * TB_N, tid);
      __syncthreads();
    }

    uint32_t remaining = 0xffffffffu;  // outputs whose deciding slab is not found yet
    if (ARGMAX) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) vals[(i * 4 + j) * NT + tid] = acc[i][j];
      // Resolve pass.  The deciding slab of an output is the last slab of the
      // piece whose improvement bit is set.  Windows of kWin slabs are taken
      // last first; in each, the outputs are bucketed by deciding slab (a
      // counting sort over the whole CTA), then only the slabs that decide
      // something are re-staged (cp.async, two stages) and every thread scans
      // at most one output of the slab per round for the first k whose
      // product equals the final value.  The found k replaces the output's
      // value in shared memory.
      using RS = ResolveStager<A_MC, B_KC>;
      RS rs;
      auto stA = [&](int q) { return (float*)smem + q * RS::STAGE; };
      auto stB = [&](int q) { return (float*)smem + q * RS::STAGE + RS::A_FLOATS; };
      for (int whi = te; whi > tb; whi -= kWin) {
        const int wlo = whi - kWin > tb ? whi - kWin : tb;
        const int wn = whi - wlo;
        for (int q = tid; q < kWin + 2; q += NT) bcount[q] = 0;
        __syncthreads();
        // pass 1: count the outputs each slab of the window decides (mask
        // words are fetched 16 at a time so their L2 latencies overlap)
        uint32_t rem = remaining;
        for (int t1 = whi; t1 > wlo && rem; t1 -= 16) {
          uint32_t mw[16];
#pragma unroll
          for (int x = 0; x < 16; ++x)
            mw[x] = (t1 - 1 - x >= wlo) ? __ldcg(masks + (size_t)(t1 - 1 - x - tb) * NT + tid) : 0u;
#pragma unroll
          for (int x = 0; x < 16; ++x) {
            const uint32_t m = mw[x] & rem;
            rem &= ~m;
            if (m) atomicAdd(bcount + (t1 - 1 - x - wlo), __popc(m));
          }
        }
        __syncthreads();
        if (warp == 0) {  // exclusive scan of the counts; list of non-empty slabs
          int carry = 0, nlist = 0;
          for (int base = 0; base < wn; base += 32) {
            const int q = base + lane;
            const int c = q < wn ? bcount[q] : 0;
            int x = c;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
              const int y = __shfl_up_sync(0xffffffffu, x, d);
              if (lane >= d) x += y;
            }
            if (q < wn) {
              bcount[q] = carry + x - c;
              bcur[q] = carry + x - c;
            }
            carry += __shfl_sync(0xffffffffu, x, 31);
            // non-empty slabs, highest first: slab wlo + q at list position
            // (number of non-empty slabs above it)
            const unsigned nz = __ballot_sync(0xffffffffu, c > 0);
            if (c > 0) blist[nlist + __popc(nz & ((1u << lane) - 1))] = q;
            nlist += __popc(nz);
          }
          if (lane == 0) {
            bcount[wn] = carry;  // end of the last bucket
            bcount[kWin + 1] = nlist;
          }
          // reverse the list in place so that it runs from the last slab down
          __syncwarp();
          for (int q = lane; q < nlist / 2; q += 32) {
            const int x = blist[q], y = blist[nlist - 1 - q];
            blist[q] = y;
            blist[nlist - 1 - q] = x;
          }
        }
        __syncthreads();
        // pass 2: scatter the outputs into their slab's bucket
        rem = remaining;
        for (int t1 = whi; t1 > wlo && rem; t1 -= 16) {
          uint32_t mw[16];
#pragma unroll
          for (int x = 0; x < 16; ++x)
            mw[x] = (t1 - 1 - x >= wlo) ? __ldcg(masks + (size_t)(t1 - 1 - x - tb) * NT + tid) : 0u;
#pragma unroll
          for (int x = 0; x < 16; ++x) {
            uint32_t m = mw[x] & rem;
            rem &= ~m;
            if (m) {
              int at = atomicAdd(bcur + (t1 - 1 - x - wlo), __popc(m));
              while (m) {
                const int e = __ffs(m) - 1;
                m &= m - 1;
                items[at++] = (uint16_t)((tid << 5) | e);
              }
            }
          }
        }
        remaining = rem;
        const int nlist = bcount[kWin + 1];
        __syncthreads();
        // re-stage and scan the deciding slabs, last first
        if (nlist > 0) rs.issue(g, Ab, Bb, m0, n0, wlo + blist[0], stA(0), stB(0), tid);
        for (int li = 0; li < nlist; ++li) {
          const int q = blist[li], t = wlo + q, s = li & 1;
          if (li + 1 < nlist) {
            rs.issue(g, Ab, Bb, m0, n0, wlo + blist[li + 1], stA(s ^ 1), stB(s ^ 1), tid);
            cp_async_wait<1>();
          } else {
            cp_async_wait<0>();
          }
          __syncthreads();
          const float* RA = stA(s);
          const float* RB = stB(s);
          const int b0 = bcount[q], b1 = bcount[q + 1];
          const int kmax = min(TB_K, g.K - t * TB_K);
          for (int x = b0 + tid; x < b1; x += NT) {
            const uint32_t it = items[x];
            const int src = (int)(it >> 5), e = (int)(it & 31);
            const int mi = row_of(src >> 5, src & 31, e >> 2), nj = col_of(src >> 5, src & 31, e & 3);
            const int slot = e * NT + src;
            const float v = vals[slot];
            int kb = 0;
#pragma unroll
            for (int kk = TB_K - 1; kk >= 0; --kk) {
              const float pr = tmul<ALG>(RA[RS::a_at(mi, kk)], RB[RS::b_at(nj, kk)]);
              if (kk < kmax && pr == v) kb = kk;
            }
            kres[slot] = (uint32_t)(t * TB_K + kb);
          }
          __syncthreads();
        }
      }
    }

    const bool whole = tb == 0 && te == g.T;
    const int64_t cbase = (int64_t)bt * g.scb;
    const int pslot = (int)(c * 2 + (tb == (int)(u0 % g.T) && tile == (int)(u0 / g.T) ? 0 : 1));
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int e = i * 4 + j;
        float v = acc[i][j];
        uint32_t k = kNoK;
        if (ARGMAX && !((remaining >> e) & 1u)) k = kres[e * NT + tid];
        if (whole) {
          const int m = m0 + row_of(warp, lane, i), n = n0 + col_of(warp, lane, j);
          if (m < g.M && n < g.N) {
            const int64_t off = cbase + (int64_t)m * g.scm + (int64_t)n * g.scn;
            if (ALG == OM_MAXMUL && v == 0.f) v = 0.f;  // zero() is +0; a -0 product never wins
            g.C[off] = v;
            if (ARGMAX) g.argmax[off] = k == kNoK ? 0u : k;
          }
        } else {
          g.part_v[((size_t)pslot * NE + e) * NT + tid] = v;
          if (ARGMAX) g.part_k[((size_t)pslot * NE + e) * NT + tid] = k;
        }
      }
    if (!whole) {
      // the CTA that finishes the last piece of the tile merges it (no wait)
      const int64_t ua = (int64_t)tile * g.T;
      const int64_t npieces = (((ua + g.T) * G + W - 1) / W - 1) - (((ua + 1) * G + W - 1) / W - 1) + 1;
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        const uint32_t prev = atomicAdd(g.arrivals + tile, 1u);
        last_piece = (prev + 1 == (uint32_t)npieces);
      }
      __syncthreads();
      if (last_piece) {
        __threadfence();
        merge_tile<ALG, ARGMAX>(g, tile, G, warp, lane, tid);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// special-value scan over the operands
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
  // one flat index space of 16-byte vectors per operand (line-major), walked
  // grid-stride with four independent loads in flight per thread, so short
  // lines do not leave threads idle
  uint32_t f = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    const ScanArgs& s = w ? s1 : s0;
    const int64_t vec = s.inner / 4, total = vec * s.lines;
    // a dense operand (lines back to back, batches back to back) is one run:
    // no index arithmetic per vector
    const bool flat = s.ld == s.inner && (s.lines <= s.outer || s.bs == (int64_t)s.inner * s.outer);
    auto at = [&](int64_t i) {
      if (flat) return ((const float4*)s.p)[i];
      const int64_t l = i / vec, v = i - l * vec;
      return ((const float4*)(s.p + (l % s.outer) * s.ld + (l / s.outer) * s.bs))[v];
    };
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    for (; i + 3 * stride < total; i += 4 * stride) {
      float4 x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) x[u] = at(i + u * stride);
#pragma unroll
      for (int u = 0; u < 4; ++u)
        f |= classify_bits(__float_as_uint(x[u].x), s.pinf_bit, s.ninf_bit) |
             classify_bits(__float_as_uint(x[u].y), s.pinf_bit, s.ninf_bit) |
             classify_bits(__float_as_uint(x[u].z), s.pinf_bit, s.ninf_bit) |
             classify_bits(__float_as_uint(x[u].w), s.pinf_bit, s.ninf_bit);
    }
    for (; i < total; i += stride) {
      const float4 x = at(i);
      f |= classify_bits(__float_as_uint(x.x), s.pinf_bit, s.ninf_bit) |
           classify_bits(__float_as_uint(x.y), s.pinf_bit, s.ninf_bit) |
           classify_bits(__float_as_uint(x.z), s.pinf_bit, s.ninf_bit) |
           classify_bits(__float_as_uint(x.w), s.pinf_bit, s.ninf_bit);
    }
  }
  f = __reduce_or_sync(0xffffffffu, f);
  if ((threadIdx.x & 31) == 0 && f) atomicOr(flags, f);
}

template <int ALG, bool ARGMAX, bool A_MC, bool B_KC>
int launch_fast(om_backend* be, const FastArgs& fa, int64_t grid_ctas) {
  const size_t smem =
      ARGMAX ? sizeof(float) * (resolve_region<A_MC, B_KC>() + NE * NT) +
                   sizeof(uint16_t) * NE * NT + sizeof(int) * (3 * kWin + 2)
             : sizeof(float) * 2 * TB_K * (TB_M + TB_N);
  auto kern = tropical_fast_kernel<ALG, ARGMAX, A_MC, B_KC>;
  OM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
          "cudaFuncSetAttribute");
  {
    ProfScope prof(be, ARGMAX ? "tropical_fast_argmax" : "tropical_fast");
    kern<<<(unsigned)grid_ctas, NT, smem, be->stream>>>(fa);
    note_launch();
    OM_CUDA(cudaGetLastError(), "tropical_fast launch");
  }
  return OM_OK;
}

template <int ALG>
int launch_fast_alg(om_backend* be, const FastArgs& fa, int64_t grid_ctas, bool amc, bool bkc) {
  const bool am = fa.argmax != nullptr;
#define OM_FAST_CASE(X, Y, Z) \
  if (am == X && amc == Y && bkc == Z) return launch_fast<ALG, X, Y, Z>(be, fa, grid_ctas);
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
static int launch_fast_impl(om_backend* be, const GemmArgs& g, bool* handled);

// C = A (x) B, or C^T = B^T (x) A^T when A has fewer than 64 rows and B at
// least 64 columns: the 64-wide side of the 128 x 64 tile then takes the
// short dimension (values and first-k argmax are the same: the products
// a (x) b and b (x) a are equal bit for bit).
int launch_gemm_tropical_fast(om_backend* be, const GemmArgs& g, bool* handled) {
  if (g.M < 64 && g.N >= 64) {
    GemmArgs t = g;
    t.M = g.N;
    t.N = g.M;
    t.A = g.B;
    t.sam = g.sbn;
    t.sak = g.sbk;
    t.sab = g.sbb;
    t.B = g.A;
    t.sbn = g.sam;
    t.sbk = g.sak;
    t.sbb = g.sab;
    t.scm = g.scn;
    t.scn = g.scm;
    t.ka1 = g.kb1;
    t.sak2 = g.sbk2;
    t.kb1 = g.ka1;
    t.sbk2 = g.sak2;
    t.ma1 = g.nb1;
    t.sam2 = g.sbn2;
    t.nb1 = g.ma1;
    t.sbn2 = g.sam2;
    return launch_fast_impl(be, t, handled);
  }
  return launch_fast_impl(be, g, handled);
}

static int launch_fast_impl(om_backend* be, const GemmArgs& g, bool* handled) {
  *handled = false;
  if (g.dtype != OM_F32 || g.alg == OM_STANDARD) return OM_OK;
  // flat (affine) k only: decoding a two-level k per slab here measured
  // 0.6-3 % slower on flat problems, so the planner gathers instead
  if (g.ka1 || g.kb1 || g.ma1 || g.nb1) return OM_OK;
  // the gate word is one per backend: concurrent graph branches would share
  // it, so they take the exact path
  if (be->branching) return OM_OK;
  // a short N (down to 16) wastes part of the tile's 64 columns, still far
  // ahead of the exact kernel on a long k
  if (g.M < 64 || g.N < 16 || g.K < 32) return OM_OK;
  if (g.M > (1 << 30) || g.N > (1 << 30) || g.K > (1 << 30) || g.batch > 65535) return OM_OK;
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
  const int64_t vecs = std::max(sa.lines * (sa.inner / 4), sb.lines * (sb.inner / 4));
  const int blocks = (int)std::min<int64_t>((vecs + 255) / 256, (int64_t)be->num_sms * 8);
  {
    ProfScope prof(be, "special_scan");
    special_scan_kernel<<<std::max(blocks, 1), 256, 0, be->stream>>>(sa, sb, be->d_flags);
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
  fa.gx = (int)((g.M + TB_M - 1) / TB_M);
  fa.gy = (int)((g.N + TB_N - 1) / TB_N);
  fa.tiles = (int)(fa.gx * fa.gy * g.batch);
  // two resident CTAs per SM, each with an equal share of the units
  const int64_t G = std::min<int64_t>(fa.tiles, 2 * (int64_t)be->num_sms);
  const int64_t W = (int64_t)fa.tiles * fa.T;
  fa.max_units = (int)((W + G - 1) / G + 1);
  Scratch ws, part;
  fa.ws = nullptr;
  fa.part_v = nullptr;
  fa.part_k = nullptr;
  if (g.argmax) {
    OM_TRY(ws.alloc(be, (size_t)G * fa.max_units * NT * sizeof(uint32_t)));
    fa.ws = (uint32_t*)ws.ptr;
  }
  fa.arrivals = nullptr;
  if (G < fa.tiles || W % G != 0) {
    const size_t pv = (size_t)G * 2 * NE * NT;
    OM_TRY(part.alloc(be, pv * (sizeof(float) + sizeof(uint32_t)) + (size_t)fa.tiles * sizeof(uint32_t)));
    fa.part_v = (float*)part.ptr;
    fa.part_k = (uint32_t*)(fa.part_v + pv);
    fa.arrivals = fa.part_k + pv;
    OM_CUDA(cudaMemsetAsync(fa.arrivals, 0, (size_t)fa.tiles * sizeof(uint32_t), be->stream),
            "arrival counters");
  }
  switch (g.alg) {
    case OM_MAXPLUS: OM_TRY(launch_fast_alg<OM_MAXPLUS>(be, fa, G, amc, bkc)); break;
    case OM_MINPLUS: OM_TRY(launch_fast_alg<OM_MINPLUS>(be, fa, G, amc, bkc)); break;
    case OM_MAXMUL: OM_TRY(launch_fast_alg<OM_MAXMUL>(be, fa, G, amc, bkc)); break;
    default: return OM_OK;
  }
  GemmArgs gated = g;
  gated.fast_gate = be->d_flags;
  OM_TRY(launch_gemm_exact(be, gated));
  *handled = true;
  return OM_OK;
}

}  // namespace om

// ---------------------------------------------------------------------------
// Allocation-free variant of the fast tropical GEMM with argmax.
//
// Some callers cannot allocate device memory while they run: code inside a
// host that owns all device memory through its own arena, real-time paths
// where a cudaMalloc / cudaMallocAsync could block or fail, and embedders that
// forbid the library any allocation of its own.  For them this entry point
// takes a caller's stream and plain column-major matrices and keeps the
// argmax kernel's scratch (per-slab improvement bitmasks, plus the flag word
// of the special-value gate) in fixed file-scope device arrays instead of the
// stream-ordered pool.  Every GPU that loads the library holds these arrays
// (32 MiB + 64 bytes) until the process exits.
// ---------------------------------------------------------------------------
#include <mutex>

namespace om {
namespace {

constexpr size_t kNoAllocMaskWords = (32u << 20) / sizeof(uint32_t);  // 32 MiB of masks
static __device__ __align__(256) uint32_t g_noalloc_masks[kNoAllocMaskWords];
static __device__ __align__(256) uint32_t g_noalloc_flag[16];

struct NoAllocSymbols {
  bool ready = false;
  uint32_t* masks = nullptr;
  uint32_t* flag = nullptr;
};

// Device addresses of the two arrays, looked up once per device with that
// device current (the host-side names are stand-ins, not device addresses).
int noalloc_symbols(int device, NoAllocSymbols* out) {
  static std::mutex mu;
  static NoAllocSymbols table[64];
  if (device < 0 || device >= 64) return set_error(OM_ERR_INVALID, "noalloc: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(mu);
  NoAllocSymbols& s = table[device];
  if (!s.ready) {
    OM_CUDA(cudaGetSymbolAddress((void**)&s.masks, g_noalloc_masks),
            "cudaGetSymbolAddress(noalloc masks)");
    OM_CUDA(cudaGetSymbolAddress((void**)&s.flag, g_noalloc_flag),
            "cudaGetSymbolAddress(noalloc flag)");
    s.ready = true;
  }
  *out = s;
  return OM_OK;
}

}  // namespace
}  // namespace om

extern "C" int om_b200_tropical_matmul_argmax_noalloc(void* stream, om_algebra alg, int64_t m,
                                                      int64_t n, int64_t k, const float* a,
                                                      int64_t lda, const float* b, int64_t ldb,
                                                      float* c, int64_t ldc, uint32_t* argmax) {
  using namespace om;
  if (!a || !b || !c || !argmax)
    return set_error(OM_ERR_INVALID, "om_b200_tropical_matmul_argmax_noalloc: null pointer");
  if (alg != OM_MAXPLUS && alg != OM_MINPLUS && alg != OM_MAXMUL)
    return set_error(OM_ERR_UNSUPPORTED,
                     "om_b200_tropical_matmul_argmax_noalloc: algebra must be MaxPlus, MinPlus or MaxMul");
  if (m < 0 || n < 0 || k < 1 || lda < std::max<int64_t>(m, 1) || ldb < k || ldc < std::max<int64_t>(m, 1))
    return set_error(OM_ERR_INVALID,
                     "om_b200_tropical_matmul_argmax_noalloc: bad sizes or leading dimensions");
  if (m == 0 || n == 0) return OM_OK;
  int device = 0;
  OM_CUDA(cudaGetDevice(&device), "cudaGetDevice");
  NoAllocSymbols sym;
  OM_TRY(noalloc_symbols(device, &sym));

  // a backend view over the caller's stream; it owns nothing
  om_backend view;
  view.device = device;
  view.stream = (cudaStream_t)stream;
  OM_CUDA(cudaDeviceGetAttribute(&view.num_sms, cudaDevAttrMultiProcessorCount, device),
          "cudaDeviceGetAttribute");
  view.d_flags = sym.flag;

  GemmArgs g{};
  g.alg = alg;
  g.dtype = OM_F32;
  g.M = m;
  g.N = n;
  g.K = k;
  g.batch = 1;
  g.A = a;
  g.sam = 1;
  g.sak = lda;
  g.B = b;
  g.sbk = 1;
  g.sbn = ldb;
  g.C = c;
  g.scm = 1;
  g.scn = ldc;
  g.argmax = argmax;

  const bool fast = m >= 64 && n >= 64 && k >= 32 && m <= (1 << 30) && n <= (1 << 30) &&
                    k <= (1 << 30) && m % 4 == 0 && k % 4 == 0 && lda % 4 == 0 && ldb % 4 == 0 &&
                    aligned16(a) && aligned16(b);
  if (!fast) return launch_gemm_exact(&view, g);  // no scratch on this path

  const int64_t gx = (m + TB_M - 1) / TB_M, gy = (n + TB_N - 1) / TB_N, T = (k + TB_K - 1) / TB_K;
  const int64_t words = gx * gy * T * NT;
  if (words > (int64_t)kNoAllocMaskWords)
    return set_error(OM_ERR_INVALID,
                     "om_b200_tropical_matmul_argmax_noalloc: ceil(m/128)*ceil(n/64)*ceil(k/32) = " +
                         std::to_string(gx * gy * T) + " exceeds the static workspace limit of " +
                         std::to_string(kNoAllocMaskWords / NT) +
                         " (32 MiB); use om_b200_contract for larger problems");

  // the gate flag must start at zero on every call; the masks need no
  // clearing (each is written before it is read)
  OM_CUDA(cudaMemsetAsync(sym.flag, 0, sizeof(uint32_t), view.stream), "noalloc flag reset");
  ScanArgs sa, sb;
  sa.p = a;
  sa.inner = (int)m;
  sa.outer = (int)k;
  sa.ld = lda;
  sa.bs = 0;
  sa.lines = k;
  sa.pinf_bit = SV_A_PINF;
  sa.ninf_bit = SV_A_NINF;
  sb.p = b;
  sb.inner = (int)k;
  sb.outer = (int)n;
  sb.ld = ldb;
  sb.bs = 0;
  sb.lines = n;
  sb.pinf_bit = SV_B_PINF;
  sb.ninf_bit = SV_B_NINF;
  const int blocks = (int)std::min<int64_t>(std::max(k, n), (int64_t)view.num_sms * 8);
  special_scan_kernel<<<std::max(blocks, 1), 128, 0, view.stream>>>(sa, sb, sym.flag);
  note_launch();
  OM_CUDA(cudaGetLastError(), "noalloc special_scan launch");

  FastArgs fa;
  fa.M = (int)m;
  fa.N = (int)n;
  fa.K = (int)k;
  fa.T = (int)T;
  fa.A = a;
  fa.lda = lda;
  fa.sab = 0;
  fa.B = b;
  fa.ldb = ldb;
  fa.sbb = 0;
  fa.C = c;
  fa.scm = 1;
  fa.scn = ldc;
  fa.scb = 0;
  fa.argmax = argmax;
  fa.gate = sym.flag;
  fa.ws = sym.masks;
  // one CTA per tile: no tile is cut, so no partial buffers are needed
  fa.gx = (int)gx;
  fa.gy = (int)gy;
  fa.tiles = (int)(gx * gy);
  fa.max_units = (int)T;
  fa.part_v = nullptr;
  fa.part_k = nullptr;
  fa.arrivals = nullptr;
  switch (alg) {
    case OM_MAXPLUS: OM_TRY((launch_fast<OM_MAXPLUS, true, true, true>(&view, fa, fa.tiles))); break;
    case OM_MINPLUS: OM_TRY((launch_fast<OM_MINPLUS, true, true, true>(&view, fa, fa.tiles))); break;
    default: OM_TRY((launch_fast<OM_MAXMUL, true, true, true>(&view, fa, fa.tiles))); break;
  }
  GemmArgs gated = g;
  gated.fast_gate = sym.flag;
  return launch_gemm_exact(&view, gated);
}
