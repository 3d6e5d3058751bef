// Exact semiring GEMM kernels for every algebra / dtype / affine layout.
//
// They restate generic_gemm / generic_gemm_with_argmax and their batched
// forms (tensor4all/omeinsum-rs src/backend/cpu/mod.rs:414-488, 862-920)
// with the same per-element compare-select, so NaN and signed-zero behaviour
// and the first-k tie rule match the reference exactly.  Standard algebra
// accumulates with fused multiply-add (the reference calls faer; parity for
// Standard is to a stated tolerance).
//
// Two shapes of kernel:
//   gemm_tiled  64x64 output tile per CTA, 16-deep k slabs staged in shared
//               memory, 4x4 outputs per thread; any strides, any batch;
//   gemm_small  one thread per output element, k loop straight from global
//               memory; for the tiny, heavily batched GEMMs of tensor-network
//               nodes (bond dimension 2), where a tile would be mostly idle.
#include <algorithm>
#include <type_traits>

#include "om_internal.h"
#include "om_semiring.cuh"

namespace om {

int launch_gemm_tropical_fast(om_backend* be, const GemmArgs& g, bool* handled);
int launch_gemm_tf32(om_backend* be, const GemmArgs& g, bool* handled);

namespace {

constexpr int BM = 64, BN = 64, BK = 16, TM = 4, TN = 4;

template <typename T, int ALG, bool ARGMAX>
__global__ void __launch_bounds__(256) gemm_tiled(GemmArgs g) {
  using S = Semi<ALG, T>;
  if (g.fast_gate && !fast_path_ruled_out(*g.fast_gate, ALG)) return;
  __shared__ T As[BK][BM];
  __shared__ T Bs[BK][BN];
  const T* __restrict__ A = (const T*)g.A;
  const T* __restrict__ B = (const T*)g.B;
  T* __restrict__ C = (T*)g.C;
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;
  for (int64_t bt = blockIdx.z; bt < g.batch; bt += gridDim.z) {
    const T* Ab = A + bt * g.sab;
    const T* Bb = B + bt * g.sbb;
    T acc[TM][TN];
    uint32_t idx[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        acc[i][j] = S::zero();
        idx[i][j] = 0;
      }
    for (int64_t k0 = 0; k0 < g.K; k0 += BK) {
      const int kc = (int)(g.K - k0 < BK ? g.K - k0 : BK);
      __syncthreads();
#pragma unroll
      for (int r = 0; r < (BM * BK) / 256; ++r) {
        int e = tid + r * 256;
        int mm = e % BM, kk = e / BM;
        int64_t m = m0 + mm, k = k0 + kk;
        As[kk][mm] = (m < g.M && kk < kc) ? Ab[m * g.sam + kofs(k, g.sak, g.ka1, g.sak2)] : T(0);
      }
#pragma unroll
      for (int r = 0; r < (BN * BK) / 256; ++r) {
        int e = tid + r * 256;
        int kk = e % BK, nn = e / BK;
        int64_t n = n0 + nn, k = k0 + kk;
        Bs[kk][nn] = (n < g.N && kk < kc) ? Bb[kofs(k, g.sbk, g.kb1, g.sbk2) + n * g.sbn] : T(0);
      }
      __syncthreads();
#pragma unroll 4
      for (int kk = 0; kk < kc; ++kk) {
        T a[TM], b[TN];
#pragma unroll
        for (int i = 0; i < TM; ++i) a[i] = As[kk][tx * TM + i];
#pragma unroll
        for (int j = 0; j < TN; ++j) b[j] = Bs[kk][ty * TN + j];
        const uint32_t kg = (uint32_t)(k0 + kk);
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) {
            if (ALG == OM_STANDARD) {
              acc[i][j] = fma(a[i], b[j], acc[i][j]);
            } else {
              T p = S::mul(a[i], b[j]);
              if (!S::keep(acc[i][j], p)) {
                acc[i][j] = p;
                if (ARGMAX) idx[i][j] = kg;
              }
            }
          }
      }
    }
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        int64_t m = m0 + tx * TM + i, n = n0 + ty * TN + j;
        if (m < g.M && n < g.N) {
          int64_t off = m * g.scm + n * g.scn + bt * g.scb;
          C[off] = acc[i][j];
          if (ARGMAX) g.argmax[off] = (ALG == OM_STANDARD) ? 0u : idx[i][j];
        }
      }
  }
}

template <typename T, int ALG, bool ARGMAX>
__global__ void __launch_bounds__(256) gemm_small(GemmArgs g, int64_t total, FastDiv dm,
                                                  FastDiv dn) {
  using S = Semi<ALG, T>;
  if (g.fast_gate && !fast_path_ruled_out(*g.fast_gate, ALG)) return;
  const T* __restrict__ A = (const T*)g.A;
  const T* __restrict__ B = (const T*)g.B;
  T* __restrict__ C = (T*)g.C;
  const bool idx32 = total < (int64_t(1) << 32);
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t m, n, bt;
    if (idx32) {  // multiply-high divisions instead of 64-bit ones
      const uint32_t e32 = (uint32_t)e, r = fast_div(e32, dm), q = fast_div(r, dn);
      m = e32 - r * dm.d;
      n = r - q * dn.d;
      bt = q;
    } else {
      m = e % g.M;
      const int64_t r = e / g.M;
      n = r % g.N;
      bt = r / g.N;
    }
    const T* a = A + m * g.sam + bt * g.sab;
    const T* b = B + n * g.sbn + bt * g.sbb;
    T acc = S::zero();
    uint32_t idx = 0;
    for (int64_t k = 0; k < g.K; ++k) {
      T av = a[kofs(k, g.sak, g.ka1, g.sak2)], bv = b[kofs(k, g.sbk, g.kb1, g.sbk2)];
      if (ALG == OM_STANDARD) {
        acc = fma(av, bv, acc);
      } else {
        T p = S::mul(av, bv);
        if (!S::keep(acc, p)) {
          acc = p;
          idx = (uint32_t)k;
        }
      }
    }
    int64_t off = m * g.scm + n * g.scn + bt * g.scb;
    C[off] = acc;
    if (ARGMAX) g.argmax[off] = (ALG == OM_STANDARD) ? 0u : idx;
  }
}

// gemm_node: a node read in place through per-mode strides.  Contracted
// offsets (K <= kNodeKTable) and the offsets of the tile's low output modes
// are tabulated in shared memory once per block; each tile row decodes its
// high modes once with 32-bit multiply-high divisions.  A thread takes V
// consecutive outputs at a time (V = 4 when the first output mode allows it:
// their operand offsets step by that mode's strides and the outputs leave as
// one 16-byte store), so the per-output index work is a few integer adds.
// The output is written at its linear index (contiguous, coalesced).
constexpr int kNodeKTable = 512, kNodeQuads = 1024, kNodeRep = 64;

template <int V, typename T>
__device__ __forceinline__ void store_v(T* p, const T (&v)[V]) {
  if constexpr (V == 4 && sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else if constexpr (V == 4 && sizeof(T) == 8) {
    reinterpret_cast<double2*>(p)[0] = make_double2(v[0], v[1]);
    reinterpret_cast<double2*>(p)[1] = make_double2(v[2], v[3]);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = v[i];
  }
}

__device__ __forceinline__ void store_idx(uint32_t* p, const uint32_t (&v)[4]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void store_idx(uint32_t* p, const uint32_t (&v)[1]) { p[0] = v[0]; }

// The V values of a group at p + off[i]: one 16-byte load when they are
// contiguous (w = 4), two 8/16-byte loads for two pairs (w = 2), one load
// when all four coincide (w = 0, a broadcast operand), two scalar loads
// when they are x x y y (w = 3) or x y x y (w = 5: the operand lacks one
// of the group's two modes), else four scalar loads.  The launcher grants
// w = 4 / 2 only when every group start is aligned.
template <int V, typename T>
__device__ __forceinline__ void load_group(const T* p, const int64_t (&off)[4], int w,
                                           T (&out)[V]) {
  if constexpr (V == 4) {
    if (w == 0) {
      out[0] = out[1] = out[2] = out[3] = p[0];
      return;
    }
    if (w == 3) {
      out[0] = out[1] = p[0];
      out[2] = out[3] = p[off[2]];
      return;
    }
    if (w == 5) {
      out[0] = out[2] = p[0];
      out[1] = out[3] = p[off[1]];
      return;
    }
    if (w == 4) {
      if constexpr (sizeof(T) == 4) {
        const float4 v = *reinterpret_cast<const float4*>(p);
        out[0] = v.x, out[1] = v.y, out[2] = v.z, out[3] = v.w;
      } else {
        const double2 v0 = reinterpret_cast<const double2*>(p)[0];
        const double2 v1 = reinterpret_cast<const double2*>(p)[1];
        out[0] = v0.x, out[1] = v0.y, out[2] = v1.x, out[3] = v1.y;
      }
      return;
    }
    if (w == 2) {
      if constexpr (sizeof(T) == 4) {
        const float2 v0 = *reinterpret_cast<const float2*>(p);
        const float2 v1 = *reinterpret_cast<const float2*>(p + off[2]);
        out[0] = v0.x, out[1] = v0.y, out[2] = v1.x, out[3] = v1.y;
      } else {
        const double2 v0 = *reinterpret_cast<const double2*>(p);
        const double2 v1 = *reinterpret_cast<const double2*>(p + off[2]);
        out[0] = v0.x, out[1] = v0.y, out[2] = v1.x, out[3] = v1.y;
      }
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < V; ++i) out[i] = p[off[i]];
}

// Blocks per SM for a gemm_node variant: it holds k * V values of A and
// min(k, 4) * V of B in registers (k = KT, or the chunk of four of the
// generic path) besides its state (about 36 registers with the loop over
// B's own row modes; 64 for single outputs, which keep 64-bit offsets),
// which sets the register cap.
template <typename T, int KT, int V>
constexpr int node_min_blocks() {
  constexpr int k = KT == 0 ? 4 : KT;
  constexpr int regs = (k + (k < 4 ? k : 4)) * V * (int)(sizeof(T) / 4) + (V == 1 ? 64 : 36);
  constexpr int b = 65536 / (256 * regs);
  return b > 8 ? 8 : (b < 2 ? 2 : b);
}

template <typename T, int ALG, bool ARGMAX, int KT, int V>
__global__ void __launch_bounds__(256, (node_min_blocks<T, KT, V>())) gemm_node(NodeArgs g) {
  using S = Semi<ALG, T>;
  // four-output groups run on 32-bit offsets (the launcher checks that
  // every offset of both operands fits); single outputs keep 64-bit ones
  using Off = std::conditional_t<V == 4, int32_t, int64_t>;
  __shared__ Off ka[kNodeKTable], kb[kNodeKTable];
  __shared__ Off la[kNodeQuads], lb[kNodeQuads];
  __shared__ int64_t rc[kNodeRep];
  __shared__ Off rb[kNodeRep];
  const int tid = threadIdx.x;
  const int R = KT > 0 && g.R > 1 ? g.R : 1;
  if (KT > 0)
    for (int q0 = tid; q0 < R; q0 += blockDim.x) {
      uint32_t r = (uint32_t)q0;
      int64_t oc = 0;
      Off ob = 0;
      for (int j = g.nlow; j < g.nlow + g.nrep; ++j) {
        const uint32_t q = fast_div(r, g.out[j].div);
        const uint32_t d = r - q * g.out[j].div.d;
        oc += (int64_t)d * g.out[j].sc;
        ob += (Off)d * (Off)g.out[j].sb;
        r = q;
      }
      rc[q0] = oc;
      rb[q0] = ob;
    }
  const bool ktab = g.K <= kNodeKTable;
  if (ktab)
    for (int k = tid; k < (int)g.K; k += blockDim.x) {
      uint32_t r = (uint32_t)k;
      Off oa = 0, ob = 0;
      for (int j = 0; j < g.nk; ++j) {
        const uint32_t q = fast_div(r, g.kmodes[j].div);
        const uint32_t d = r - q * g.kmodes[j].div.d;
        oa += (Off)d * (Off)g.kmodes[j].sa;
        ob += (Off)d * (Off)g.kmodes[j].sb;
        r = q;
      }
      ka[k] = oa;
      kb[k] = ob;
    }
  const int Q = g.P / V;  // groups of V outputs in a tile row
  for (int q0 = tid; q0 < Q; q0 += blockDim.x) {
    uint32_t r = (uint32_t)(q0 * V);
    Off oa = 0, ob = 0;
    for (int j = 0; j < g.nlow; ++j) {
      const uint32_t q = fast_div(r, g.out[j].div);
      const uint32_t d = r - q * g.out[j].div.d;
      oa += (Off)d * (Off)g.out[j].sa;
      ob += (Off)d * (Off)g.out[j].sb;
      r = q;
    }
    la[q0] = oa;
    lb[q0] = ob;
  }
  __syncthreads();
  const T* __restrict__ A = (const T*)g.A;
  const T* __restrict__ B = (const T*)g.B;
  T* __restrict__ C = (T*)g.C;
  // rows per block iteration: one when the row fills the block, else several
  const int rpi = Q >= 256 ? 1 : 256 / Q;
  const int sub = Q >= 256 ? 0 : tid / Q;
  const int q_first = Q >= 256 ? tid : tid % Q;
  const int q_step = Q >= 256 ? 256 : Q;
  if (sub >= rpi) return;
  for (int64_t r0 = (int64_t)blockIdx.x * rpi; r0 < g.rows; r0 += (int64_t)gridDim.x * rpi) {
    const int64_t row = r0 + sub;
    if (row >= g.rows) break;
    uint32_t r = (uint32_t)row;
    Off ha = 0, hb = 0;
    int64_t hc = 0;
    for (int j = g.nlow + (KT > 0 ? g.nrep : 0); j < g.nout; ++j) {
      const uint32_t q = fast_div(r, g.out[j].div);
      const uint32_t d = r - q * g.out[j].div.d;
      ha += (Off)d * (Off)g.out[j].sa;
      hb += (Off)d * (Off)g.out[j].sb;
      hc += (int64_t)d * g.out[j].sc;
      r = q;
    }
    for (int q = q_first; q < Q; q += q_step) {
      const T* a = A + (int64_t)(ha + la[q]);
      const T* b = B + (int64_t)(hb + lb[q]);
      T acc[V];
      uint32_t idx[V];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        acc[i] = S::zero();
        idx[i] = 0;
      }
      if constexpr (KT > 0) {
        // K == KT: A's values are loaded once and serve the R row
        // combinations of B's own modes; every load is issued before use
        T av[KT][V];
#pragma unroll
        for (int k = 0; k < KT; ++k) load_group<V>(a + ka[k], g.ia, g.wa, av[k]);
        constexpr int KC = KT < 4 ? KT : 4;  // B's values in chunks of k
        for (int rr = 0; rr < R; ++rr) {
          const T* br = b + (int64_t)rb[rr];
#pragma unroll
          for (int i = 0; i < V; ++i) {
            acc[i] = S::zero();
            idx[i] = 0;
          }
#pragma unroll
          for (int k0 = 0; k0 < KT; k0 += KC) {
            T bv[KC][V];
#pragma unroll
            for (int k = 0; k < KC; ++k) load_group<V>(br + kb[k0 + k], g.ib, g.wb, bv[k]);
#pragma unroll
            for (int k = 0; k < KC; ++k)
#pragma unroll
              for (int i = 0; i < V; ++i) {
                if (ALG == OM_STANDARD) {
                  acc[i] = fma(av[k0 + k][i], bv[k][i], acc[i]);
                } else {
                  const T p = S::mul(av[k0 + k][i], bv[k][i]);
                  if (!S::keep(acc[i], p)) {
                    acc[i] = p;
                    idx[i] = (uint32_t)(k0 + k);
                  }
                }
              }
          }
          const int64_t e = hc + rc[rr] + (int64_t)q * V;
          store_v<V>(C + e, acc);
          if (ARGMAX) {
            if (ALG == OM_STANDARD) {
#pragma unroll
              for (int i = 0; i < V; ++i) idx[i] = 0;
            }
            store_idx(g.argmax + e, idx);
          }
        }
        continue;
      } else if (ktab) {
        // tabulated k in chunks of four: the chunk's loads go out together
        // and a group of V outputs loads as one vector where it can
        for (int k0 = 0; k0 < (int)g.K; k0 += 4) {
          const int kn = (int)g.K - k0 < 4 ? (int)g.K - k0 : 4;
          T av[4][V], bv[4][V];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (k < kn) {
              load_group<V>(a + ka[k0 + k], g.ia, g.wa, av[k]);
              load_group<V>(b + kb[k0 + k], g.ib, g.wb, bv[k]);
            }
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (k < kn) {
#pragma unroll
              for (int i = 0; i < V; ++i) {
                if (ALG == OM_STANDARD) {
                  acc[i] = fma(av[k][i], bv[k][i], acc[i]);
                } else {
                  const T p = S::mul(av[k][i], bv[k][i]);
                  if (!S::keep(acc[i], p)) {
                    acc[i] = p;
                    idx[i] = (uint32_t)(k0 + k);
                  }
                }
              }
            }
        }
      } else {
        for (int64_t k = 0; k < g.K; ++k) {
          int64_t xa, xb;
          {
            xa = xb = 0;
            uint32_t rk = (uint32_t)k;
            for (int j = 0; j < g.nk; ++j) {
              const uint32_t qq = fast_div(rk, g.kmodes[j].div);
              const uint32_t d = rk - qq * g.kmodes[j].div.d;
              xa += (int64_t)d * g.kmodes[j].sa;
              xb += (int64_t)d * g.kmodes[j].sb;
              rk = qq;
            }
          }
#pragma unroll
          for (int i = 0; i < V; ++i) {
            const T av = a[xa + g.ia[i]], bv = b[xb + g.ib[i]];
            if (ALG == OM_STANDARD) {
              acc[i] = fma(av, bv, acc[i]);
            } else {
              const T p = S::mul(av, bv);
              if (!S::keep(acc[i], p)) {
                acc[i] = p;
                idx[i] = (uint32_t)k;
              }
            }
          }
        }
      }
      const int64_t e = hc + (int64_t)q * V;
      store_v<V>(C + e, acc);
      if (ARGMAX) {
        if (ALG == OM_STANDARD) {
#pragma unroll
          for (int i = 0; i < V; ++i) idx[i] = 0;
        }
        store_idx(g.argmax + e, idx);
      }
    }
  }
}

template <typename T, int ALG>
int launch_node_typed(om_backend* be, const NodeArgs& g, int vec) {
  const int Q = g.P / vec;
  const int rpi = Q >= 256 ? 1 : 256 / Q;
  int64_t blocks = std::min<int64_t>((g.rows + rpi - 1) / rpi, (int64_t)be->num_sms * 8);
  if (blocks < 1) blocks = 1;
  ProfScope prof(be, "gemm_node");
  auto go = [&](auto am, auto kt, auto v) {
    gemm_node<T, ALG, decltype(am)::value, decltype(kt)::value, decltype(v)::value>
        <<<(int)blocks, 256, 0, be->stream>>>(g);
  };
  auto with_v = [&](auto am, auto kt) {
    if (vec == 4) go(am, kt, std::integral_constant<int, 4>{});
    else go(am, kt, std::integral_constant<int, 1>{});
  };
  auto with_k = [&](auto am) {
    switch (g.K) {
      case 1: with_v(am, std::integral_constant<int, 1>{}); break;
      case 2: with_v(am, std::integral_constant<int, 2>{}); break;
      case 4: with_v(am, std::integral_constant<int, 4>{}); break;
      case 8:
        if constexpr (sizeof(T) == 4) {
          with_v(am, std::integral_constant<int, 8>{});
          break;
        }
        [[fallthrough]];
      default: with_v(am, std::integral_constant<int, 0>{}); break;
    }
  };
  if (g.argmax) with_k(std::true_type{});
  else with_k(std::false_type{});
  note_launch();
  return check_cuda(cudaGetLastError(), "gemm_node launch");
}

template <typename T, int ALG>
int launch_typed(om_backend* be, const GemmArgs& g) {
  const int64_t outputs = g.M * g.N * g.batch;
  // thread per output: tiny tiles, and k too short for a tile's reuse to pay
  const bool small = (g.M * g.N <= 1024) || g.M < 16 || g.N < 16 || g.K <= 8;
  ProfScope prof(be, small ? "gemm_exact_small" : "gemm_exact_tiled");
  if (small) {
    int64_t blocks = std::min<int64_t>((outputs + 255) / 256, (int64_t)be->num_sms * 64);
    if (blocks < 1) blocks = 1;
    FastDiv dm{}, dn{};
    if (outputs < (int64_t(1) << 32)) {
      dm = make_fastdiv((uint32_t)g.M);
      dn = make_fastdiv((uint32_t)g.N);
    }
    if (g.argmax)
      gemm_small<T, ALG, true><<<(int)blocks, 256, 0, be->stream>>>(g, outputs, dm, dn);
    else
      gemm_small<T, ALG, false><<<(int)blocks, 256, 0, be->stream>>>(g, outputs, dm, dn);
  } else {
    dim3 grid((unsigned)((g.M + BM - 1) / BM), (unsigned)((g.N + BN - 1) / BN),
              (unsigned)std::min<int64_t>(g.batch, 65535));
    if (grid.y > 65535) return set_error(OM_ERR_UNSUPPORTED, "gemm: N too large for tiled grid");
    if (g.argmax)
      gemm_tiled<T, ALG, true><<<grid, 256, 0, be->stream>>>(g);
    else
      gemm_tiled<T, ALG, false><<<grid, 256, 0, be->stream>>>(g);
  }
  note_launch();
  return check_cuda(cudaGetLastError(), "gemm launch");
}

}  // namespace

int launch_gemm_exact(om_backend* be, const GemmArgs& g) {
  if (g.dtype == OM_F32) {
    OM_DISPATCH_ALG(g.alg, ALG, return launch_typed<float, ALG>(be, g));
  } else if (g.dtype == OM_F64) {
    OM_DISPATCH_ALG(g.alg, ALG, return launch_typed<double, ALG>(be, g));
  }
  return set_error(OM_ERR_UNSUPPORTED, "gemm: dtype must be f32 or f64");
}

// A node with few outputs and a long contracted range (the root of a network
// is often a dot product of two large intermediates; annealed trees also
// contract two large intermediates into a few thousand outputs): one CTA per
// output, the threads interleaved over k so that a warp reads consecutive
// k.  The offsets of the low contracted modes (up to kSplitTable k values)
// sit in a shared-memory table; the high modes are decoded once per table
// pass.  Tropical: each thread keeps its first best element (strict
// improvement, k visited in increasing order), and the merge takes the
// better value, then the smaller k -- the first k reaching the maximum, as
// the sequential rule of generic_gemm_with_argmax gives.  A NaN product
// breaks that equivalence (the sequential rule lets a NaN replace the
// accumulator and the next product replace the NaN), so an output that meets
// one is recomputed sequentially by thread 0.  Standard: a tree sum.
constexpr int kSplitThreads = 256, kSplitTable = 2048;

template <typename T, int ALG, bool ARGMAX>
__global__ void __launch_bounds__(kSplitThreads) gemm_node_splitk(NodeArgs g, int nklo,
                                                                  int64_t klo) {
  using S = Semi<ALG, T>;
  __shared__ int64_t ta[kSplitTable], tb[kSplitTable];
  __shared__ T sv[kSplitThreads / 32];
  __shared__ int64_t sk[kSplitThreads / 32];
  __shared__ int snan;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int k = tid; k < (int)klo; k += kSplitThreads) {
    uint32_t r = (uint32_t)k;
    int64_t xa = 0, xb = 0;
    for (int j = 0; j < nklo; ++j) {
      const uint32_t q = fast_div(r, g.kmodes[j].div);
      const uint32_t d = r - q * g.kmodes[j].div.d;
      xa += (int64_t)d * g.kmodes[j].sa;
      xb += (int64_t)d * g.kmodes[j].sb;
      r = q;
    }
    ta[k] = xa;
    tb[k] = xb;
  }
  __syncthreads();
  const T* __restrict__ A = (const T*)g.A;
  const T* __restrict__ B = (const T*)g.B;
  const int64_t khi_n = g.K / klo;
  auto prod_at = [&](int64_t oa, int64_t ob, int64_t k) {
    uint32_t r = (uint32_t)k;
    int64_t xa = oa, xb = ob;
    for (int j = 0; j < g.nk; ++j) {
      const uint32_t q = fast_div(r, g.kmodes[j].div);
      const uint32_t d = r - q * g.kmodes[j].div.d;
      xa += (int64_t)d * g.kmodes[j].sa;
      xb += (int64_t)d * g.kmodes[j].sb;
      r = q;
    }
    return ALG == OM_STANDARD ? A[xa] * B[xb] : S::mul(A[xa], B[xb]);
  };
  for (int64_t o = blockIdx.x; o < g.total; o += gridDim.x) {
    int64_t oa = 0, ob = 0;
    {
      uint32_t r = (uint32_t)o;
      for (int j = 0; j < g.nout; ++j) {
        const uint32_t q = fast_div(r, g.out[j].div);
        const uint32_t d = r - q * g.out[j].div.d;
        oa += (int64_t)d * g.out[j].sa;
        ob += (int64_t)d * g.out[j].sb;
        r = q;
      }
    }
    T acc = ALG == OM_STANDARD ? T(0) : S::zero();
    int64_t bk = INT64_MAX;
    bool nan = false;
    for (int64_t h = 0; h < khi_n; ++h) {
      uint32_t r = (uint32_t)h;
      int64_t ha = oa, hb = ob;
      for (int j = nklo; j < g.nk; ++j) {
        const uint32_t q = fast_div(r, g.kmodes[j].div);
        const uint32_t d = r - q * g.kmodes[j].div.d;
        ha += (int64_t)d * g.kmodes[j].sa;
        hb += (int64_t)d * g.kmodes[j].sb;
        r = q;
      }
      for (int k = tid; k < (int)klo; k += kSplitThreads) {
        const T av = A[ha + ta[k]], bv = B[hb + tb[k]];
        if (ALG == OM_STANDARD) {
          acc = fma(av, bv, acc);
        } else {
          const T p = S::mul(av, bv);
          nan |= p != p;
          if (S::better(p, acc)) {  // visited in increasing k: the first best stays
            acc = p;
            bk = h * klo + k;
          }
        }
      }
    }
    // merge: warps, then the block
    for (int sh = 16; sh; sh >>= 1) {
      const T ov = __shfl_xor_sync(0xffffffffu, acc, sh);
      if (ALG == OM_STANDARD) {
        acc += ov;
      } else {
        const int64_t okk = __shfl_xor_sync(0xffffffffu, bk, sh);
        if (S::better(ov, acc) || (ov == acc && okk < bk)) {
          acc = ov;
          bk = okk;
        }
      }
    }
    if (tid == 0) snan = 0;
    __syncthreads();
    if (nan) snan = 1;
    if (lane == 0) {
      sv[warp] = acc;
      sk[warp] = bk;
    }
    __syncthreads();
    if (tid == 0) {
      T v = sv[0];
      int64_t w = sk[0];
      for (int q = 1; q < kSplitThreads / 32; ++q) {
        if (ALG == OM_STANDARD) {
          v += sv[q];
        } else if (S::better(sv[q], v) || (sv[q] == v && sk[q] < w)) {
          v = sv[q];
          w = sk[q];
        }
      }
      if (ALG != OM_STANDARD && snan) {  // the sequential rule, as in the forward
        v = S::zero();
        w = 0;
        for (int64_t k = 0; k < g.K; ++k) {
          const T p = prod_at(oa, ob, k);
          if (!S::keep(v, p)) {
            v = p;
            w = k;
          }
        }
      }
      if (ALG != OM_STANDARD && w == INT64_MAX) w = 0;  // nothing beat zero()
      ((T*)g.C)[o] = v;
      if (ARGMAX) g.argmax[o] = ALG == OM_STANDARD ? 0u : (uint32_t)w;
    }
    __syncthreads();
  }
}

int launch_gemm_node(om_backend* be, const NodeArgs& g0) {
  if (g0.total <= 0) return OM_OK;
  if (g0.K >= (int64_t(1) << 32) || g0.nout > kMaxNodeModes || g0.nk > kMaxNodeModes)
    return set_error(OM_ERR_INVALID, "gemm_node: plan out of range");
  if (g0.K >= 2048 && g0.total <= 64 * (int64_t)be->num_sms) {
    // few outputs, long k: the k range of each output over a CTA; the low
    // contracted modes whose extents multiply to at most kSplitTable are
    // tabulated
    int nklo = 0;
    int64_t klo = 1;
    while (nklo < g0.nk && klo * g0.kmodes[nklo].div.d <= kSplitTable) klo *= g0.kmodes[nklo++].div.d;
    const int grid = (int)std::min<int64_t>(g0.total, (int64_t)be->num_sms * 64);
    ProfScope prof(be, "gemm_node_splitk");
    if (g0.dtype == OM_F32) {
      OM_DISPATCH_ALG(g0.alg, ALG, {
        if (g0.argmax) gemm_node_splitk<float, ALG, true><<<grid, kSplitThreads, 0, be->stream>>>(g0, nklo, klo);
        else gemm_node_splitk<float, ALG, false><<<grid, kSplitThreads, 0, be->stream>>>(g0, nklo, klo);
      });
    } else {
      OM_DISPATCH_ALG(g0.alg, ALG, {
        if (g0.argmax) gemm_node_splitk<double, ALG, true><<<grid, kSplitThreads, 0, be->stream>>>(g0, nklo, klo);
        else gemm_node_splitk<double, ALG, false><<<grid, kSplitThreads, 0, be->stream>>>(g0, nklo, klo);
      });
    }
    note_launch();
    return check_cuda(cudaGetLastError(), "gemm_node_splitk launch");
  }
  // V = 4 outputs per thread when the first output mode splits into groups
  // of four and the outputs take 16-byte stores; the tile row then spans up
  // to 4 * kNodeQuads outputs
  NodeArgs g = g0;
  const size_t es = dtype_size(g.dtype);
  // the larger operand goes first (A): its values are the ones a thread
  // keeps across the other operand's own modes.  Every algebra's product
  // is commutative, and k's order is the contracted modes' order, which the
  // swap keeps.
  {
    auto footprint = [&](bool is_a) {
      int64_t n = 1;
      for (int j = 0; j < g.nout; ++j)
        if ((is_a ? g.out[j].sa : g.out[j].sb) != 0) n *= g.out[j].div.d;
      for (int j = 0; j < g.nk; ++j)
        if ((is_a ? g.kmodes[j].sa : g.kmodes[j].sb) != 0) n *= g.kmodes[j].div.d;
      return n;
    };
    if (footprint(false) > footprint(true)) {
      std::swap(g.A, g.B);
      for (int j = 0; j < g.nout; ++j) std::swap(g.out[j].sa, g.out[j].sb);
      for (int j = 0; j < g.nk; ++j) std::swap(g.kmodes[j].sa, g.kmodes[j].sb);
    }
  }
  // A tile row spans the leading output modes while their product stays
  // within kNodeQuads * 4; a large mode that would end the row early (a
  // leading 2 x 2 and then an extent of 2^21 leaves rows of four outputs,
  // each decoding every high mode) is split into two modes, f x e / f, with
  // f the largest divisor of its extent that fills the row.  Linear output
  // order is unchanged (the first factor runs fastest).
  {
    int64_t P = 1;
    const int64_t L = (int64_t)kNodeQuads * 4;
    for (int j = 0; j < g.nout; ++j) {
      const int64_t e = g.out[j].div.d;
      if (P * e <= L) {
        P *= e;
        continue;
      }
      if (P * 64 > L || g.nout >= kMaxNodeModes) break;  // the row is long enough
      int64_t f = L / P;
      while (f > 1 && e % f) --f;
      if (f > 1) {
        for (int q = g.nout; q > j + 1; --q) g.out[q] = g.out[q - 1];
        const NodeMode m = g.out[j];
        g.out[j] = NodeMode{make_fastdiv((uint32_t)f), m.sa, m.sb};
        g.out[j + 1] = NodeMode{make_fastdiv((uint32_t)(e / f)), m.sa * f, m.sb * f};
        ++g.nout;
      }
      break;
    }
  }
  // a group of 4 consecutive outputs must decode separably: 4 = (product of
  // the leading modes) x (a divisor of the next mode's extent)
  bool sep = false;
  {
    int64_t pre = 1;
    for (int j = 0; j < g.nout && !sep; ++j) {
      const int64_t e = g.out[j].div.d;
      if (4 % pre == 0 && e % (4 / pre) == 0) sep = true;
      pre *= e;
      if (pre > 4) break;
    }
  }
  // groups of four use 32-bit offsets: every offset of A and B must fit
  auto span_fits = [&](bool is_a) {
    int64_t span = 0;
    for (int j = 0; j < g.nout; ++j) {
      const int64_t st = is_a ? g.out[j].sa : g.out[j].sb;
      if (st < 0) return false;
      span += (int64_t)(g.out[j].div.d - 1) * st;
    }
    for (int j = 0; j < g.nk; ++j) {
      const int64_t st = is_a ? g.kmodes[j].sa : g.kmodes[j].sb;
      if (st < 0) return false;
      span += (int64_t)(g.kmodes[j].div.d - 1) * st;
    }
    return span < (int64_t(1) << 31);
  };
  const bool v4 = sep && g.total % 4 == 0 && ((uintptr_t)g.C % (4 * es)) == 0 &&
                  (!g.argmax || ((uintptr_t)g.argmax % 16) == 0) && span_fits(true) &&
                  span_fits(false);
  int vec = v4 ? 4 : 1;
  auto tile = [&](int v) {
    g.nlow = 0;
    int64_t P = 1;
    while (g.nlow < g.nout && P * g.out[g.nlow].div.d <= (int64_t)kNodeQuads * v)
      P *= g.out[g.nlow++].div.d;
    return P;
  };
  int64_t P = tile(vec);
  if (P % vec) P = tile(vec = 1);
  auto width = [&](const int64_t* o) {
    if (vec != 4) return 1;
    if (o[1] == 0 && o[2] == 0 && o[3] == 0) return 0;
    if (o[1] == 1 && o[2] == 2 && o[3] == 3) return 4;
    if (o[1] == 1 && o[3] == o[2] + 1) return 2;
    if (o[1] == 0 && o[3] == o[2]) return 3;
    if (o[2] == 0 && o[3] == o[1]) return 5;
    return 1;
  };
  for (int i = 0; i < 4; ++i) {
    g.ia[i] = g.ib[i] = 0;
    if (i >= vec) continue;
    int64_t r = i;
    for (int j = 0; j < g.nout && r; ++j) {
      const int64_t e = g.out[j].div.d;
      g.ia[i] += (r % e) * g.out[j].sa;
      g.ib[i] += (r % e) * g.out[j].sb;
      r /= e;
    }
  }
  // a vector width holds only if every group start is aligned to it: the
  // base, the contracted strides and the stride steps between group starts
  auto aligned_to = [&](int w, bool is_a) {
    if (w != 2 && w != 4) return true;
    const uintptr_t base = (uintptr_t)(is_a ? g.A : g.B);
    if (base % (w * es)) return false;
    const int64_t* io = is_a ? g.ia : g.ib;
    if (w == 2 && io[2] % 2) return false;
    int64_t pre = 1;
    for (int j = 0; j < g.nout; ++j) {
      const int64_t st = is_a ? g.out[j].sa : g.out[j].sb;
      const int64_t step = pre >= vec ? 1 : vec / pre;  // digit step between group starts
      if ((st * step) % w) return false;
      pre *= g.out[j].div.d;
    }
    for (int j = 0; j < g.nk; ++j)
      if ((is_a ? g.kmodes[j].sa : g.kmodes[j].sb) % w) return false;
    return true;
  };
  g.wa = width(g.ia);
  g.wb = width(g.ib);
  if (!aligned_to(g.wa, true)) g.wa = 1;
  if (!aligned_to(g.wb, false)) g.wb = 1;
  g.P = (int32_t)P;
  g.rows = g.total / P;
  if (g.rows >= (int64_t(1) << 32)) return set_error(OM_ERR_INVALID, "gemm_node: too many rows");
  // Row order.  C is contiguous in mode order, so each row mode's C stride
  // is the product of the extents below it.  The row modes that A (the
  // larger operand) does not carry are decoded first, so that the rows that
  // read the same part of A run back to back and A is read from DRAM about
  // once (in C's own order those rows can lie a whole tensor apart, and a
  // node of 2^28 outputs then read its 2^28-element operand 7 times over).
  // When k has a compiled length, the leading such modes (up to kNodeRep
  // combinations) run inside each thread on A values held in registers.
  g.nrep = 0;
  g.R = 1;
  {
    int64_t sc = 1;
    for (int j = 0; j < g.nout; ++j) {
      g.out[j].sc = sc;
      sc *= g.out[j].div.d;
    }
    NodeMode first[kMaxNodeModes], rest[kMaxNodeModes];
    int nf = 0, nr = 0;
    for (int j = g.nlow; j < g.nout; ++j) {
      if (g.out[j].sa == 0) first[nf++] = g.out[j];
      else rest[nr++] = g.out[j];
    }
    for (int j = 0; j < nf; ++j) g.out[g.nlow + j] = first[j];
    for (int j = 0; j < nr; ++j) g.out[g.nlow + nf + j] = rest[j];
    const bool kt = g.K == 1 || g.K == 2 || g.K == 4 || (g.K == 8 && g.dtype == OM_F32);
    if (kt)
      while (g.nrep < nf && (int64_t)g.R * g.out[g.nlow + g.nrep].div.d <= kNodeRep)
        g.R *= (int32_t)g.out[g.nlow + g.nrep++].div.d;
    g.rows /= g.R;
  }
  if (g.dtype == OM_F32) {
    OM_DISPATCH_ALG(g.alg, ALG, return launch_node_typed<float, ALG>(be, g, vec));
  } else if (g.dtype == OM_F64) {
    OM_DISPATCH_ALG(g.alg, ALG, return launch_node_typed<double, ALG>(be, g, vec));
  }
  return set_error(OM_ERR_UNSUPPORTED, "gemm: dtype must be f32 or f64");
}

int launch_gemm(om_backend* be, const GemmArgs& g) {
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return OM_OK;
  bool handled = false;
  OM_TRY(launch_gemm_tf32(be, g, &handled));
  if (handled) return OM_OK;
  OM_TRY(launch_gemm_tropical_fast(be, g, &handled));
  if (handled) return OM_OK;
  OM_TRY(launch_gemm_f64(be, g, &handled));
  if (handled) return OM_OK;
  return launch_gemm_exact(be, g);
}

}  // namespace om
