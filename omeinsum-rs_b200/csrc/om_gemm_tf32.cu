// K3: Standard f32 GEMM on the 5th-generation tensor cores (tcgen05, TMEM,
// TMA) in a 3xTF32 split, for the reference's Standard<f32> contraction
// (faer GEMM in src/backend/cpu/mod.rs:176-287,621-859).
//
// Every f32 operand x is split into hi = tf32(x) (round to nearest) and
// lo = tf32(x - hi); the product is accumulated as
//     A_lo B_hi + A_hi B_lo + A_hi B_hi
// in f32, chunk by chunk in tensor memory and across chunks in registers
// (see CHUNK), which keeps the error near that of an f32 FMA loop.
//
// Two kernels:
//   split_tf32_kernel  one HBM pass: reads an operand through its strides
//                      (any layout, batched), writes hi and lo as K-major
//                      rows [batch][rows][Kp] (Kp = K rounded up to 32, zero
//                      padded).  This is also the operand gather (K1) fused
//                      with the split, staged through a 32 x 32 shared tile so
//                      reads and writes stay coalesced.
//   gemm_tf32x3_kernel persistent (one CTA per SM, tiles of 128 x 128 taken
//                      round robin), 320 threads: warp 0 issues TMA loads
//                      (cp.async.bulk.tensor, 128-byte swizzle, no multicast)
//                      of the four 128 x 32 slabs (A_hi, A_lo, B_hi, B_lo)
//                      into a 3-stage ring with full / empty mbarriers; warp 1
//                      allocates 2 x 128 TMEM columns and one thread issues 12
//                      tcgen05.mma kind::tf32 (M = N = 128, K = 8) per slab,
//                      committing each stage back to the producer; the k range
//                      of a tile is cut into chunks of CHUNK slabs, each
//                      accumulated from zero in one of the two TMEM
//                      accumulators (alternating), and warps 2..9 read every
//                      finished chunk with tcgen05.ld.32x32b (warp w reads TMEM
//                      lanes 32*(w%4).., columns 64*((w-2)/4)..) and add it
//                      into f32 registers while the MMAs of the next chunk fill
//                      the other accumulator; after the tile's last chunk they
//                      store C.
// Every mbarrier wait is bounded; on expiry the kernel records an error word
// that om_b200_sync reports, and every warp leaves after its own bounded
// waits so that TMEM is always freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "om_internal.h"

namespace om {
namespace {

constexpr int TM = 128, TN = 128, TK = 32, STAGES = 3, NTH = 320;
constexpr int EPI_WARPS = 8;  // warps 2..9: lane quadrant (warp % 4), column half (warp - 2) / 4
constexpr int SLAB_BYTES = TM * TK * 4;      // 16 KiB: 128 rows x 128 bytes
constexpr int STAGE_BYTES = 4 * SLAB_BYTES;  // A_hi, A_lo, B_hi, B_lo
constexpr uint32_t kWaitLimit = 1u << 24;    // polls of a try_wait before giving up
// Slabs per accumulation chunk.  The tensor core adds the products of each
// 8-deep MMA step into its f32 accumulator with its own (not round-to-nearest)
// alignment and rounding, an error of the order of one ulp of the running
// sum per step; over K = 1024 that bias reaches ~2^-16 of the partial sums.
// Each chunk of CHUNK * 32 k is therefore accumulated in TMEM from zero and
// added into f32 registers by the epilogue warps, which bounds the tensor
// core's share of the error by CHUNK * 4 steps of a chunk-sized sum.
constexpr int CHUNK = 4;

// ---------------------------------------------------------------------------
// split pre-pass
// ---------------------------------------------------------------------------
struct SplitArgs {
  const float* x;
  int64_t rows, K, Kp, batch;
  int64_t sr, sk, sb;  // element strides of (row, k, batch)
  int64_t k1, sk2;     // k = k1-index + k1 * k2-index, read at k1i * sk + k2i * sk2
  int64_t r1, sr2;     // rows likewise
  float* hi;
  float* lo;
};

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__global__ void split_tf32_kernel(SplitArgs a, int64_t tiles_k, int64_t tiles_r, int64_t total) {
  __shared__ float tile[32][33];
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  const bool k_fast = a.sk == 1;
  for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
    const int64_t tk = t % tiles_k, rest = t / tiles_k;
    const int64_t tr = rest % tiles_r, b = rest / tiles_r;
    const int64_t r0 = tr * 32, k0 = tk * 32;
    // a 32-wide tile never straddles an outer level (k1 % 32 == r1 % 32 == 0)
    const int64_t ok_ = k0 / a.k1, or_ = r0 / a.r1;
    const float* xb = a.x + (b * a.sb + ok_ * (a.sk2 - a.k1 * a.sk) + or_ * (a.sr2 - a.r1 * a.sr));
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + (k_fast ? i : tx), k = k0 + (k_fast ? tx : i);
      float v = 0.f;
      if (r < a.rows && k < a.K) v = xb[r * a.sr + k * a.sk];
      if (k_fast) tile[i][tx] = v;
      else tile[tx][i] = v;
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
      const int64_t r = r0 + i, k = k0 + tx;
      if (r < a.rows && k < a.Kp) {
        const float v = tile[i][tx];
        const float h = tf32_rna(v);
        const int64_t o = (b * a.rows + r) * a.Kp + k;
        a.hi[o] = h;
        a.lo[o] = tf32_rna(v - h);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// tcgen05 GEMM
// ---------------------------------------------------------------------------
struct Tf32Args {
  int M, N, T, batch;
  float* C;
  int64_t scm, scn, scb;
  uint32_t* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// K-major, 128-byte swizzle: 8-row groups 1024 B apart; k steps of 8 tf32
// advance the start address by 32 B inside the swizzle atom
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

// kind::tf32, D f32, A/B tf32 K-major, M = 128, N = 128
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(TN >> 3) << 17) |
                            ((uint32_t)(TM >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Persistent: CTA c takes tiles c, c + G, c + 2G, ...; all roles walk the same
// sequence.  Two 128-column TMEM accumulators alternate between tiles so the
// epilogue of tile i overlaps the MMAs of tile i + 1.
__global__ void __launch_bounds__(NTH, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap ahi, const __grid_constant__ CUtensorMap alo,
                       const __grid_constant__ CUtensorMap bhi, const __grid_constant__ CUtensorMap blo,
                       Tf32Args g) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2];
  __shared__ uint32_t tmem_base;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gx = (g.M + TM - 1) / TM, gy = (g.N + TN - 1) / TN;
  const int tiles = gx * gy * g.batch;
  const int G = gridDim.x;
  const int nch = (g.T + CHUNK - 1) / CHUNK;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_base)),
                 "r"(2 * TN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&empty[s])));
    }
    for (int b = 0; b < 2; ++b) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&tfull[b])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&tempty[b])),
                   "r"(EPI_WARPS));
    }
    asm volatile("fence.mbarrier_init.release.cluster;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = tmem_base;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      int q = 0;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += G) {
        const int bx = tile % gx, by = (tile / gx) % gy, bt = tile / (gx * gy);
        for (int t = 0; t < g.T && ok; ++t, ++q) {
          const int s = q % STAGES;
          if (q >= STAGES) ok = mbar_wait(smem_u32(&empty[s]), ((q / STAGES) - 1) & 1);
          if (!ok) break;
          const uint32_t bar = smem_u32(&full[s]);
          asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                       "r"(STAGE_BYTES)
                       : "memory");
          const uint32_t dst = smem_u32(smem + s * STAGE_BYTES);
          tma_load_3d(dst, &ahi, t * TK, bx * TM, bt, bar);
          tma_load_3d(dst + SLAB_BYTES, &alo, t * TK, bx * TM, bt, bar);
          tma_load_3d(dst + 2 * SLAB_BYTES, &bhi, t * TK, by * TN, bt, bar);
          tma_load_3d(dst + 3 * SLAB_BYTES, &blo, t * TK, by * TN, bt, bar);
        }
      }
      if (!ok) atomicOr(g.err, 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer: one TMEM accumulator per k-chunk, alternating
      int q = 0, i = 0;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += G) {
        for (int c = 0; c < nch && ok; ++c, ++i) {
          const int ab = i & 1;
          if (i >= 2) ok = mbar_wait(smem_u32(&tempty[ab]), ((i >> 1) - 1) & 1);
          if (!ok) break;
          asm volatile("tcgen05.fence::after_thread_sync;");
          const uint32_t d = tmem + (uint32_t)(ab * TN);
          const int t0 = c * CHUNK, t1 = min(g.T, t0 + CHUNK);
          for (int t = t0; t < t1 && ok; ++t, ++q) {
            const int s = q % STAGES;
            ok = mbar_wait(smem_u32(&full[s]), (q / STAGES) & 1);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
#pragma unroll
            for (int j = 0; j < TK / 8; ++j) {
              const uint64_t a_h = sw128_desc(base + j * 32);
              const uint64_t a_l = sw128_desc(base + SLAB_BYTES + j * 32);
              const uint64_t b_h = sw128_desc(base + 2 * SLAB_BYTES + j * 32);
              const uint64_t b_l = sw128_desc(base + 3 * SLAB_BYTES + j * 32);
              mma_tf32(d, a_l, b_h, (t > t0 || j > 0) ? 1u : 0u);
              mma_tf32(d, a_h, b_l, 1u);
              mma_tf32(d, a_h, b_h, 1u);
            }
            mma_commit(smem_u32(&empty[s]));
          }
          mma_commit(smem_u32(&tfull[ab]));  // fires when this chunk's MMAs are done
        }
      }
      if (!ok) atomicOr(g.err, 1u);
    }
  } else {  // epilogue warps 2..9: TMEM lanes 32*(warp % 4), columns 64*half..
    const int quad = warp & 3, half = (warp - 2) >> 2;
    constexpr int HN = TN / 2;
    int i = 0;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += G) {
      const int bx = tile % gx, by = (tile / gx) % gy, bt = tile / (gx * gy);
      const int m = bx * TM + 32 * quad + lane;
      // the tile's row m (this warp's half of it), summed chunk by chunk in
      // f32 registers (round to nearest): the tensor core's own accumulation
      // is only trusted over CHUNK slabs
      float acc[HN];
#pragma unroll
      for (int n = 0; n < HN; ++n) acc[n] = 0.f;
      for (int c = 0; c < nch && ok; ++c, ++i) {
        const int ab = i & 1;
        ok = mbar_wait(smem_u32(&tfull[ab]), (i >> 1) & 1);
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;");
        uint32_t r[HN];
#pragma unroll
        for (int c0 = 0; c0 < HN; c0 += 32) {
          const uint32_t taddr =
              tmem + ((uint32_t)(32 * quad) << 16) + (uint32_t)(ab * TN + half * HN + c0);
          uint32_t* x = r + c0;
          asm volatile(
              "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
              "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
              : "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]),
                "=r"(x[6]), "=r"(x[7]), "=r"(x[8]), "=r"(x[9]), "=r"(x[10]), "=r"(x[11]),
                "=r"(x[12]), "=r"(x[13]), "=r"(x[14]), "=r"(x[15]), "=r"(x[16]), "=r"(x[17]),
                "=r"(x[18]), "=r"(x[19]), "=r"(x[20]), "=r"(x[21]), "=r"(x[22]), "=r"(x[23]),
                "=r"(x[24]), "=r"(x[25]), "=r"(x[26]), "=r"(x[27]), "=r"(x[28]), "=r"(x[29]),
                "=r"(x[30]), "=r"(x[31])
              : "r"(taddr));
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        // the accumulator is free as soon as it is in registers
        asm volatile("tcgen05.fence::before_thread_sync;");
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&tempty[ab]));
#pragma unroll
        for (int qq = 0; qq < HN; ++qq) acc[qq] += __uint_as_float(r[qq]);
      }
      if (!ok) break;
      float* Cb = g.C + (int64_t)bt * g.scb;
      if (m < g.M) {
#pragma unroll
        for (int n0 = 0; n0 < HN; ++n0) {
          const int n = by * TN + half * HN + n0;
          if (n < g.N) Cb[(int64_t)m * g.scm + (int64_t)n * g.scn] = acc[n0];
        }
      }
    }
    if (!ok && lane == 0) atomicOr(g.err, 1u);
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(2 * TN));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  return fn;
}

// 3-D map over a split operand [batch][rows][Kp] f32, box 32 (k) x 128 rows
int make_map(CUtensorMap* map, float* base, int64_t rows, int64_t Kp, int64_t batch) {
  auto fn = encode_fn();
  if (!fn) return set_error(OM_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");
  cuuint64_t dims[3] = {(cuuint64_t)Kp, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(Kp * 4), (cuuint64_t)(rows * Kp * 4)};
  cuuint32_t box[3] = {(cuuint32_t)TK, (cuuint32_t)TM, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(OM_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return OM_OK;
}

int launch_split(om_backend* be, const float* x, int64_t rows, int64_t K, int64_t Kp,
                 int64_t batch, int64_t sr, int64_t sk, int64_t sb, int64_t k1, int64_t sk2,
                 int64_t r1, int64_t sr2, float* hi, float* lo) {
  if (k1 <= 0) {  // flat: one level covering every k (and the padding)
    k1 = Kp;
    sk2 = 0;
  }
  if (r1 <= 0) {
    r1 = (rows + 31) / 32 * 32;
    sr2 = 0;
  }
  SplitArgs a{x, rows, K, Kp, batch, sr, sk, sb, k1, sk2, r1, sr2, hi, lo};
  const int64_t tk = Kp / 32, tr = (rows + 31) / 32, total = tk * tr * batch;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(total, (int64_t)be->num_sms * 16));
  ProfScope prof(be, "split_tf32");
  split_tf32_kernel<<<blocks, dim3(32, 8), 0, be->stream>>>(a, tk, tr, total);
  note_launch();
  return check_cuda(cudaGetLastError(), "split_tf32 launch");
}

}  // namespace

bool tf32_takes(const om_backend* be, om_algebra alg, om_dtype dt, bool argmax, int64_t M,
                int64_t N, int64_t K, int64_t batch) {
  if (dt != OM_F32 || alg != OM_STANDARD || argmax || be->f32_exact) return false;
  if (M < 64 || N < 64 || K < 16 || batch > 65535) return false;
  if (M > (1 << 30) || N > (1 << 30) || K > (1 << 30)) return false;
  const int64_t tiles = ((M + TM - 1) / TM) * ((N + TN - 1) / TN) * batch;
  return tiles <= (1ll << 31) - 1;
}

// Takes a Standard f32 GEMM when the tensor-core path applies.
int launch_gemm_tf32(om_backend* be, const GemmArgs& g, bool* handled) {
  *handled = false;
  if (!tf32_takes(be, g.alg, g.dtype, g.argmax != nullptr, g.M, g.N, g.K, g.batch)) {
    // two-level rows / columns exist only for this path; two-level k is
    // also read by the fast tropical, f64 and exact kernels
    if (g.ma1 > 0 || g.nb1 > 0)
      return set_error(OM_ERR_INVALID, "gemm: two-level rows or columns off the tensor-core path");
    return OM_OK;
  }
  const int64_t Kp = (g.K + TK - 1) / TK * TK;
  const size_t na = (size_t)(g.batch * g.M * Kp), nb = (size_t)(g.batch * g.N * Kp);
  Scratch ws;
  OM_TRY(ws.alloc(be, 4 * (2 * na + 2 * nb)));
  float* a_hi = (float*)ws.ptr;
  float* a_lo = a_hi + na;
  float* b_hi = a_lo + na;
  float* b_lo = b_hi + nb;
  OM_TRY(launch_split(be, (const float*)g.A, g.M, g.K, Kp, g.batch, g.sam, g.sak, g.sab, g.ka1,
                      g.sak2, g.ma1, g.sam2, a_hi, a_lo));
  OM_TRY(launch_split(be, (const float*)g.B, g.N, g.K, Kp, g.batch, g.sbn, g.sbk, g.sbb, g.kb1,
                      g.sbk2, g.nb1, g.sbn2, b_hi, b_lo));
  CUtensorMap m_ahi, m_alo, m_bhi, m_blo;
  OM_TRY(make_map(&m_ahi, a_hi, g.M, Kp, g.batch));
  OM_TRY(make_map(&m_alo, a_lo, g.M, Kp, g.batch));
  OM_TRY(make_map(&m_bhi, b_hi, g.N, Kp, g.batch));
  OM_TRY(make_map(&m_blo, b_lo, g.N, Kp, g.batch));
  Tf32Args a;
  a.M = (int)g.M;
  a.N = (int)g.N;
  a.T = (int)(Kp / TK);
  a.C = (float*)g.C;
  a.scm = g.scm;
  a.scn = g.scn;
  a.scb = g.scb;
  a.err = be->d_flags + 1;
  const size_t smem = (size_t)STAGES * STAGE_BYTES + 1024;
  OM_CUDA(cudaFuncSetAttribute(gemm_tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem),
          "cudaFuncSetAttribute(tf32)");
  a.batch = (int)g.batch;
  const int64_t tiles = (int64_t)((a.M + TM - 1) / TM) * ((a.N + TN - 1) / TN) * g.batch;
  const unsigned grid = (unsigned)std::min<int64_t>(tiles, be->num_sms);
  {
    ProfScope prof(be, "gemm_tf32x3_tcgen05");
    gemm_tf32x3_kernel<<<grid, NTH, smem, be->stream>>>(m_ahi, m_alo, m_bhi, m_blo, a);
    note_launch();
    OM_CUDA(cudaGetLastError(), "gemm_tf32x3 launch");
  }
  *handled = true;
  return OM_OK;
}

}  // namespace om
