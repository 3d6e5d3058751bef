// K1: strided gather / permute into a contiguous column-major buffer.
//
// Device replacement of the reference's odometer loops
// materialize_with_permutation_into (tensor4all/omeinsum-rs
// src/backend/cpu/contract.rs:709-748) and Cpu::copy_strided
// (src/backend/cpu/mod.rs:584-619).  HBM-bound: every path reads and writes
// each element once; the tiled path keeps both sides coalesced by staging a
// 32x32 tile in shared memory when the source's unit-stride axis is not the
// destination's first axis.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <type_traits>
#include <vector>

#include "om_internal.h"

namespace om {
namespace {

struct GatherDesc {
  int nd;
  int64_t shape[OM_MAX_DIMS];
  int64_t sstride[OM_MAX_DIMS];
};

constexpr int kTile = 32;

// one thread per destination element; source offset by mixed-radix decode
template <typename T>
__global__ void gather_generic(const T* __restrict__ src, T* __restrict__ dst, GatherDesc d,
                               int64_t n) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = e, off = 0;
#pragma unroll 1
    for (int k = 0; k < d.nd; ++k) {
      int64_t c = rem % d.shape[k];
      rem /= d.shape[k];
      off += c * d.sstride[k];
    }
    dst[e] = src[off];
  }
}

// destination axis 0 is unit stride in the source too: copy rows of length
// shape[0]; the remaining axes index the row.
template <typename T>
__global__ void gather_rows(const T* __restrict__ src, T* __restrict__ dst, GatherDesc d,
                            int64_t rows) {
  const int64_t len = d.shape[0];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    int64_t rem = r, off = 0;
#pragma unroll 1
    for (int k = 1; k < d.nd; ++k) {
      int64_t c = rem % d.shape[k];
      rem /= d.shape[k];
      off += c * d.sstride[k];
    }
    const T* s = src + off;
    T* o = dst + r * len;
    for (int64_t i = threadIdx.x; i < len; i += blockDim.x) o[i] = s[i];
  }
}

// destination axis 0 (stride 1 in dst) vs. destination axis p (stride 1 in
// src): 32x32 tile transposed through shared memory.
template <typename T>
__global__ void gather_transpose(const T* __restrict__ src, T* __restrict__ dst, GatherDesc d,
                                 int p, int64_t dstride_p, int64_t tiles0, int64_t tilesp,
                                 int64_t total_tiles) {
  __shared__ T tile[kTile][kTile + 1];
  const int64_t s0 = d.shape[0], sp = d.shape[p];
  const int64_t st0 = d.sstride[0];
  for (int64_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
    int64_t t0 = t % tiles0;
    int64_t rest = t / tiles0;
    int64_t tp = rest % tilesp;
    int64_t outer = rest / tilesp;
    // decode the outer index over axes other than 0 and p
    int64_t soff = 0, doff = 0, dstr = d.shape[0];
    int64_t rem = outer;
    for (int k = 1; k < d.nd; ++k) {
      if (k == p) {
        dstr *= d.shape[k];
        continue;
      }
      int64_t c = rem % d.shape[k];
      rem /= d.shape[k];
      soff += c * d.sstride[k];
      doff += c * dstr;
      dstr *= d.shape[k];
    }
    // dst strides of axis k are products of earlier shapes; recompute for k<p
    // (already folded above, dstr runs in order of axes)
    const int64_t i0 = t0 * kTile, j0 = tp * kTile;
    __syncthreads();
    // read: consecutive threads walk axis p (unit stride in src)
    for (int r = threadIdx.y; r < kTile; r += blockDim.y) {
      int64_t i = i0 + r, j = j0 + threadIdx.x;
      if (i < s0 && j < sp) tile[r][threadIdx.x] = src[soff + i * st0 + j];
    }
    __syncthreads();
    // write: consecutive threads walk axis 0 (unit stride in dst)
    for (int r = threadIdx.y; r < kTile; r += blockDim.y) {
      int64_t j = j0 + r, i = i0 + threadIdx.x;
      if (i < s0 && j < sp) dst[doff + i + j * dstride_p] = tile[threadIdx.x][r];
    }
  }
}

// Batched 32 x 32 transpose with 16-byte accesses on both sides: destination
// axis 0 (unit stride in dst) against axis p (unit stride in src), both
// multiples of 32, every other axis indexing tiles.  Each thread moves one
// 16-byte vector per tile in and out of a padded shared tile (conflict-free
// in both phases); a CTA takes kTv tiles per round so that several loads are
// in flight per thread.
constexpr int kTv = 2;

template <typename T>
__global__ void __launch_bounds__(256) gather_transpose_vec(const T* __restrict__ src,
                                                            T* __restrict__ dst, GatherDesc d,
                                                            int p, int64_t dstride_p,
                                                            int64_t tiles0, int64_t tilesp,
                                                            int64_t total_tiles) {
  constexpr int V = 16 / sizeof(T);      // elements per vector
  constexpr int VR = kTile / V;          // vectors per 32-element row
  constexpr int UPT = kTile * VR / 256;  // vectors per thread per tile (1 or 2)
  using Vec = typename std::conditional<sizeof(T) == 4, uint4, ulonglong2>::type;
  __shared__ T tile[kTv][kTile][kTile + 1];
  const int tid = threadIdx.x;
  for (int64_t t0 = (int64_t)blockIdx.x * kTv; t0 < total_tiles; t0 += (int64_t)gridDim.x * kTv) {
    int64_t soff[kTv], doff[kTv];
    Vec v[kTv][UPT];
#pragma unroll
    for (int q = 0; q < kTv; ++q) {
      const int64_t t = t0 + q;
      soff[q] = doff[q] = -1;
      if (t >= total_tiles) continue;
      const int64_t ti = t % tiles0, rest = t / tiles0;
      const int64_t tp = rest % tilesp;
      int64_t rem = rest / tilesp, so = 0, dof = 0, dstr = d.shape[0];
      for (int k = 1; k < d.nd; ++k) {
        if (k == p) {
          dstr *= d.shape[k];
          continue;
        }
        const int64_t c = rem % d.shape[k];
        rem /= d.shape[k];
        so += c * d.sstride[k];
        dof += c * dstr;
        dstr *= d.shape[k];
      }
      soff[q] = so + ti * kTile * d.sstride[0] + tp * kTile;
      doff[q] = dof + ti * kTile + tp * kTile * dstride_p;
#pragma unroll
      for (int u = 0; u < UPT; ++u) {
        const int w = tid + 256 * u, i = w / VR, jv = w % VR;
        v[q][u] = *(const Vec*)(src + soff[q] + i * d.sstride[0] + jv * V);
      }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kTv; ++q) {
      if (soff[q] < 0) continue;
#pragma unroll
      for (int u = 0; u < UPT; ++u) {
        const int w = tid + 256 * u, i = w / VR, jv = w % VR;
        const T* e = (const T*)&v[q][u];
#pragma unroll
        for (int c = 0; c < V; ++c) tile[q][i][jv * V + c] = e[c];
      }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < kTv; ++q) {
      if (doff[q] < 0) continue;
#pragma unroll
      for (int u = 0; u < UPT; ++u) {
        const int w = tid + 256 * u, j = w / VR, iv = w % VR;
        Vec o;
        T* e = (T*)&o;
#pragma unroll
        for (int c = 0; c < V; ++c) e[c] = tile[q][iv * V + c][j];
        *(Vec*)(dst + doff[q] + iv * V + j * dstride_p) = o;
      }
    }
  }
}

// Permutation of a dense source (its axes, sorted by stride, form a
// column-major layout) where no single axis is long enough for the row or
// 32x32-transpose paths -- e.g. a network intermediate of many extent-2
// modes.  A tile is the product of a set U of axes holding at least 32
// elements contiguous in the source and at least 32 contiguous in the
// destination; the remaining axes R index tiles.  Three per-CTA tables
// (built once) give the source offset of each tile element in source order,
// its slot in the tile (destination order) and its destination offset, so
// both global sides move in runs of >= 32 elements and the per-element index
// work is two shared-memory reads.  Each CTA walks a contiguous range of
// tiles with an odometer over R, so tile bases cost O(1) per tile.
constexpr int kPermMaxTile = 2048;

struct PermDesc {
  int nu, nr;
  int32_t t;                        // tile size = prod of U extents
  int32_t u_shape[OM_MAX_DIMS];     // U in destination order
  int32_t u_sstr[OM_MAX_DIMS];      // source stride of each U axis
  int32_t u_dstr[OM_MAX_DIMS];      // destination stride of each U axis
  int32_t u_tpos[OM_MAX_DIMS];      // stride of each U axis inside the tile
  int32_t us_order[OM_MAX_DIMS];    // U indices sorted by source stride
  int64_t r_shape[OM_MAX_DIMS];     // R in destination order
  int64_t r_sstr[OM_MAX_DIMS];
  int64_t r_dstr[OM_MAX_DIMS];
  int64_t ntiles;
};

__device__ __forceinline__ int perm_pad(int j) { return j + (j >> 5); }

template <typename T>
__global__ void __launch_bounds__(256) gather_perm_tiled(const T* __restrict__ src,
                                                         T* __restrict__ dst, PermDesc p) {
  extern __shared__ __align__(16) unsigned char perm_smem[];
  int32_t* s_src = reinterpret_cast<int32_t*>(perm_smem);  // by source order
  int32_t* s_slot = s_src + p.t;                             // by source order
  int32_t* s_dst = s_slot + p.t;                             // by tile slot
  int64_t* s_base = reinterpret_cast<int64_t*>(s_dst + p.t + (p.t & 1));  // [2][2]
  int64_t* s_coord = s_base + 4;                                           // [nr]
  T* tile = reinterpret_cast<T*>(s_coord + OM_MAX_DIMS);
  const int tid = threadIdx.x, nth = blockDim.x;

  for (int j = tid; j < p.t; j += nth) {
    int rem = j, doff = 0;
    for (int u = 0; u < p.nu; ++u) {
      int c = rem % p.u_shape[u];
      rem /= p.u_shape[u];
      doff += c * p.u_dstr[u];
    }
    s_dst[j] = doff;
    // j read as an index in source order
    rem = j;
    int soff = 0, slot = 0;
    for (int q = 0; q < p.nu; ++q) {
      int u = p.us_order[q];
      int c = rem % p.u_shape[u];
      rem /= p.u_shape[u];
      soff += c * p.u_sstr[u];
      slot += c * p.u_tpos[u];
    }
    s_src[j] = soff;
    s_slot[j] = slot;
  }
  const int64_t per = (p.ntiles + gridDim.x - 1) / gridDim.x;
  const int64_t o0 = blockIdx.x * per;
  const int64_t o1 = o0 + per < p.ntiles ? o0 + per : p.ntiles;
  if (tid == 0) {
    int64_t rem = o0, sb = 0, db = 0;
    for (int r = 0; r < p.nr; ++r) {
      int64_t c = rem % p.r_shape[r];
      rem /= p.r_shape[r];
      s_coord[r] = c;
      sb += c * p.r_sstr[r];
      db += c * p.r_dstr[r];
    }
    s_base[0] = sb;
    s_base[1] = db;
  }
  __syncthreads();
  int cur = 0;
  for (int64_t o = o0; o < o1; ++o) {
    const int64_t sb = s_base[2 * cur], db = s_base[2 * cur + 1];
#pragma unroll 4
    for (int i = tid; i < p.t; i += nth) tile[perm_pad(s_slot[i])] = src[sb + s_src[i]];
    __syncthreads();
    if (tid == 0) {  // odometer step to tile o + 1
      int64_t nsb = sb, ndb = db;
      for (int r = 0; r < p.nr; ++r) {
        int64_t c = s_coord[r] + 1;
        if (c < p.r_shape[r]) {
          s_coord[r] = c;
          nsb += p.r_sstr[r];
          ndb += p.r_dstr[r];
          break;
        }
        s_coord[r] = 0;
        nsb -= (p.r_shape[r] - 1) * p.r_sstr[r];
        ndb -= (p.r_shape[r] - 1) * p.r_dstr[r];
      }
      s_base[2 * (cur ^ 1)] = nsb;
      s_base[2 * (cur ^ 1) + 1] = ndb;
    }
#pragma unroll 4
    for (int j = tid; j < p.t; j += nth) dst[db + s_dst[j]] = tile[perm_pad(j)];
    __syncthreads();
    cur ^= 1;
  }
}

// Plans the tiled permutation; false when the source is not a dense
// permutation or no tile of at most kPermMaxTile elements has 32-element
// runs on both sides.
bool plan_perm(const GatherDesc& d0, const int64_t* dstr0, int64_t n, PermDesc& p) {
  if (d0.nd < 2 || n >= (int64_t(1) << 31)) return false;
  // Split each long axis into (piece, rest) so that a tile can take a
  // 32-element piece of it: a transpose of an extent-2 axis against a long
  // contiguous one then still gets 128-byte runs on both sides.
  GatherDesc d;
  int64_t dstr[OM_MAX_DIMS];
  d.nd = 0;
  for (int k = 0; k < d0.nd; ++k) {
    const int64_t e = d0.shape[k];
    int64_t piece = 0;
    if (e > 64)
      for (int64_t c : {32, 64, 16, 48, 40, 24, 56, 8})
        if (e % c == 0) {
          piece = c;
          break;
        }
    if (d.nd + (piece ? 2 : 1) > OM_MAX_DIMS) return false;
    if (piece) {
      d.shape[d.nd] = piece;
      d.sstride[d.nd] = d0.sstride[k];
      dstr[d.nd++] = dstr0[k];
      d.shape[d.nd] = e / piece;
      d.sstride[d.nd] = d0.sstride[k] * piece;
      dstr[d.nd++] = dstr0[k] * piece;
    } else {
      d.shape[d.nd] = e;
      d.sstride[d.nd] = d0.sstride[k];
      dstr[d.nd++] = dstr0[k];
    }
  }
  int sorder[OM_MAX_DIMS];
  for (int k = 0; k < d.nd; ++k) sorder[k] = k;
  std::sort(sorder, sorder + d.nd, [&](int x, int y) { return d.sstride[x] < d.sstride[y]; });
  int64_t expect = 1;
  for (int q = 0; q < d.nd; ++q) {
    if (d.sstride[sorder[q]] != expect) return false;
    expect *= d.shape[sorder[q]];
  }
  bool in_u[OM_MAX_DIMS] = {};
  int64_t t = 1, run = 1;
  for (int k = 0; k < d.nd && run < 32; ++k) {
    in_u[k] = true;
    t *= d.shape[k];
    run *= d.shape[k];
  }
  run = 1;
  for (int q = 0; q < d.nd && run < 32; ++q) {
    int k = sorder[q];
    run *= d.shape[k];
    if (!in_u[k]) {
      in_u[k] = true;
      t *= d.shape[k];
    }
  }
  if (t > kPermMaxTile) return false;
  for (int k = 0; k < d.nd && t < 1024; ++k)
    if (!in_u[k] && t * d.shape[k] <= kPermMaxTile) {
      in_u[k] = true;
      t *= d.shape[k];
    }
  p.nu = p.nr = 0;
  p.t = (int32_t)t;
  int32_t tp = 1;
  for (int k = 0; k < d.nd; ++k) {
    if (in_u[k]) {
      p.u_shape[p.nu] = (int32_t)d.shape[k];
      p.u_sstr[p.nu] = (int32_t)d.sstride[k];
      p.u_dstr[p.nu] = (int32_t)dstr[k];
      p.u_tpos[p.nu] = tp;
      tp *= (int32_t)d.shape[k];
      p.nu++;
    } else {
      p.r_shape[p.nr] = d.shape[k];
      p.r_sstr[p.nr] = d.sstride[k];
      p.r_dstr[p.nr] = dstr[k];
      p.nr++;
    }
  }
  for (int u = 0; u < p.nu; ++u) p.us_order[u] = u;
  std::sort(p.us_order, p.us_order + p.nu,
            [&](int x, int y) { return p.u_sstr[x] < p.u_sstr[y]; });
  p.ntiles = n / t;
  return true;
}

int perm_pad_host(int j) { return j + (j >> 5); }

size_t perm_smem_bytes(const PermDesc& p, size_t es) {
  size_t tables = 4 * (3 * (size_t)p.t + (p.t & 1));
  return tables + 8 * (4 + OM_MAX_DIMS) + es * (size_t)perm_pad_host(p.t);
}

int grid_for(om_backend* be, int64_t work, int per_block) {
  int64_t g = (work + per_block - 1) / per_block;
  int64_t cap = (int64_t)be->num_sms * 32;
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, cap));
}

template <typename T>
int gather_typed(om_backend* be, const T* src, T* dst, GatherDesc d, int64_t n) {
  // destination strides (contiguous column-major)
  int64_t dstr[OM_MAX_DIMS];
  int64_t s = 1;
  for (int k = 0; k < d.nd; ++k) {
    dstr[k] = s;
    s *= d.shape[k];
  }
  if (d.nd == 0) {
    OM_CUDA(cudaMemcpyAsync(dst, src, sizeof(T), cudaMemcpyDeviceToDevice, be->stream), "gather copy");
    return OM_OK;
  }
  if (d.nd == 1 && d.sstride[0] == 1) {
    OM_CUDA(cudaMemcpyAsync(dst, src, sizeof(T) * n, cudaMemcpyDeviceToDevice, be->stream),
            "gather copy");
    return OM_OK;
  }
  if (d.sstride[0] == 1 && d.shape[0] >= 32) {
    int64_t rows = n / d.shape[0];
    int threads = d.shape[0] >= 256 ? 256 : 128;
    gather_rows<T><<<grid_for(be, rows, 1), threads, 0, be->stream>>>(src, dst, d, rows);
    note_launch();
    return check_cuda(cudaGetLastError(), "gather_rows launch");
  }
  {
    // batched 32 x 32 transpose with 16-byte vectors on both sides
    int pv = -1;
    for (int k = 1; k < d.nd; ++k)
      if (d.sstride[k] == 1) pv = k;
    constexpr int64_t V = 16 / sizeof(T);
    bool vec = pv > 0 && d.shape[0] % kTile == 0 && d.shape[pv] % kTile == 0 &&
               ((uintptr_t)src % 16) == 0 && ((uintptr_t)dst % 16) == 0;
    for (int k = 0; k < d.nd && vec; ++k)
      if (k != pv && d.sstride[k] % V != 0) vec = false;
    if (vec) {
      const int64_t tiles0 = d.shape[0] / kTile, tilesp = d.shape[pv] / kTile;
      const int64_t total = n / (kTile * kTile);
      const int64_t g = std::min<int64_t>((total + kTv - 1) / kTv, (int64_t)be->num_sms * 8);
      gather_transpose_vec<T><<<(int)std::max<int64_t>(g, 1), 256, 0, be->stream>>>(
          src, dst, d, pv, dstr[pv], tiles0, tilesp, total);
      note_launch();
      return check_cuda(cudaGetLastError(), "gather_transpose_vec launch");
    }
  }
  {
    PermDesc pd;
    if (plan_perm(d, dstr, n, pd)) {
      size_t smem = perm_smem_bytes(pd, sizeof(T));  // <= 42 KB: no opt-in needed
      int64_t g = std::min<int64_t>(pd.ntiles, (int64_t)be->num_sms * 4);
      gather_perm_tiled<T><<<(int)g, 256, smem, be->stream>>>(src, dst, pd);
      note_launch();
      return check_cuda(cudaGetLastError(), "gather_perm_tiled launch");
    }
  }
  int p = -1;
  for (int k = 1; k < d.nd; ++k)
    if (d.sstride[k] == 1 && d.shape[k] >= 8) p = k;
  if (p > 0 && d.shape[0] >= 8) {
    int64_t tiles0 = (d.shape[0] + kTile - 1) / kTile;
    int64_t tilesp = (d.shape[p] + kTile - 1) / kTile;
    int64_t outer = n / (d.shape[0] * d.shape[p]);
    int64_t total = tiles0 * tilesp * outer;
    dim3 block(kTile, 8);
    gather_transpose<T><<<grid_for(be, total, 1), block, 0, be->stream>>>(
        src, dst, d, p, dstr[p], tiles0, tilesp, total);
    note_launch();
    return check_cuda(cudaGetLastError(), "gather_transpose launch");
  }
  gather_generic<T><<<grid_for(be, n, 256), 256, 0, be->stream>>>(src, dst, d, n);
  note_launch();
  return check_cuda(cudaGetLastError(), "gather_generic launch");
}

template <typename T>
__global__ void fill_kernel(T* dst, int64_t n, T v) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x)
    dst[e] = v;
}

}  // namespace

int launch_fill(om_backend* be, void* dst, size_t es, int64_t n, uint64_t pattern) {
  if (n <= 0) return OM_OK;
  if (es == 8) {
    fill_kernel<uint64_t><<<grid_for(be, n, 256), 256, 0, be->stream>>>((uint64_t*)dst, n, pattern);
  } else {
    fill_kernel<uint32_t><<<grid_for(be, n, 256), 256, 0, be->stream>>>((uint32_t*)dst, n,
                                                                        (uint32_t)pattern);
  }
  note_launch();
  return check_cuda(cudaGetLastError(), "fill launch");
}

int launch_gather(om_backend* be, size_t es, const void* src, int ndim, const int64_t* shape,
                  const int64_t* strides, int64_t offset, void* dst) {
  if (ndim < 0 || ndim > OM_MAX_DIMS) return set_error(OM_ERR_INVALID, "gather: bad rank");
  int64_t n = 1;
  for (int k = 0; k < ndim; ++k) {
    if (shape[k] < 0) return set_error(OM_ERR_INVALID, "gather: negative extent");
    n *= shape[k];
  }
  if (n == 0) return OM_OK;
  // simplify: drop unit axes, then merge axis k+1 into k when the source is
  // contiguous across them (the destination always is)
  GatherDesc d;
  d.nd = 0;
  for (int k = 0; k < ndim; ++k) {
    if (shape[k] == 1) continue;
    if (d.nd > 0 && strides[k] == d.sstride[d.nd - 1] * d.shape[d.nd - 1]) {
      d.shape[d.nd - 1] *= shape[k];
      continue;
    }
    d.shape[d.nd] = shape[k];
    d.sstride[d.nd] = strides[k];
    d.nd++;
  }
  const char* s = (const char*)src + offset * (int64_t)es;
  if (trace_on()) {
    fprintf(stderr, "[om trace] gather es=%zu n=%lld axes=", es, (long long)n);
    for (int k = 0; k < d.nd; ++k)
      fprintf(stderr, "%s%lld:%lld", k ? "," : "", (long long)d.shape[k], (long long)d.sstride[k]);
    fprintf(stderr, "\n");
  }
  ProfScope prof(be, "gather");
  if (es == 8) return gather_typed<uint64_t>(be, (const uint64_t*)s, (uint64_t*)dst, d, n);
  if (es == 4) return gather_typed<uint32_t>(be, (const uint32_t*)s, (uint32_t*)dst, d, n);
  return set_error(OM_ERR_UNSUPPORTED, "gather: element size must be 4 or 8");
}

}  // namespace om

extern "C" int om_b200_copy_strided(om_backend* be, om_dtype dtype, const void* src, int ndim,
                                    const int64_t* shape, const int64_t* strides, int64_t offset,
                                    void* dst) {
  using namespace om;
  if (!be || !src || !dst || (ndim > 0 && (!shape || !strides)))
    return set_error(OM_ERR_INVALID, "om_b200_copy_strided: null argument");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  if (is_complex(dtype)) {  // the two parts as a leading unit-stride axis of extent 2
    if (ndim < 0 || ndim + 1 > OM_MAX_DIMS) return set_error(OM_ERR_INVALID, "gather: bad rank");
    std::vector<int64_t> sh{2}, st{1};
    for (int k = 0; k < ndim; ++k) {
      sh.push_back(shape[k]);
      st.push_back(2 * strides[k]);
    }
    return launch_gather(be, dtype_size(real_part(dtype)), src, ndim + 1, sh.data(), st.data(),
                         2 * offset, dst);
  }
  return launch_gather(be, dtype_size(dtype), src, ndim, shape, strides, offset, dst);
}

// ---- slice staging: many strided views in one launch -----------------------
// Descriptor of one view, as 2 + 2 * kStageDims + 2 int64 words:
//   [src, dst, ndim, numel, shape[kStageDims], strides[kStageDims]]
// (pointers as integers).  The offset of view v in slice s is
// offsets[s * nviews + v]; s is read from the device word *sel, so a
// recorded graph serves every slice and a slice is chosen by one 4-byte
// device copy before the replay.
namespace om {
namespace {
constexpr int kStageDims = 12;
constexpr int kStageWords = 4 + 2 * kStageDims;

template <typename T>
__global__ void gather_views_kernel(const int64_t* __restrict__ desc, int nviews,
                                    const int64_t* __restrict__ offsets,
                                    const int32_t* __restrict__ sel) {
  const int v = blockIdx.y;
  const int64_t* d = desc + (int64_t)v * kStageWords;
  const T* src = (const T*)d[0];
  T* dst = (T*)d[1];
  const int nd = (int)d[2];
  const int64_t n = d[3];
  const int64_t off = offsets[(int64_t)(*sel) * nviews + v];
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = e, at = off;
    for (int q = 0; q < nd; ++q) {
      const int64_t c = rem % d[4 + q];
      rem /= d[4 + q];
      at += c * d[4 + kStageDims + q];
    }
    dst[e] = src[at];
  }
}
}  // namespace
}  // namespace om

extern "C" int om_b200_gather_views(om_backend* be, om_dtype dtype, int nviews, const int64_t* desc,
                                    const int64_t* offsets, const int32_t* sel, int64_t max_numel) {
  using namespace om;
  if (!be || nviews < 0 || (nviews > 0 && (!desc || !offsets || !sel)) || max_numel < 0)
    return set_error(OM_ERR_INVALID, "om_b200_gather_views: bad argument");
  if (nviews > 65535) return set_error(OM_ERR_INVALID, "om_b200_gather_views: more than 65535 views");
  if (nviews == 0 || max_numel == 0) return OM_OK;
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  const unsigned gx = (unsigned)std::max<int64_t>(1, std::min<int64_t>((max_numel + 255) / 256, be->num_sms * 4));
  const dim3 grid(gx, (unsigned)nviews);
  ProfScope prof(be, "gather_views");
  if (dtype == OM_F64)
    gather_views_kernel<double><<<grid, 256, 0, be->stream>>>(desc, nviews, offsets, sel);
  else if (dtype == OM_F32 || dtype == OM_U32)
    gather_views_kernel<float><<<grid, 256, 0, be->stream>>>(desc, nviews, offsets, sel);
  else
    return set_error(OM_ERR_UNSUPPORTED, "om_b200_gather_views: unknown dtype");
  note_launch();
  return check_cuda(cudaGetLastError(), "gather_views launch");
}
