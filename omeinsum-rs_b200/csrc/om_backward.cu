// K6: argmax-routed gradient scatter for one tropical binary node.
//
// Restates tropical_backward_normalized (tensor4all/omeinsum-rs
// src/einsum/backward.rs:90-166): for every output element, the argmax is
// decoded (column-major) into the contracted labels, and grad_c is added to
// the one element of A and the one element of B that produced the winner.
// One thread per output element; the additions use atomics, so sums of
// several contributions into one element may round in a different order than
// the reference's sequential loop (exact for integer-valued gradients such as
// the one-hot configurations of MIS problems).
#include <map>

#include "om_internal.h"

namespace om {
namespace {

struct BwdDesc {
  int nc, nk, na, nb;
  int64_t cshape[OM_MAX_DIMS];
  int cslot[OM_MAX_DIMS];
  int64_t kshape[OM_MAX_DIMS];
  int kslot[OM_MAX_DIMS];
  int aslot[OM_MAX_DIMS];
  int64_t astride[OM_MAX_DIMS];
  int bslot[OM_MAX_DIMS];
  int64_t bstride[OM_MAX_DIMS];
};

template <typename T>
__global__ void tropical_scatter(const T* __restrict__ gc, const uint32_t* __restrict__ am,
                                 T* ga, T* gb, BwdDesc d, int64_t n) {
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < n;
       o += (int64_t)gridDim.x * blockDim.x) {
    if (gc[o] == T(0)) continue;
    int64_t val[2 * OM_MAX_DIMS];
    int64_t rem = o;
    for (int k = 0; k < d.nc; ++k) {
      val[d.cslot[k]] = rem % d.cshape[k];
      rem /= d.cshape[k];
    }
    int64_t w = am[o];
    for (int k = 0; k < d.nk; ++k) {
      val[d.kslot[k]] = w % d.kshape[k];
      w /= d.kshape[k];
    }
    int64_t pa = 0, pb = 0;
    for (int k = 0; k < d.na; ++k) pa += val[d.aslot[k]] * d.astride[k];
    for (int k = 0; k < d.nb; ++k) pb += val[d.bslot[k]] * d.bstride[k];
    T g = gc[o];
    // adding an exact zero changes no sum, so zeros are skipped: the
    // gradients of optimisation problems are one-hot and mostly zero, and
    // their many zero contributions would otherwise contend for the same
    // broadcast targets
    if (g != T(0)) {
      atomicAdd(ga + pa, g);
      atomicAdd(gb + pb, g);
    }
  }
}

}  // namespace
}  // namespace om

extern "C" int om_b200_tropical_backward(om_backend* be, om_dtype dtype, const void* grad_c,
                                         const uint32_t* argmax, int nda, const int64_t* shape_a,
                                         const int32_t* modes_a, int ndb, const int64_t* shape_b,
                                         const int32_t* modes_b, int ndc, const int64_t* shape_c,
                                         const int32_t* modes_c, void* grad_a, void* grad_b) {
  using namespace om;
  if (!be || !grad_c || !argmax || !grad_a || !grad_b)
    return set_error(OM_ERR_INVALID, "om_b200_tropical_backward: null pointer");
  if (nda > OM_MAX_DIMS || ndb > OM_MAX_DIMS || ndc > OM_MAX_DIMS || nda < 0 || ndb < 0 || ndc < 0)
    return set_error(OM_ERR_INVALID, "om_b200_tropical_backward: rank out of range");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  BwdDesc d{};
  std::map<int32_t, int> slot;
  auto slot_of = [&](int32_t l) {
    auto it = slot.find(l);
    if (it != slot.end()) return it->second;
    int s = (int)slot.size();
    slot[l] = s;
    return s;
  };
  int64_t n = 1;
  d.nc = ndc;
  for (int k = 0; k < ndc; ++k) {
    d.cslot[k] = slot_of(modes_c[k]);
    d.cshape[k] = shape_c[k];
    n *= shape_c[k];
  }
  d.nk = 0;
  for (int k = 0; k < nda; ++k) {
    bool inb = false, inc = false;
    for (int q = 0; q < ndb; ++q) inb |= modes_b[q] == modes_a[k];
    for (int q = 0; q < ndc; ++q) inc |= modes_c[q] == modes_a[k];
    if (inb && !inc) {
      d.kslot[d.nk] = slot_of(modes_a[k]);
      d.kshape[d.nk] = shape_a[k];
      d.nk++;
    } else if (!inc) {
      return set_error(OM_ERR_SHAPE, "tropical_backward: A has a label outside output/contracted sets");
    }
  }
  int64_t s = 1;
  d.na = nda;
  for (int k = 0; k < nda; ++k) {
    d.aslot[k] = slot_of(modes_a[k]);
    d.astride[k] = s;
    s *= shape_a[k];
  }
  s = 1;
  d.nb = ndb;
  for (int k = 0; k < ndb; ++k) {
    bool ina = false, inc = false;
    for (int q = 0; q < nda; ++q) ina |= modes_a[q] == modes_b[k];
    for (int q = 0; q < ndc; ++q) inc |= modes_c[q] == modes_b[k];
    if (!ina && !inc)
      return set_error(OM_ERR_SHAPE, "tropical_backward: B has a label outside output/contracted sets");
    d.bslot[k] = slot_of(modes_b[k]);
    d.bstride[k] = s;
    s *= shape_b[k];
  }
  if ((int)slot.size() > 2 * OM_MAX_DIMS) return set_error(OM_ERR_INVALID, "too many labels");
  if (n == 0) return OM_OK;
  int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)be->num_sms * 32));
  ProfScope prof(be, "tropical_scatter");
  if (dtype == OM_F32)
    tropical_scatter<float><<<blocks, 256, 0, be->stream>>>((const float*)grad_c, argmax,
                                                            (float*)grad_a, (float*)grad_b, d, n);
  else if (dtype == OM_F64)
    tropical_scatter<double><<<blocks, 256, 0, be->stream>>>((const double*)grad_c, argmax,
                                                             (double*)grad_a, (double*)grad_b, d, n);
  else
    return set_error(OM_ERR_UNSUPPORTED, "tropical_backward: dtype must be f32 or f64");
  note_launch();
  return check_cuda(cudaGetLastError(), "tropical_scatter launch");
}

// ---- index scatter -----------------------------------------------------------
// dst[idx[i]] (+)= src[i]: places the gradient of a slice of a sliced network
// (a strided view of each input tensor) into the full tensors' buffer, or sums
// several slices' gradients there.  The indices are distinct within one call,
// so no atomics are needed.
namespace om {
namespace {
template <typename T>
__global__ void scatter_index_kernel(const T* __restrict__ src, const int64_t* __restrict__ idx,
                                     T* __restrict__ dst, int64_t n, int accumulate) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = idx[i];
    dst[j] = accumulate ? dst[j] + src[i] : src[i];
  }
}
}  // namespace
}  // namespace om

extern "C" int om_b200_scatter_index(om_backend* be, om_dtype dtype, const void* src, int64_t n,
                                     const int64_t* idx, void* dst, int accumulate) {
  using namespace om;
  if (!be || (n > 0 && (!src || !idx || !dst)))
    return set_error(OM_ERR_INVALID, "om_b200_scatter_index: null argument");
  if (n < 0) return set_error(OM_ERR_INVALID, "om_b200_scatter_index: negative length");
  if (n == 0) return OM_OK;
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  const int blocks =
      (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)be->num_sms * 8));
  ProfScope prof(be, "scatter_index");
  if (dtype == OM_F32)
    scatter_index_kernel<float><<<blocks, 256, 0, be->stream>>>((const float*)src, idx,
                                                                (float*)dst, n, accumulate);
  else if (dtype == OM_F64)
    scatter_index_kernel<double><<<blocks, 256, 0, be->stream>>>((const double*)src, idx,
                                                                 (double*)dst, n, accumulate);
  else
    return set_error(OM_ERR_UNSUPPORTED, "om_b200_scatter_index: dtype must be f32 or f64");
  note_launch();
  return check_cuda(cudaGetLastError(), "scatter_index launch");
}
