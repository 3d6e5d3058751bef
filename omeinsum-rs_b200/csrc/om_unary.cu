// K5: unary einsum on the device -- trace, diagonal, reduction, permutation
// and diagonal embedding, with optional argmax.
//
// Restates execute_unary_naive / execute_unary_with_argmax
// (tensor4all/omeinsum-rs src/einsum/engine.rs:752-832, 841-926):
//   * inner labels = labels of ix absent from iy, deduplicated in ix order,
//     enumerated column-major;
//   * repeated output labels select the diagonal; other positions get zero();
//   * the value path folds with Semiring::add (first element wins ties);
//   * the argmax path starts from the first inner element and replaces it only
//     when Algebra::is_better (strict), recording the column-major linear
//     position of the winner in the input's logical shape.
// One thread per output element; the inner loop runs in the reference's order.
#include <algorithm>
#include <map>
#include <vector>

#include "om_internal.h"
#include "om_semiring.cuh"

namespace om {
namespace {

struct UnaryDesc {
  int nx, ny, ninner, nslots;
  int xslot[OM_MAX_DIMS];
  int64_t xstride[OM_MAX_DIMS];
  int64_t xlogical[OM_MAX_DIMS];  // column-major strides of the logical shape
  int yslot[OM_MAX_DIMS];
  int64_t ysize[OM_MAX_DIMS];
  int islot[OM_MAX_DIMS];
  int64_t isize[OM_MAX_DIMS];
  int64_t inner_total;
};

template <typename T, int ALG, bool ARGMAX>
__global__ void unary_kernel(const T* __restrict__ x, T* __restrict__ y, uint32_t* __restrict__ am,
                             UnaryDesc d, int64_t nout) {
  using S = Semi<ALG, T>;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < nout;
       o += (int64_t)gridDim.x * blockDim.x) {
    int64_t val[OM_MAX_DIMS];
    bool set[OM_MAX_DIMS];
    for (int s = 0; s < d.nslots; ++s) set[s] = false;
    int64_t rem = o;
    bool skip = false;
    for (int k = 0; k < d.ny; ++k) {
      int64_t c = rem % d.ysize[k];
      rem /= d.ysize[k];
      int s = d.yslot[k];
      if (set[s] && val[s] != c) skip = true;
      set[s] = true;
      val[s] = c;
    }
    T best = S::zero();
    uint32_t bpos = 0;
    if (!skip) {
      for (int64_t in = 0; in < d.inner_total; ++in) {
        int64_t r2 = in;
        for (int k = 0; k < d.ninner; ++k) {
          val[d.islot[k]] = r2 % d.isize[k];
          r2 /= d.isize[k];
        }
        int64_t off = 0, lpos = 0;
        for (int k = 0; k < d.nx; ++k) {
          off += val[d.xslot[k]] * d.xstride[k];
          lpos += val[d.xslot[k]] * d.xlogical[k];
        }
        T v = x[off];
        if (ARGMAX) {
          if (in == 0 || S::better(v, best)) {
            best = v;
            bpos = (uint32_t)lpos;
          }
        } else {
          best = S::add(best, v);
        }
      }
    }
    y[o] = best;
    if (ARGMAX) am[o] = bpos;
  }
}

template <typename T, int ALG>
int launch_typed(om_backend* be, const T* x, T* y, uint32_t* am, const UnaryDesc& d, int64_t nout) {
  int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((nout + 127) / 128, (int64_t)be->num_sms * 32));
  ProfScope prof(be, "unary");
  if (am)
    unary_kernel<T, ALG, true><<<blocks, 128, 0, be->stream>>>(x, y, am, d, nout);
  else
    unary_kernel<T, ALG, false><<<blocks, 128, 0, be->stream>>>(x, y, am, d, nout);
  note_launch();
  return check_cuda(cudaGetLastError(), "unary launch");
}

}  // namespace

int launch_unary(om_backend* be, om_algebra alg, om_dtype dt, const void* x, int nx,
                 const int32_t* ix, const int64_t* shape_x, const int64_t* strides_x, int ny,
                 const int32_t* iy, const int64_t* sizes_y, void* y, uint32_t* argmax) {
  if (nx < 0 || ny < 0 || nx > OM_MAX_DIMS || ny > OM_MAX_DIMS)
    return set_error(OM_ERR_INVALID, "unary: rank out of range");
  if (is_complex(dt)) {
    // Standard sums act on the real and imaginary parts alike: a real unary
    // einsum with a part label (extent 2, stride 1) kept in front
    if (alg != OM_STANDARD)
      return set_error(OM_ERR_UNSUPPORTED, "unary: complex dtypes take the Standard algebra only");
    if (nx + 1 > OM_MAX_DIMS || ny + 1 > OM_MAX_DIMS)
      return set_error(OM_ERR_INVALID, "unary: rank out of range");
    int32_t top = 0;
    for (int k = 0; k < nx; ++k) top = std::max(top, ix[k]);
    for (int k = 0; k < ny; ++k) top = std::max(top, iy[k]);
    std::vector<int32_t> rix{top + 1}, riy{top + 1};
    std::vector<int64_t> rsh{2}, rst{1}, rsy{2};
    for (int k = 0; k < nx; ++k) {
      rix.push_back(ix[k]);
      rsh.push_back(shape_x[k]);
      rst.push_back(2 * strides_x[k]);
    }
    for (int k = 0; k < ny; ++k) {
      riy.push_back(iy[k]);
      rsy.push_back(sizes_y[k]);
    }
    int64_t nout = 1;
    for (int k = 0; k < ny; ++k) nout *= sizes_y[k];
    if (argmax && nout > 0)
      OM_CUDA(cudaMemsetAsync(argmax, 0, 4 * (size_t)nout, be->stream), "argmax zero");
    return launch_unary(be, alg, real_part(dt), x, nx + 1, rix.data(), rsh.data(), rst.data(),
                        ny + 1, riy.data(), rsy.data(), y, nullptr);
  }
  UnaryDesc d{};
  std::map<int32_t, int> slot;
  std::map<int32_t, int64_t> size;
  auto slot_of = [&](int32_t l) {
    auto it = slot.find(l);
    if (it != slot.end()) return it->second;
    int s = (int)slot.size();
    slot[l] = s;
    return s;
  };
  d.nx = nx;
  d.ny = ny;
  int64_t ls = 1;
  for (int k = 0; k < nx; ++k) {
    d.xslot[k] = slot_of(ix[k]);
    d.xstride[k] = strides_x[k];
    d.xlogical[k] = ls;
    ls *= shape_x[k];
    auto it = size.find(ix[k]);
    if (it != size.end() && it->second != shape_x[k])
      return set_error(OM_ERR_SHAPE, "unary: repeated input label with different extents");
    size[ix[k]] = shape_x[k];
  }
  int64_t nout = 1;
  for (int k = 0; k < ny; ++k) {
    d.yslot[k] = slot_of(iy[k]);
    d.ysize[k] = sizes_y[k];
    auto it = size.find(iy[k]);
    if (it != size.end() && it->second != sizes_y[k])
      return set_error(OM_ERR_SHAPE, "unary: output label extent differs from input");
    size[iy[k]] = sizes_y[k];
    nout *= sizes_y[k];
  }
  d.ninner = 0;
  d.inner_total = 1;
  for (int k = 0; k < nx; ++k) {
    bool in_y = false, seen = false;
    for (int q = 0; q < ny; ++q) in_y |= (iy[q] == ix[k]);
    for (int q = 0; q < d.ninner; ++q) seen |= (d.islot[q] == d.xslot[k]);
    if (in_y || seen) continue;
    d.islot[d.ninner] = d.xslot[k];
    d.isize[d.ninner] = shape_x[k];
    d.inner_total *= shape_x[k];
    d.ninner++;
  }
  d.nslots = (int)slot.size();
  if (d.nslots > OM_MAX_DIMS) return set_error(OM_ERR_INVALID, "unary: too many labels");
  if (nout == 0) return OM_OK;
  if (dt == OM_F32) {
    OM_DISPATCH_ALG(alg, ALG,
                    return launch_typed<float, ALG>(be, (const float*)x, (float*)y, argmax, d, nout));
  } else if (dt == OM_F64) {
    OM_DISPATCH_ALG(alg, ALG,
                    return launch_typed<double, ALG>(be, (const double*)x, (double*)y, argmax, d, nout));
  }
  return set_error(OM_ERR_UNSUPPORTED, "unary: dtype must be f32 or f64");
}

}  // namespace om

extern "C" int om_b200_unary(om_backend* be, om_algebra alg, om_dtype dtype, const void* x, int nx,
                             const int32_t* ix, const int64_t* shape_x, const int64_t* strides_x,
                             int ny, const int32_t* iy, const int64_t* sizes_y, void* y_out,
                             uint32_t* argmax_out) {
  using namespace om;
  if (!be || !x || !y_out || (nx && (!ix || !shape_x || !strides_x)) || (ny && (!iy || !sizes_y)))
    return set_error(OM_ERR_INVALID, "om_b200_unary: null argument");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  return launch_unary(be, alg, dtype, x, nx, ix, shape_x, strides_x, ny, iy, sizes_y, y_out,
                      argmax_out);
}
