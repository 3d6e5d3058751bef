// Internal host-side declarations shared by the translation units of
// libomeinsum_b200.so.  Nothing here is part of the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <string>
#include <utility>
#include <vector>

#include "omeinsum_b200.h"

struct om_backend {
  int device = 0;
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  // device flag word used by kernels that pick a path on the device
  // (special-value scan of the fast tropical GEMM); lives for the backend.
  uint32_t* d_flags = nullptr;
  // per-kernel event timing (om_b200_profile_*)
  bool profiling = false;
  struct Pending {
    const char* name;
    cudaEvent_t start, stop;
  };
  std::vector<Pending> pending;
  std::vector<std::pair<std::string, std::pair<double, int64_t>>> prof_totals;
};

namespace om {

// ---- errors ---------------------------------------------------------------
int set_error(int code, const std::string& msg);
int check_cuda(cudaError_t e, const char* what);
void note_launch(int n = 1);

// Brackets the kernel launches of its lifetime with CUDA events when the
// backend's profiling is on.
struct ProfScope {
  om_backend* be;
  om_backend::Pending p{};
  ProfScope(om_backend* b, const char* name);
  ~ProfScope();
};

#define OM_TRY(expr)            \
  do {                          \
    int _rc = (expr);           \
    if (_rc != OM_OK) return _rc; \
  } while (0)

#define OM_CUDA(expr, what) OM_TRY(::om::check_cuda((expr), (what)))

inline size_t dtype_size(om_dtype dt) { return dt == OM_F64 ? 8 : 4; }

// ---- scratch memory (stream-ordered, cached by the device pool) -----------
struct Scratch {
  om_backend* be = nullptr;
  void* ptr = nullptr;
  Scratch() = default;
  Scratch(const Scratch&) = delete;
  Scratch& operator=(const Scratch&) = delete;
  ~Scratch();
  int alloc(om_backend* b, size_t bytes);
};

// ---- kernels' host launchers ----------------------------------------------
// Strided gather of an n-d view into a contiguous column-major buffer.
// dst axis d has extent shape[d] and source stride strides[d].
int launch_gather(om_backend* be, size_t elem_size, const void* src, int ndim,
                  const int64_t* shape, const int64_t* strides, int64_t offset, void* dst);

// Batched semiring GEMM on affine layouts:
//   C[m,n,b] = (+)_k A[m,k,b] (x) B[k,n,b]
// with element offsets m*sam + k*sak + b*sab etc.  argmax (optional) shares
// the C strides.
struct GemmArgs {
  om_algebra alg;
  om_dtype dtype;
  int64_t M, N, K, batch;
  const void* A;
  int64_t sam, sak, sab;
  const void* B;
  int64_t sbk, sbn, sbb;
  void* C;
  int64_t scm, scn, scb;
  uint32_t* argmax;  // may be null
  // When set, the exact kernel runs only if the special-value scan of the
  // fast tropical path (bits in *fast_gate) rules the fast path out.
  const uint32_t* fast_gate = nullptr;
};
int launch_gemm(om_backend* be, const GemmArgs& g);

// A mode group decoded element by element: index i of the group is the
// column-major number over its modes (extents ext), and contributes
// sum_j digit_j * s<op>[j] to each operand's offset.
constexpr int kMaxGroupModes = 16;
struct ModeGroup {
  int n = 0;
  int64_t ext[kMaxGroupModes];
  int64_t s0[kMaxGroupModes], s1[kMaxGroupModes], s2[kMaxGroupModes];
};
// Batched small GEMM over strided operands whose groups need not flatten:
// gm strides (A, C), gn (B, C), gk (A, B), gb (A, B, C).
struct StridedGemmArgs {
  om_algebra alg;
  om_dtype dtype;
  int64_t M, N, K, batch;
  const void* A;
  const void* B;
  void* C;
  uint32_t* argmax;
  ModeGroup gm, gn, gk, gb;
};
int launch_gemm_small_strided(om_backend* be, const StridedGemmArgs& g);

// Unary einsum (trace / diagonal / reduce / permute / embed).
int launch_unary(om_backend* be, om_algebra alg, om_dtype dt, const void* x, int nx,
                 const int32_t* ix, const int64_t* shape_x, const int64_t* strides_x, int ny,
                 const int32_t* iy, const int64_t* sizes_y, void* y, uint32_t* argmax);

int launch_fill(om_backend* be, void* dst, size_t elem_size, int64_t n, uint64_t pattern);

}  // namespace om
