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

namespace om {
struct Arena;
}

struct om_backend {
  int device = 0;
  // process-unique id: a freed backend's address can be reused by a later
  // one, so owners of its buffers check liveness by (address, id)
  uint64_t id = 0;
  // while a graph is being recorded, the library's own device memory comes
  // from this arena (owned by the graph) instead of the stream-ordered pool
  om::Arena* recording = nullptr;
  cudaStream_t stream = nullptr;
  // branches of a recording (om_b200_graph_branch): while one is selected,
  // `stream` is that branch's stream and `main_stream` the backend's own
  cudaStream_t main_stream = nullptr;
  std::vector<cudaStream_t> branch_streams;
  std::vector<char> branch_joined;  // branch forked into the current recording
  cudaEvent_t fork_event = nullptr;
  bool branching = false;           // a recording with branches is open
  int num_sms = 148;
  // device flag word used by kernels that pick a path on the device
  // (special-value scan of the fast tropical GEMM); lives for the backend.
  uint32_t* d_flags = nullptr;
  // Standard f32 products on the tensor cores (3xTF32) or exact FMA
  bool f32_exact = false;
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
// OM_B200_TRACE=1 in the environment: one stderr line per planner decision
bool trace_on();

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

inline size_t dtype_size(om_dtype dt) {
  return dt == OM_C64 ? 16 : (dt == OM_F64 || dt == OM_C32) ? 8 : 4;
}
inline bool is_complex(om_dtype dt) { return dt == OM_C32 || dt == OM_C64; }
// the real type of a complex dtype's parts
inline om_dtype real_part(om_dtype dt) { return dt == OM_C64 ? OM_F64 : OM_F32; }

// ---- device memory of the library's own buffers --------------------------
// Outside a recording: the device's stream-ordered pool (cudaMallocAsync /
// cudaFreeAsync).  While a graph is recorded: a first-fit arena owned by the
// graph, so the recorded work always finds its buffers at the same addresses
// and different graphs never trade physical memory between replays (all
// recorded work runs on one stream, in recording order, so reusing a freed
// block inside the arena is safe).
struct Arena {
  // while branches record concurrently running work, freed blocks are not
  // handed out again (another branch may still be using them at replay)
  bool defer = false;
  std::vector<void*> deferred;
  std::vector<std::pair<char*, size_t>> chunks;
  std::map<char*, size_t> free_blocks;  // address-ordered, coalesced
  std::map<char*, size_t> used;
  bool owns(const void* p) const;
  int alloc(size_t bytes, void** out);
  void release(void* p);
  void destroy();
};
int be_alloc(om_backend* be, size_t bytes, void** out);
// frees p: into the live arena that holds it, if any (a destroyed arena's
// blocks are gone with it), else stream-ordered to the pool
void be_free(om_backend* be, uint64_t id, void* p);
void arena_register(Arena* a);
void arena_unregister(Arena* a);

// ---- scratch memory (stream-ordered, cached by the device pool) -----------
struct Scratch {
  om_backend* be = nullptr;
  uint64_t be_id = 0;
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
  // Two-level indices, only for the tensor-core Standard f32 path
  // (tf32_takes): k = k1 + ka1 * k2 reads A at k1 * sak + k2 * sak2 (ka1 a
  // multiple of 32; ka1 == 0 means the flat stride sak), and likewise for
  // B's k (kb1, sbk2), A's rows (ma1, sam2) and B's columns (nb1, sbn2).
  int64_t ka1 = 0, sak2 = 0, kb1 = 0, sbk2 = 0;
  int64_t ma1 = 0, sam2 = 0, nb1 = 0, sbn2 = 0;
};
int launch_gemm(om_backend* be, const GemmArgs& g);
// Whether the f64 DFMA kernel takes these arguments (orientation,
// alignment, two-level k)
bool f64_dfma_takes(om_backend* be, const GemmArgs& g);
#ifdef __CUDACC__
// offset of contracted index k along a possibly two-level k (n1 == 0: flat)
__host__ __device__ __forceinline__ int64_t kofs(int64_t k, int64_t s1, int64_t n1, int64_t s2) {
  return n1 ? (k % n1) * s1 + (k / n1) * s2 : k * s1;
}
#endif
// Standard f64 GEMM on the FP64 pipes; *handled false leaves the shape to
// the generic kernels
int launch_gemm_f64(om_backend* be, const GemmArgs& g, bool* handled);
// Whether launch_gemm gives this Standard f32 problem to the tensor-core
// kernel (the only kernel that reads a two-level contracted index).
bool tf32_takes(const om_backend* be, om_algebra alg, om_dtype dt, bool argmax, int64_t M,
                int64_t N, int64_t K, int64_t batch);

// Unsigned 32-bit division by an invariant divisor d >= 1 with one
// multiply-high, exact for every dividend below 2^32 (Granlund & Montgomery,
// "Division by invariant integers using multiplication", PLDI 1994, fig. 4.1):
// l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1,
// q = (t + ((n - t) >> min(l, 1))) >> max(l - 1, 0) with t = umulhi(m, n).
struct FastDiv {
  uint32_t d, m, s1, s2;
};
inline FastDiv make_fastdiv(uint32_t d) {
  int l = 0;
  while ((uint64_t(1) << l) < d) ++l;
  const uint64_t m = ((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1;
  return FastDiv{d, (uint32_t)m, (uint32_t)(l < 1 ? l : 1), (uint32_t)(l > 0 ? l - 1 : 0)};
}
#ifdef __CUDACC__
__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv& f) {
  const uint32_t t = __umulhi(f.m, n);
  return (t + ((n - t) >> f.s1)) >> f.s2;
}
#endif

// Contraction of a small or heavily batched tensor-network node read in
// place through per-mode strides (no gather, no flattening needed).  The
// output is contiguous; its modes are listed in memory order with the
// strides they have in A and B (0 where absent), adjacent modes that are
// contiguous in both operands merged.  The first nlow output modes (product
// P) form a tile whose A/B offsets are tabulated per block; the remaining
// modes are decoded once per tile row.  The contracted modes are listed in
// modes_a order, so k is the reference's column-major argmax index.
constexpr int kMaxNodeModes = 40;
struct NodeMode {
  FastDiv div;
  int64_t sa, sb;
  int64_t sc;  // C stride (gemm_node's row modes; set by its launcher)
};
struct NodeArgs {
  om_algebra alg;
  om_dtype dtype;
  int64_t K;
  int64_t total;  // output elements
  int64_t rows;   // total / P, below 2^32
  int32_t P;
  int nlow, nout, nk;
  const void* A;
  const void* B;
  void* C;
  uint32_t* argmax;
  NodeMode out[kMaxNodeModes];
  NodeMode kmodes[kMaxNodeModes];
  int64_t ia[4], ib[4];  // A/B offsets of the outputs inside a group of 4 (set by the launcher)
  int wa, wb;  // 4: ia = {0,1,2,3}; 2: {0,1,x,x+1}; 0: all 0; 3: {0,0,x,x}; 5: {0,x,0,x}; 1: other
  // gemm_node: the first nrep row modes (out[nlow .. nlow + nrep)) are ones
  // A does not carry; their R combinations run inside a thread, which keeps
  // its A values in registers across them (set by the launcher)
  int nrep;
  int32_t R;
};
int launch_gemm_node(om_backend* be, const NodeArgs& g);

// Unary einsum (trace / diagonal / reduce / permute / embed).
int launch_unary(om_backend* be, om_algebra alg, om_dtype dt, const void* x, int nx,
                 const int32_t* ix, const int64_t* shape_x, const int64_t* strides_x, int ny,
                 const int32_t* iy, const int64_t* sizes_y, void* y, uint32_t* argmax);

int launch_fill(om_backend* be, void* dst, size_t elem_size, int64_t n, uint64_t pattern);

}  // namespace om
