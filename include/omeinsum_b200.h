/*
 * omeinsum_b200.h -- C ABI of the B200 (sm_100a) execution backend for
 * omeinsum-rs.
 *
 * The entry points replace the reference's `Backend` trait for a new `B200`
 * backend (tensor4all/omeinsum-rs, src/backend/traits.rs:42-199): a Rust
 * `impl Backend for B200` binds them one-to-one.
 *
 * Conventions (same as the reference):
 *   - tensors are column-major: axis 0 is fastest; strides count ELEMENTS;
 *   - modes are arbitrary int32 labels, unique within one operand;
 *   - a mode in A, B and C is a batch mode; in A and B only, contracted; in
 *     one input and C, free; in one input only, traced (reduced first);
 *   - outputs are written contiguous column-major in modes_c order;
 *   - argmax (u32) is the column-major linear index over the contracted
 *     modes, taken in modes_a order; ties go to the smallest index;
 *   - MaxPlus zero = -FLT_MAX (f32::MIN), MinPlus zero = +FLT_MAX, MaxMul zero = 0.
 *
 * All device pointers are plain CUDA device addresses on the backend's device.
 * Every call is ordered on the backend's own stream; om_b200_sync waits for it.
 * Every function returns OM_OK (0) or an OM_ERR_* code; om_b200_last_error
 * gives the message of the last failure on the calling thread.
 */
#ifndef OMEINSUM_B200_H
#define OMEINSUM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct om_backend om_backend;

/* semirings: src/algebra/standard.rs, src/algebra/tropical.rs */
typedef enum {
  OM_STANDARD = 0, /* (+, x)   zero 0            */
  OM_MAXPLUS = 1,  /* (max, +) zero -FLT_MAX     */
  OM_MINPLUS = 2,  /* (min, +) zero +FLT_MAX     */
  OM_MAXMUL = 3    /* (max, x) zero 0            */
} om_algebra;

/* OM_C32 / OM_C64: complex numbers as interleaved (re, im) pairs of
 * f32 / f64 (the layout of num_complex::Complex and of the reference's
 * CudaComplex, src/backend/cuda/mod.rs:56-208); Standard algebra only. */
typedef enum { OM_F32 = 0, OM_F64 = 1, OM_U32 = 2, OM_C32 = 3, OM_C64 = 4 } om_dtype;

enum {
  OM_OK = 0,
  OM_ERR_INVALID = 1,     /* bad argument: null pointer, bad rank, size mismatch */
  OM_ERR_UNSUPPORTED = 2, /* dtype / algebra combination not provided            */
  OM_ERR_CUDA = 3,        /* CUDA runtime error                                  */
  OM_ERR_OOM = 4,         /* device allocation failed                            */
  OM_ERR_SHAPE = 5,       /* modes / shapes inconsistent                         */
  OM_ERR_NCCL = 6,        /* collective failed                                   */
  OM_ERR_TIMEOUT = 7      /* a bounded wait ran out                              */
};

#define OM_MAX_DIMS 64

/* Backend::name (traits.rs:50) -- returns "b200". */
const char* om_b200_name(void);

/* Copies the last error message of this thread into buf (NUL-terminated). */
int om_b200_last_error(char* buf, size_t len);

/* Creates a backend bound to CUDA device `device` with its own non-blocking
 * stream and a stream-ordered caching allocator.  Mirrors `Cuda::on_device`
 * (src/backend/cuda/mod.rs:258-265): a bad ordinal is an error, not a panic. */
int om_b200_create(int device, om_backend** out);
int om_b200_destroy(om_backend* be);

/* The backend's stream (a cudaStream_t), for callers that interoperate. */
int om_b200_stream(om_backend* be, void** stream_out);

/* Backend::synchronize (traits.rs:53). */
int om_b200_sync(om_backend* be);

/* Backend::alloc (traits.rs:56): zero-filled device buffer of `bytes`. */
int om_b200_alloc(om_backend* be, size_t bytes, void** dptr);
int om_b200_free(om_backend* be, void* dptr);

/* Backend::from_slice (traits.rs:60) is alloc + upload; Storage::to_vec
 * (traits.rs:20) is download.  Both are stream-ordered; download waits. */
int om_b200_upload(om_backend* be, void* dst_device, const void* src_host, size_t bytes);
int om_b200_download(om_backend* be, void* dst_host, const void* src_device, size_t bytes);
/* om_b200_download without the wait: the copy is queued on the backend's
 * stream and dst_host must stay valid until om_b200_sync returns (use pinned
 * host memory for a truly asynchronous copy).  No counterpart in the
 * reference (Storage::to_vec always waits); a caller that overlaps one
 * step's copies with another step's contraction on a second backend uses it. */
int om_b200_download_async(om_backend* be, void* dst_host, const void* src_device, size_t bytes);

/* Backend::copy_strided (traits.rs:71-77): gathers the strided view
 * (shape, strides, offset in elements) of src into the contiguous
 * column-major dst.  dtype gives the element size (OM_U32 allowed). */
int om_b200_copy_strided(om_backend* be, om_dtype dtype, const void* src, int ndim,
                         const int64_t* shape, const int64_t* strides, int64_t offset, void* dst);

/* Backend::contract (traits.rs:147-166) when argmax_out == NULL, and
 * Backend::contract_with_argmax (traits.rs:180-199) otherwise.  The output
 * c_out (and argmax_out) hold prod(shape_c) elements (1 when ndc == 0).
 * Inputs are read through their strides; nothing is copied back to the host. */
int om_b200_contract(om_backend* be, om_algebra alg, om_dtype dtype,
                     const void* a, int nda, const int64_t* shape_a, const int64_t* strides_a,
                     const int32_t* modes_a,
                     const void* b, int ndb, const int64_t* shape_b, const int64_t* strides_b,
                     const int32_t* modes_b,
                     int ndc, const int64_t* shape_c, const int32_t* modes_c,
                     void* c_out, uint32_t* argmax_out);

/* Unary einsum ix -> iy (execute_unary_naive / execute_unary_with_argmax,
 * src/einsum/engine.rs:752-926): trace, diagonal, reduction, permutation and
 * diagonal embedding.  ix may repeat labels; iy may repeat labels (off-diagonal
 * entries get the algebra's zero).  sizes_y[d] is the size of iy[d]; the input
 * is read through shape_x/strides_x.  argmax_out (optional) receives the
 * column-major linear input position of the winner (is_better, first wins). */
int om_b200_unary(om_backend* be, om_algebra alg, om_dtype dtype,
                  const void* x, int nx, const int32_t* ix, const int64_t* shape_x,
                  const int64_t* strides_x,
                  int ny, const int32_t* iy, const int64_t* sizes_y,
                  void* y_out, uint32_t* argmax_out);

/* Tropical backward of one binary node (src/einsum/backward.rs:90-166):
 * scatters grad_c into grad_a / grad_b (contiguous, column-major, shapes of
 * the normalised operands, ACCUMULATED into) through the argmax of the
 * forward contraction.  Operands are given by shape and modes only. */
int om_b200_tropical_backward(om_backend* be, om_dtype dtype,
                              const void* grad_c, const uint32_t* argmax,
                              int nda, const int64_t* shape_a, const int32_t* modes_a,
                              int ndb, const int64_t* shape_b, const int32_t* modes_b,
                              int ndc, const int64_t* shape_c, const int32_t* modes_c,
                              void* grad_a, void* grad_b);

/* Arithmetic of Standard<f32> products (no counterpart in the reference,
 * whose faer path is plain f32):
 *   OM_F32_TENSOR_3XTF32 (default): shapes of at least 64 x 64 x 16 run on the
 *     tensor cores (tcgen05) as three TF32 products per f32 product
 *     (A_lo B_hi + A_hi B_lo + A_hi B_hi) accumulated in f32; the error is
 *     about 2^-21 * sum_k |a||b|.  Smaller shapes use the exact path.
 *   OM_F32_EXACT: every Standard f32 product is an f32 FMA on the CUDA cores.
 * The environment variable OM_DISABLE_TCGEN05 (any value) makes OM_F32_EXACT
 * the default of new backends.  f64 and the tropical algebras are unaffected. */
typedef enum { OM_F32_TENSOR_3XTF32 = 0, OM_F32_EXACT = 1 } om_f32_mode;
int om_b200_set_f32_mode(om_backend* be, om_f32_mode mode);

/* dst[idx[i]] = src[i] (accumulate == 0) or dst[idx[i]] += src[i]
 * (accumulate != 0) for 0 <= i < n; idx is a device array of distinct int64
 * element offsets into dst.  No counterpart in the reference: the sliced
 * network driver uses it to place a slice's gradients (views of the inputs)
 * into the full gradient tensors on the device, and to sum slices there. */
int om_b200_scatter_index(om_backend* be, om_dtype dtype, const void* src, int64_t n,
                          const int64_t* idx, void* dst, int accumulate);

/* Many strided gathers in one launch (no counterpart in the reference: the
 * sliced network driver stages a slice's views of the sliced input tensors
 * with it).  desc (device) holds nviews descriptors of 28 int64 words each:
 * source pointer, destination pointer, ndim (<= 12), element count, then 12
 * extents and 12 element strides (column-major odometer over the extents).
 * View v of slice s starts at element offsets[s * nviews + v] (device) of its
 * source; s is read on the device from *sel, so a graph recorded around this
 * call serves every slice.  Destinations are contiguous.  max_numel bounds
 * the views' element counts (it sizes the grid). */
int om_b200_gather_views(om_backend* be, om_dtype dtype, int nviews, const int64_t* desc,
                         const int64_t* offsets, const int32_t* sel, int64_t max_numel);

/* Contraction-order optimisation by tree simulated annealing (host code;
 * replaces the reference's call into omeco's optimize_treesa,
 * src/einsum/engine.rs:84-91).  Network as in om_b200_einsum (ntensors,
 * ndims, ixs, iy, size dictionary).  init_children (2 * (ntensors - 1),
 * post order, may be NULL) seeds the first of ntrials runs; the others start
 * from random trees.  Cost: log2 sum of 2^tc over nodes + sc_weight * sum
 * of max(0, log2 size - sc_target) over intermediates + rw_weight * log2 of
 * the read-write volume; Metropolis moves (rotations at a node), beta from
 * beta_start to beta_end by beta_step, niters sweeps per beta.  Writes the
 * best tree to children_out (post order) and its log2 time / space
 * complexity to tc_out / sc_out (may be NULL). */
int om_b200_optimize_tree(int ntensors, const int32_t* ndims, const int32_t* ixs, int niy,
                          const int32_t* iy, int nsizes, const int32_t* size_labels,
                          const int64_t* size_values, const int32_t* init_children,
                          double sc_target, double sc_weight, double rw_weight, int ntrials,
                          int niters, double beta_start, double beta_end, double beta_step,
                          uint64_t seed, int32_t* children_out, double* tc_out, double* sc_out);

/* Kernel launches issued by this thread since the last call (counter reset
 * on read); used by benchmarks to report how many device kernels ran. */
int64_t om_b200_launch_count(void);

/* Per-kernel device timing: with profiling on, each kernel launch of this
 * backend is bracketed by CUDA events on the backend's stream.  Turning it on
 * clears the accumulators.  om_b200_profile_query synchronises the stream and
 * returns, for kernel class `index` (0, 1, ...), its name, summed device time
 * and launch count; OM_ERR_INVALID once index runs past the last class. */
int om_b200_profile_enable(om_backend* be, int on);
int om_b200_profile_query(om_backend* be, int index, char* name, size_t len, double* total_ms,
                          int64_t* launches);

/* ---- einsum engine over a contraction tree --------------------------------
 * Restates Einsum::execute / execute_with_argmax and the gradient tape of
 * cost_and_gradient (src/einsum/engine.rs:125-301,392-578;
 * src/einsum/backward.rs:405-799) on the device.
 *
 * Inputs: `ntensors` device tensors; tensor t has rank ndims[t], and its
 * shape, strides and labels are the next ndims[t] entries of shapes / strides
 * / ixs (concatenated over t).  Labels are int32 >= 0; size_labels[q] has
 * extent size_values[q] (the size dictionary).  iy (length niy) are the
 * output labels.
 *
 * Tree: `nnodes` binary nodes in post order.  Node i contracts children
 * children[2i], children[2i+1]; a child value c < ntensors is leaf tensor c,
 * c >= ntensors is node c - ntensors.  Its output labels are
 * node_iy[node_iy_off[i] .. node_iy_off[i+1]).  The last node is the root.
 * nnodes == 0 means the tree is the single leaf 0 (a unary einsum).
 *
 * Operands are normalised before each node (labels in neither the other
 * operand nor the node output are reduced first, repeated labels take the
 * diagonal), and the root is reduced / permuted to iy at the end.  `out`
 * receives prod(extent of iy) contiguous column-major elements.
 *
 * With tape_out non-NULL the forward keeps a gradient tape (argmax of every
 * node for the tropical algebras, every intermediate for Standard); pass it
 * to om_b200_einsum_backward, then free it with om_b200_tape_free. */
typedef struct om_tape om_tape;
int om_b200_einsum(om_backend* be, om_algebra alg, om_dtype dtype, int ntensors,
                   const void* const* tensors, const int32_t* ndims, const int64_t* shapes,
                   const int64_t* strides, const int32_t* ixs, int niy, const int32_t* iy,
                   int nsizes, const int32_t* size_labels, const int64_t* size_values,
                   int nnodes, const int32_t* children, const int32_t* node_iy_off,
                   const int32_t* node_iy, void* out, om_tape** tape_out);

/* om_b200_einsum with a tape of values only (tropical algebras): every
 * intermediate is kept, but no node computes its argmax.  The backward
 * (om_b200_einsum_backward / _linked, outputs of at most 4096 elements)
 * then finds the argmax of just the elements the gradient visits, from the
 * children's values, with the same rule as the forward (generic_gemm_with_argmax,
 * src/backend/cpu/mod.rs:889-920, and execute_unary_with_argmax,
 * src/einsum/engine.rs:841-926), so the gradient is the one the argmax tape
 * gives.  No counterpart in the reference: it lets a caller contract many
 * candidates (the slices of a sliced network) at value cost and take the
 * gradient of the winner only. */
int om_b200_einsum_tape_values(om_backend* be, om_algebra alg, om_dtype dtype, int ntensors,
                               const void* const* tensors, const int32_t* ndims,
                               const int64_t* shapes, const int64_t* strides, const int32_t* ixs,
                               int niy, const int32_t* iy, int nsizes, const int32_t* size_labels,
                               const int64_t* size_values, int nnodes, const int32_t* children,
                               const int32_t* node_iy_off, const int32_t* node_iy, void* out,
                               om_tape** tape_out);

/* GradientTape::backward (backward.rs:498-506, 678-728): given dy (shaped
 * like the output, contiguous), writes the gradient of every input tensor t,
 * contiguous column-major in the input's shape, to grads[t]. */
int om_b200_einsum_backward(om_tape* tape, const void* dy, void* const* grads);

/* One backward through several tapes (no counterpart in the reference):
 * input tensor link_leaf[i] of `tape` is the output of the contraction
 * recorded in link_tapes[i] (same algebra and dtype, its output contiguous in
 * that leaf's label order); the gradient continues through it, and the
 * inputs of link_tapes[i] receive theirs in link_grads[i][...].  grads[] of
 * linked leaves are not written.  Tropical tapes whose output has at most
 * 4096 elements only (the walk of om_b200_einsum_backward for small
 * gradients, in one launch for all tapes); otherwise OM_ERR_UNSUPPORTED. */
int om_b200_einsum_backward_linked(om_tape* tape, const void* dy, void* const* grads, int nlinks,
                                   const int32_t* link_leaf, om_tape* const* link_tapes,
                                   void* const* const* link_grads);
int om_b200_tape_free(om_tape* tape);

/* For a tape recorded inside a graph (om_b200_graph_begin/end): frees the
 * device buffers the tape refers to, stream-ordered, and keeps the tape.  A
 * later replay of the graph allocates the same addresses again, after which
 * om_b200_einsum_backward may run on the tape once more.  This keeps a
 * recorded tape from holding its memory between replays.  Not meant for
 * tapes made outside a graph (their buffers would not come back). */
int om_b200_tape_release(om_tape* tape);

/* Stream capture into a CUDA graph.  No counterpart in the reference (its
 * CPU backend has no launch cost to amortise); it serves callers that repeat
 * the same sequence of library calls on the same buffers, such as the slices
 * of a sliced network.  Between om_b200_graph_begin and om_b200_graph_end,
 * work issued on the backend's stream (om_b200_contract, om_b200_einsum,
 * copies, ...) is recorded instead of run; the library's own stream-ordered
 * allocations inside become part of the graph.  om_b200_graph_launch runs the
 * recorded work on the backend's stream.  Calls that wait for the device
 * (om_b200_sync, om_b200_download, profile queries) must not be made while
 * capturing. */
typedef struct om_graph om_graph;
int om_b200_graph_begin(om_backend* be);
int om_b200_graph_end(om_backend* be, om_graph** graph_out);
int om_b200_graph_launch(om_backend* be, om_graph* graph);
int om_b200_graph_free(om_graph* graph);

/* Concurrent branches of a recording (no reference counterpart): after
 * om_b200_graph_branch(be, b) with 0 <= b < 64, the work issued on the
 * backend is recorded on branch b, which starts after everything recorded
 * before the first branch call; om_b200_graph_branch(be, -1) returns to the
 * backend's own stream.  om_b200_graph_end joins every branch, so the graph
 * ends after all of them.  Branches run concurrently at replay and must use
 * disjoint buffers; blocks the library frees inside them are not reused
 * within the recording.  Tropical f32 GEMMs inside branches take the exact
 * compare-select path (the fast path's gate word is one per backend). */
int om_b200_graph_branch(om_backend* be, int branch);

/* Allocation-free tropical matrix product with argmax.  No counterpart in the
 * reference: it exists for callers that must not allocate device memory
 * while they run (a host that hands all device memory out of its own arena,
 * a latency-critical path where an allocation could block or fail, an
 * embedder that forbids library-owned allocations).
 *
 * C = A (x) B in MaxPlus / MinPlus / MaxMul f32, with the u32 argmax of the
 * first winning k (same results as om_b200_contract with modes
 * 'ij,jk->ik').  A (m x k, leading dimension lda), B (k x n, ldb), C and
 * argmax (m x n, ldc) are column-major device buffers owned by the caller;
 * work is issued on `stream` (a cudaStream_t; NULL = legacy default stream)
 * and no om_backend is needed.  Nothing is allocated: the kernel's scratch
 * lives in fixed device arrays of the library (32 MiB + 64 bytes, held on
 * every GPU that loads the library until the process exits), which limits
 * ceil(m/128) * ceil(n/64) * ceil(k/32) to 32768; larger problems on the
 * fast path fail with OM_ERR_INVALID (use om_b200_contract for them).
 * The first call on a device looks up the arrays' device addresses; make
 * that first call before any stream capture.  All calls share the arrays,
 * so calls that overlap on the GPU (other streams, other threads) race:
 * serialise them. */
int om_b200_tropical_matmul_argmax_noalloc(void* stream, om_algebra alg, int64_t m, int64_t n,
                                           int64_t k, const float* a, int64_t lda, const float* b,
                                           int64_t ldb, float* c, int64_t ldc, uint32_t* argmax);

#ifdef __cplusplus
}
#endif
#endif /* OMEINSUM_B200_H */
