// Backend object, errors, stream-ordered device memory and host transfers.
//
// Replaces the reference's cudarc-based `Cuda` device handle
// (tensor4all/omeinsum-rs src/backend/cuda/mod.rs:214-265, storage.rs):
// one non-blocking stream per backend instead of the null stream, and device
// memory from the CUDA stream-ordered pool (cudaMallocAsync) with an unbounded
// release threshold, so freed blocks are cached and reused without a device
// synchronisation -- the device-side counterpart of the CPU ScratchPool
// (src/backend/cpu/buffer_pool.rs:2-47).
#include <map>
#include <mutex>
#include <set>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <string>

#include "om_internal.h"

namespace om {

static thread_local std::string g_last_error;
static thread_local int64_t g_launches = 0;

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return OM_OK;
  int code = (e == cudaErrorMemoryAllocation) ? OM_ERR_OOM : OM_ERR_CUDA;
  return set_error(code, std::string(what) + ": " + cudaGetErrorString(e));
}

void note_launch(int n) { g_launches += n; }

bool trace_on() {
  static const bool on = [] {
    const char* v = std::getenv("OM_B200_TRACE");
    return v && v[0] && v[0] != '0';
  }();
  return on;
}

ProfScope::ProfScope(om_backend* b, const char* name) : be(b) {
  if (!be || !be->profiling) return;
  p.name = name;
  if (cudaEventCreate(&p.start) != cudaSuccess || cudaEventCreate(&p.stop) != cudaSuccess) {
    p.name = nullptr;
    return;
  }
  cudaEventRecord(p.start, be->stream);
}

ProfScope::~ProfScope() {
  if (!be || !be->profiling || !p.name) return;
  cudaEventRecord(p.stop, be->stream);
  be->pending.push_back(p);
}

static void resolve_pending(om_backend* be) {
  cudaStreamSynchronize(be->stream);
  for (auto& q : be->pending) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, q.start, q.stop);
    cudaEventDestroy(q.start);
    cudaEventDestroy(q.stop);
    bool found = false;
    for (auto& t : be->prof_totals)
      if (t.first == q.name) {
        t.second.first += ms;
        t.second.second += 1;
        found = true;
      }
    if (!found) be->prof_totals.push_back({q.name, {(double)ms, 1}});
  }
  be->pending.clear();
}

Scratch::~Scratch() {
  if (ptr && be) be_free(be, be_id, ptr);
}

int Scratch::alloc(om_backend* b, size_t bytes) {
  be = b;
  be_id = b->id;
  if (bytes == 0) bytes = 16;
  return be_alloc(b, bytes, &ptr);
}

// ---- arenas ------------------------------------------------------------------
// Registries of live arenas and backends.  Never destroyed: buffers (a
// tape's, a graph's) can be released during process teardown, after static
// destructors would have run.
static std::mutex& g_arena_mu = *new std::mutex;
static std::set<Arena*>& g_arenas = *new std::set<Arena*>;
static std::map<const om_backend*, uint64_t>& g_live = *new std::map<const om_backend*, uint64_t>;
static uint64_t g_next_backend_id = 1;

static void backend_live(om_backend* be, bool on) {
  std::lock_guard<std::mutex> lk(g_arena_mu);
  if (on) g_live[be] = be->id = g_next_backend_id++;
  else g_live.erase(be);
}

void arena_register(Arena* a) {
  std::lock_guard<std::mutex> lk(g_arena_mu);
  g_arenas.insert(a);
}
void arena_unregister(Arena* a) {
  std::lock_guard<std::mutex> lk(g_arena_mu);
  g_arenas.erase(a);
}

bool Arena::owns(const void* p) const {
  for (auto& c : chunks)
    if ((const char*)p >= c.first && (const char*)p < c.first + c.second) return true;
  return false;
}

int Arena::alloc(size_t bytes, void** out) {
  bytes = (bytes + 255) & ~size_t(255);
  for (auto it = free_blocks.begin(); it != free_blocks.end(); ++it) {
    if (it->second < bytes) continue;
    char* p = it->first;
    const size_t rest = it->second - bytes;
    free_blocks.erase(it);
    if (rest) free_blocks[p + bytes] = rest;
    used[p] = bytes;
    *out = p;
    return OM_OK;
  }
  // grow: a new chunk of at least 64 MiB (plain cudaMalloc is allowed while
  // recording; it is not stream work)
  const size_t sz = std::max(bytes, size_t(64) << 20);
  void* c = nullptr;
  OM_CUDA(cudaMalloc(&c, sz), "arena cudaMalloc");
  chunks.push_back({(char*)c, sz});
  if (sz > bytes) free_blocks[(char*)c + bytes] = sz - bytes;
  used[(char*)c] = bytes;
  *out = c;
  return OM_OK;
}

void Arena::release(void* p) {
  if (defer) {
    deferred.push_back(p);
    return;
  }
  auto it = used.find((char*)p);
  if (it == used.end()) return;
  char* a = it->first;
  size_t n = it->second;
  used.erase(it);
  char *lo = nullptr, *hi = nullptr;  // the chunk holding the block
  for (auto& c : chunks)
    if (a >= c.first && a < c.first + c.second) {
      lo = c.first;
      hi = c.first + c.second;
    }
  auto nx = free_blocks.lower_bound(a);
  if (nx != free_blocks.end() && nx->first == a + n && nx->first < hi) {
    n += nx->second;
    free_blocks.erase(nx);
  }
  auto pv = free_blocks.lower_bound(a);
  if (pv != free_blocks.begin()) {
    --pv;
    if (pv->first >= lo && pv->first + pv->second == a) {
      pv->second += n;
      return;
    }
  }
  free_blocks[a] = n;
}

void Arena::destroy() {
  for (auto& c : chunks) cudaFree(c.first);
  chunks.clear();
  free_blocks.clear();
  used.clear();
}

int be_alloc(om_backend* be, size_t bytes, void** out) {
  if (bytes == 0) bytes = 16;
  if (be->recording) return be->recording->alloc(bytes, out);
  OM_CUDA(cudaMallocAsync(out, bytes, be->stream), "cudaMallocAsync");
  return OM_OK;
}

void be_free(om_backend* be, uint64_t id, void* p) {
  if (!p) return;
  {
    std::lock_guard<std::mutex> lk(g_arena_mu);
    for (Arena* a : g_arenas)
      if (a->owns(p)) {
        a->release(p);
        return;
      }
    // a buffer that outlives its backend (a tape freed after
    // om_b200_destroy) goes back with the device's pool at teardown
    auto it = g_live.find(be);
    if (it == g_live.end() || it->second != id) return;
  }
  cudaFreeAsync(p, be->stream);
}

}  // namespace om

using namespace om;

extern "C" {

const char* om_b200_name(void) { return "b200"; }

int om_b200_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return OM_ERR_INVALID;
  std::snprintf(buf, len, "%s", g_last_error.c_str());
  return OM_OK;
}

int64_t om_b200_launch_count(void) {
  int64_t n = g_launches;
  g_launches = 0;
  return n;
}

int om_b200_create(int device, om_backend** out) {
  if (!out) return set_error(OM_ERR_INVALID, "om_b200_create: out is null");
  *out = nullptr;
  int count = 0;
  OM_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (device < 0 || device >= count)
    return set_error(OM_ERR_INVALID, "om_b200_create: device ordinal " + std::to_string(device) +
                                         " out of range (" + std::to_string(count) + " devices)");
  OM_CUDA(cudaSetDevice(device), "cudaSetDevice");
  cudaDeviceProp prop;
  OM_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major < 10)
    return set_error(OM_ERR_UNSUPPORTED, std::string("om_b200_create: device '") + prop.name +
                                             "' is not sm_100 class; this library is built for sm_100a");
  auto* be = new om_backend();
  be->device = device;
  be->num_sms = prop.multiProcessorCount;
  cudaError_t e = cudaStreamCreateWithFlags(&be->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete be;
    return check_cuda(e, "cudaStreamCreateWithFlags");
  }
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  e = cudaMalloc(&be->d_flags, 64);
  if (e == cudaSuccess) e = cudaMemset(be->d_flags, 0, 64);
  if (e != cudaSuccess) {
    cudaStreamDestroy(be->stream);
    delete be;
    return check_cuda(e, "cudaMalloc(flags)");
  }
  be->f32_exact = std::getenv("OM_DISABLE_TCGEN05") != nullptr;
  backend_live(be, true);
  *out = be;
  return OM_OK;
}

int om_b200_destroy(om_backend* be) {
  if (!be) return OM_OK;
  backend_live(be, false);
  cudaSetDevice(be->device);
  resolve_pending(be);
  cudaFree(be->d_flags);
  be->d_flags = nullptr;
  for (cudaStream_t st : be->branch_streams) cudaStreamDestroy(st);
  be->branch_streams.clear();
  if (be->fork_event) cudaEventDestroy(be->fork_event);
  be->fork_event = nullptr;
  cudaStreamDestroy(be->stream);
  be->stream = nullptr;
  be->pending.clear();
  be->prof_totals.clear();
  // The control block itself is kept (a few hundred bytes per destroyed
  // backend): buffers released after om_b200_destroy are recognised by this
  // address, and a later om_b200_create must never reuse it.
  return OM_OK;
}

int om_b200_set_f32_mode(om_backend* be, om_f32_mode mode) {
  if (!be) return set_error(OM_ERR_INVALID, "om_b200_set_f32_mode: null backend");
  if (mode != OM_F32_TENSOR_3XTF32 && mode != OM_F32_EXACT)
    return set_error(OM_ERR_INVALID, "om_b200_set_f32_mode: unknown mode");
  be->f32_exact = mode == OM_F32_EXACT;
  return OM_OK;
}

int om_b200_profile_enable(om_backend* be, int on) {
  if (!be) return set_error(OM_ERR_INVALID, "om_b200_profile_enable: null backend");
  resolve_pending(be);
  be->prof_totals.clear();
  be->profiling = on != 0;
  return OM_OK;
}

int om_b200_profile_query(om_backend* be, int index, char* name, size_t len, double* total_ms,
                          int64_t* launches) {
  if (!be) return set_error(OM_ERR_INVALID, "om_b200_profile_query: null backend");
  resolve_pending(be);
  if (index < 0 || index >= (int)be->prof_totals.size())
    return set_error(OM_ERR_INVALID, "om_b200_profile_query: index past the last kernel class");
  const auto& t = be->prof_totals[index];
  if (name && len) std::snprintf(name, len, "%s", t.first.c_str());
  if (total_ms) *total_ms = t.second.first;
  if (launches) *launches = t.second.second;
  return OM_OK;
}

int om_b200_stream(om_backend* be, void** stream_out) {
  if (!be || !stream_out) return set_error(OM_ERR_INVALID, "om_b200_stream: null argument");
  *stream_out = (void*)be->stream;
  return OM_OK;
}

int om_b200_sync(om_backend* be) {
  if (!be) return set_error(OM_ERR_INVALID, "om_b200_sync: null backend");
  OM_CUDA(cudaStreamSynchronize(be->stream), "cudaStreamSynchronize");
  // error word of kernels with bounded waits (flags[1]): non-zero means a
  // wait ran out and that kernel's output is not valid
  uint32_t err = 0;
  OM_CUDA(cudaMemcpy(&err, be->d_flags + 1, sizeof(err), cudaMemcpyDeviceToHost), "error word");
  if (err) {
    cudaMemset(be->d_flags + 1, 0, sizeof(err));
    return set_error(OM_ERR_TIMEOUT, "a device wait ran out (tensor-core GEMM); results invalid");
  }
  return OM_OK;
}

int om_b200_alloc(om_backend* be, size_t bytes, void** dptr) {
  if (!be || !dptr) return set_error(OM_ERR_INVALID, "om_b200_alloc: null argument");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  size_t n = bytes ? bytes : 16;
  OM_CUDA(cudaMallocAsync(dptr, n, be->stream), "cudaMallocAsync");
  OM_CUDA(cudaMemsetAsync(*dptr, 0, n, be->stream), "cudaMemsetAsync");
  return OM_OK;
}

int om_b200_free(om_backend* be, void* dptr) {
  if (!be) return set_error(OM_ERR_INVALID, "om_b200_free: null backend");
  if (!dptr) return OM_OK;
  OM_CUDA(cudaFreeAsync(dptr, be->stream), "cudaFreeAsync");
  return OM_OK;
}

int om_b200_upload(om_backend* be, void* dst, const void* src, size_t bytes) {
  if (!be || (!dst && bytes) || (!src && bytes))
    return set_error(OM_ERR_INVALID, "om_b200_upload: null argument");
  if (!bytes) return OM_OK;
  OM_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, be->stream), "upload");
  return OM_OK;
}

int om_b200_download_async(om_backend* be, void* dst, const void* src, size_t bytes) {
  if (!be || (!dst && bytes) || (!src && bytes))
    return set_error(OM_ERR_INVALID, "om_b200_download_async: null argument");
  if (!bytes) return OM_OK;
  OM_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, be->stream), "download");
  return OM_OK;
}

int om_b200_download(om_backend* be, void* dst, const void* src, size_t bytes) {
  if (!be || (!dst && bytes) || (!src && bytes))
    return set_error(OM_ERR_INVALID, "om_b200_download: null argument");
  if (!bytes) return OM_OK;
  OM_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, be->stream), "download");
  OM_CUDA(cudaStreamSynchronize(be->stream), "download sync");
  return OM_OK;
}

}  // extern "C"

struct om_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  om::Arena* arena = nullptr;  // the recorded work's buffers
  int device = 0;
};

extern "C" int om_b200_graph_begin(om_backend* be) {
  using namespace om;
  if (!be) return set_error(OM_ERR_INVALID, "om_b200_graph_begin: null backend");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  if (be->recording) return set_error(OM_ERR_INVALID, "om_b200_graph_begin: already recording");
  // relaxed: the library may set function attributes or grow its arena
  // (cudaMalloc) while recording
  OM_CUDA(cudaStreamBeginCapture(be->stream, cudaStreamCaptureModeRelaxed), "cudaStreamBeginCapture");
  be->recording = new Arena();
  arena_register(be->recording);
  return OM_OK;
}

extern "C" int om_b200_graph_branch(om_backend* be, int branch) {
  using namespace om;
  if (!be) return set_error(OM_ERR_INVALID, "om_b200_graph_branch: null backend");
  if (!be->recording) return set_error(OM_ERR_INVALID, "om_b200_graph_branch: not recording");
  if (branch < -1 || branch >= 64) return set_error(OM_ERR_INVALID, "om_b200_graph_branch: branch out of range");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  if (!be->branching) {
    // fork point: everything recorded so far on the backend's stream
    be->main_stream = be->stream;
    if (!be->fork_event)
      OM_CUDA(cudaEventCreateWithFlags(&be->fork_event, cudaEventDisableTiming), "fork event");
    OM_CUDA(cudaEventRecord(be->fork_event, be->main_stream), "fork record");
    be->branching = true;
    be->branch_joined.assign(be->branch_streams.size(), 0);
    be->recording->defer = true;
  }
  if (branch < 0) {
    be->stream = be->main_stream;
    return OM_OK;
  }
  while ((int)be->branch_streams.size() <= branch) {
    cudaStream_t st;
    OM_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "branch stream");
    be->branch_streams.push_back(st);
    be->branch_joined.push_back(0);
  }
  cudaStream_t st = be->branch_streams[branch];
  if (!be->branch_joined[branch]) {
    OM_CUDA(cudaStreamWaitEvent(st, be->fork_event, 0), "fork wait");
    be->branch_joined[branch] = 1;
  }
  be->stream = st;
  return OM_OK;
}

// joins every branch forked into the recording back into the backend's
// stream and releases the blocks their work freed
static int join_branches(om_backend* be) {
  using namespace om;
  if (!be->branching) return OM_OK;
  be->stream = be->main_stream;
  int rc = OM_OK;
  for (size_t b = 0; b < be->branch_streams.size(); ++b) {
    if (!be->branch_joined[b]) continue;
    cudaEvent_t ev;
    cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(ev, be->branch_streams[b]);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(be->main_stream, ev, 0);
    if (e != cudaSuccess && rc == OM_OK) rc = check_cuda(e, "branch join");
    cudaEventDestroy(ev);
  }
  be->branching = false;
  Arena* a = be->recording;
  a->defer = false;
  for (void* p : a->deferred) a->release(p);
  a->deferred.clear();
  return rc;
}

extern "C" int om_b200_graph_end(om_backend* be, om_graph** graph_out) {
  using namespace om;
  if (!be || !graph_out) return set_error(OM_ERR_INVALID, "om_b200_graph_end: null argument");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  if (be->recording) {
    const int jr = join_branches(be);
    if (jr != OM_OK) return jr;
  }
  Arena* arena = be->recording;
  be->recording = nullptr;
  auto drop_arena = [&] {
    if (arena) {
      arena_unregister(arena);
      arena->destroy();
      delete arena;
    }
  };
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(be->stream, &g);
  if (e != cudaSuccess) {
    drop_arena();
    return check_cuda(e, "cudaStreamEndCapture");
  }
  cudaGraphExec_t x = nullptr;
  e = cudaGraphInstantiateWithFlags(&x, g, cudaGraphInstantiateFlagAutoFreeOnLaunch);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    drop_arena();
    return check_cuda(e, "cudaGraphInstantiate");
  }
  *graph_out = new om_graph{g, x, arena, be->device};
  return OM_OK;
}

extern "C" int om_b200_graph_launch(om_backend* be, om_graph* graph) {
  using namespace om;
  if (!be || !graph) return set_error(OM_ERR_INVALID, "om_b200_graph_launch: null argument");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  OM_CUDA(cudaGraphLaunch(graph->exec, be->stream), "cudaGraphLaunch");
  return OM_OK;
}

extern "C" int om_b200_graph_free(om_graph* graph) {
  if (!graph) return OM_OK;
  if (graph->exec) cudaGraphExecDestroy(graph->exec);
  if (graph->graph) cudaGraphDestroy(graph->graph);
  if (graph->arena) {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(graph->device);
    cudaDeviceSynchronize();  // a replay may still use the buffers
    om::arena_unregister(graph->arena);
    graph->arena->destroy();
    delete graph->arena;
    if (prev >= 0) cudaSetDevice(prev);  // the caller's current device
  }
  delete graph;
  return OM_OK;
}
