// Backend object, errors, stream-ordered device memory and host transfers.
//
// Replaces the reference's cudarc-based `Cuda` device handle
// (tensor4all/omeinsum-rs src/backend/cuda/mod.rs:214-265, storage.rs):
// one non-blocking stream per backend instead of the null stream, and device
// memory from the CUDA stream-ordered pool (cudaMallocAsync) with an unbounded
// release threshold, so freed blocks are cached and reused without a device
// synchronisation -- the device-side counterpart of the CPU ScratchPool
// (src/backend/cpu/buffer_pool.rs:2-47).
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
  if (ptr && be) cudaFreeAsync(ptr, be->stream);
}

int Scratch::alloc(om_backend* b, size_t bytes) {
  be = b;
  if (bytes == 0) bytes = 16;
  OM_CUDA(cudaMallocAsync(&ptr, bytes, b->stream), "scratch cudaMallocAsync");
  return OM_OK;
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
  *out = be;
  return OM_OK;
}

int om_b200_destroy(om_backend* be) {
  if (!be) return OM_OK;
  cudaSetDevice(be->device);
  resolve_pending(be);
  cudaFree(be->d_flags);
  cudaStreamDestroy(be->stream);
  delete be;
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
};

extern "C" int om_b200_graph_begin(om_backend* be) {
  using namespace om;
  if (!be) return set_error(OM_ERR_INVALID, "om_b200_graph_begin: null backend");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  // relaxed: the library may query or set function attributes while recording
  OM_CUDA(cudaStreamBeginCapture(be->stream, cudaStreamCaptureModeRelaxed), "cudaStreamBeginCapture");
  return OM_OK;
}

extern "C" int om_b200_graph_end(om_backend* be, om_graph** graph_out) {
  using namespace om;
  if (!be || !graph_out) return set_error(OM_ERR_INVALID, "om_b200_graph_end: null argument");
  OM_CUDA(cudaSetDevice(be->device), "cudaSetDevice");
  cudaGraph_t g = nullptr;
  OM_CUDA(cudaStreamEndCapture(be->stream, &g), "cudaStreamEndCapture");
  cudaGraphExec_t x = nullptr;
  cudaError_t e = cudaGraphInstantiateWithFlags(&x, g, cudaGraphInstantiateFlagAutoFreeOnLaunch);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    return check_cuda(e, "cudaGraphInstantiate");
  }
  *graph_out = new om_graph{g, x};
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
  delete graph;
  return OM_OK;
}
