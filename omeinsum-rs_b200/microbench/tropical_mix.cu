// Instruction-mix micro-benchmark behind the tropical GEMM's design: the
// throughput of (add, max) instruction pairs on one B200, register-only.
// Build and run:  make -C omeinsum-rs_b200 microbench && omeinsum-rs_b200/build/tropical_mix
#include <cstdio>
#include <cuda_runtime.h>
typedef unsigned long long u64;
__device__ __forceinline__ u64 padd(u64 a, u64 b) {
  u64 d;
  asm volatile("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm volatile("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float max2f(float a, float b) {
  float d;
  asm volatile("max.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ float addf(float a, float b) {
  float d;
  asm volatile("add.rn.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
// 16 independent chains of each of the two instructions per iteration
template <int MODE>
__global__ void mix(float* out, int iters, float seed) {
  float s[16], m[16];
  u64 s2[16];
  for (int i = 0; i < 16; i++) {
    s[i] = seed * i + threadIdx.x;
    m[i] = seed - i;
    s2[i] = ((u64)__float_as_uint(s[i]) << 32) | __float_as_uint(m[i]);
  }
  const float c1 = 1.0001f, c2 = 0.9999f;
  const u64 cc = ((u64)__float_as_uint(c1) << 32) | __float_as_uint(c2);
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 16; i++) {
      if (MODE == 0) { s[i] = addf(s[i], c1); m[i] = max2f(m[i], c2); }
      if (MODE == 1) { s2[i] = padd(s2[i], cc); m[i] = max2f(m[i], c2); }
      if (MODE == 2) { s[i] = addf(s[i], c1); m[i] = max3f(m[i], c2, c1); }
      if (MODE == 3) { s2[i] = padd(s2[i], cc); m[i] = max3f(m[i], c2, c1); }
      if (MODE == 4) { s[i] = addf(s[i], c1); m[i] = addf(m[i], c2); }
      if (MODE == 5) { s[i] = max2f(s[i], c1); m[i] = max2f(m[i], c2); }
    }
  }
  float r = 0;
  for (int i = 0; i < 16; i++) r += s[i] + m[i] + __uint_as_float((unsigned)s2[i]);
  out[blockIdx.x * blockDim.x + threadIdx.x] = r;
}
template <int MODE>
void run(float* out, int sms, int iters, const char* what) {
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  float ms = 0;
  for (int rep = 0; rep < 2; ++rep) {
    cudaEventRecord(e0);
    mix<MODE><<<sms * 4, 256>>>(out, iters, 1.5f);
    cudaEventRecord(e1);
    cudaEventSynchronize(e1);
    cudaEventElapsedTime(&ms, e0, e1);
  }
  int clk_khz = 0;
  cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, 0);
  const double pairs = (double)sms * 4 * 256 * iters * 16;
  printf("%-16s %8.3f ms  %6.1f pairs/clk/SM (at %.0f MHz)\n", what, ms,
         pairs / (ms * 1e-3) / sms / (clk_khz * 1e3), clk_khz / 1e3);
}
int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  float* out;
  cudaMalloc(&out, (size_t)sms * 4 * 256 * sizeof(float));
  const int it = 8192;
  run<0>(out, sms, it, "FADD + FMNMX");
  run<1>(out, sms, it, "FADD2 + FMNMX");
  run<2>(out, sms, it, "FADD + max3");
  run<3>(out, sms, it, "FADD2 + max3");
  run<4>(out, sms, it, "FADD + FADD");
  run<5>(out, sms, it, "FMNMX + FMNMX");
  printf("status: %s\n", cudaGetErrorString(cudaGetLastError()));
  cudaFree(out);
  return 0;
}
