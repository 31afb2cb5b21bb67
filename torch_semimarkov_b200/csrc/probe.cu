// probe.cu -- device-rate probes that bench.py uses as roofline denominators.
//
// Built into its own library (libsemicrf_probe.so), apart from the product
// library: these kernels measure the GPU, they compute nothing of the scan.
// They read no GPU setting and change none.
//
//   semicrf_probe_fp64_fma   float64 FMA throughput of the whole device: every
//                            thread runs 8 independent FMA chains, so the FP64
//                            pipe (not latency) bounds it.  The caller times the
//                            launch with CUDA events; FMAs per launch =
//                            grid * 256 * iters * 32 (8 chains, 4 per iteration).
//   semicrf_probe_fp64_latency  cycles per dependent float64 FMA (one warp, one
//                            chain, clock64 around the loop).
//   semicrf_probe_dmma       float64 tensor-core throughput: every warp runs 4
//                            independent chains of mma.sync m8n8k4 f64 (256
//                            FMAs each); FMAs per launch = grid * 8 warps *
//                            iters * 4 * 4 * 256.
//   semicrf_probe_dmma_latency  cycles per dependent m8n8k4 f64 MMA (one warp).

#include <cuda_runtime.h>

#include <cstdint>

namespace {

constexpr int kProbeThreads = 256;

__global__ void __launch_bounds__(kProbeThreads) fp64_fma_kernel(double* out, int iters,
                                                                 double a, double b) {
  double x[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] = 1.0 + 1e-3 * j + 1e-9 * threadIdx.x;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = fma(x[j], a, b);
  }
  double s = 0.0;
#pragma unroll
  for (int j = 0; j < 8; ++j) s += x[j];
  out[(size_t)blockIdx.x * kProbeThreads + threadIdx.x] = s;
}

__global__ void fp64_latency_kernel(long long* cycles, double* out, int iters, double a,
                                    double b) {
  double x = 1.0 + 1e-9 * threadIdx.x;
  const long long t0 = clock64();
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int r = 0; r < 16; ++r) x = fma(x, a, b);
  }
  const long long t1 = clock64();
  out[threadIdx.x] = x;
  if (threadIdx.x == 0) cycles[0] = t1 - t0;
}

// D = A * B + D, m8n8k4, float64 (one A and one B element, two D elements per lane)
__device__ __forceinline__ void dmma(double& d0, double& d1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
               : "+d"(d0), "+d"(d1)
               : "d"(a), "d"(b));
}

__global__ void __launch_bounds__(kProbeThreads) dmma_kernel(double* out, int iters) {
  const double a = 0.999 + 1e-6 * (threadIdx.x & 31), b = 1e-3;
  double d[4][2];
#pragma unroll
  for (int j = 0; j < 4; ++j) d[j][0] = d[j][1] = 1e-3 * j;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) dmma(d[j][0], d[j][1], a, b);
  }
  double s = 0.0;
#pragma unroll
  for (int j = 0; j < 4; ++j) s += d[j][0] + d[j][1];
  out[(size_t)blockIdx.x * kProbeThreads + threadIdx.x] = s;
}

__global__ void dmma_latency_kernel(long long* cycles, double* out, int iters) {
  double d0 = 0.0, d1 = 0.0;
  const double a = 0.5, b = 1e-3;
  const long long t0 = clock64();
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int r = 0; r < 16; ++r) dmma(d0, d1, a, b);
  }
  const long long t1 = clock64();
  out[threadIdx.x] = d0 + d1;
  if (threadIdx.x == 0) cycles[0] = t1 - t0;
}

}  // namespace

extern "C" {

// Threads per block of semicrf_probe_fp64_fma.
int semicrf_probe_threads(void) { return kProbeThreads; }

// grid blocks of 256 threads; each thread runs 32 * iters FMAs (8 chains, 4
// per iteration).  out: grid * 256 doubles (device).
int semicrf_probe_fp64_fma(int grid, int iters, double* out, void* stream) {
  if (grid < 1 || iters < 1 || !out) return 1;
  fp64_fma_kernel<<<grid, kProbeThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      out, iters, 0.9999999, 1e-7);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

// One warp, a chain of 16*iters dependent FMAs; cycles[0] = elapsed clock64
// cycles (device), out: 32 doubles (device).
int semicrf_probe_fp64_latency(int iters, long long* cycles, double* out, void* stream) {
  if (iters < 1 || !cycles || !out) return 1;
  fp64_latency_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(cycles, out, iters,
                                                                       0.9999999, 1e-7);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

// grid blocks of 256 threads (8 warps); each warp runs 16 * iters m8n8k4 f64
// MMAs (4 chains, 4 per iteration), 256 FMAs each.  out: grid * 256 doubles.
int semicrf_probe_dmma(int grid, int iters, double* out, void* stream) {
  if (grid < 1 || iters < 1 || !out) return 1;
  dmma_kernel<<<grid, kProbeThreads, 0, static_cast<cudaStream_t>(stream)>>>(out, iters);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

// One warp, a chain of 16*iters dependent m8n8k4 f64 MMAs; cycles[0] = clock64
// cycles, out: 32 doubles (device).
int semicrf_probe_dmma_latency(int iters, long long* cycles, double* out, void* stream) {
  if (iters < 1 || !cycles || !out) return 1;
  dmma_latency_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(cycles, out, iters);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

}  // extern "C"
