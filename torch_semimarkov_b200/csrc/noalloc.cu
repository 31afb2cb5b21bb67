// noalloc.cu -- semicrf_forward_noalloc: the partition-only forward scan with
// its scratch space in a fixed file-scope device array instead of a
// caller-supplied workspace.
//
// Who needs it: hosts that cannot hand the library a device buffer.  A
// foreign-language runtime (JNI, cgo, N-API) that binds the C ABI usually has
// no device allocator of its own, and calling cudaMalloc/cudaFree from its
// request path would both synchronise the device and compete with whatever
// caching allocator already owns the GPU's memory.  Such a caller can still
// run inference (the log-partition or the Viterbi score) with this entry
// point: it allocates nothing at run time.
//
// Limits and rules:
//  - The scratch holds the forward's prepared constants (the exponentiated
//    transition and duration tables, about 16*C*C + 8*(K+16)*C bytes in the
//    log semiring).  It is kNoallocScratchBytes (2 MiB) large.  Every shape
//    with (C, C) transitions fits (the largest, at C=256, need about 1.3 MiB);
//    (K, C, C) transitions need per-duration factor tables, 32*K*C*C + 24*K*C
//    + 8*C bytes (48*K*C*C + 24*K*C + 8*C for max), so only those up to about
//    K*C*C = 65k (43k for max) fit.  A problem whose forward workspace
//    (semicrf_forward_workspace_size) exceeds 2 MiB is rejected with
//    SEMICRF_ERR_WORKSPACE before any CUDA call.
//  - Nothing in the scratch has to start at zero: every byte the scan reads
//    is first written by the preparation kernel of the same call, earlier on
//    the same stream.
//  - There is one scratch per device, shared by every call on that device.
//    Calls that can overlap in time (different streams, or different host
//    threads without ordering between their streams) race on it; the caller
//    must order them.
//  - Every call resolves the scratch's device address with
//    cudaGetSymbolAddress in the CUDA context current on the calling thread
//    (the device's primary context for runtime-API callers, or a driver-API
//    context that a JNI/cgo host made current).  Module addresses belong to a
//    context, so nothing is cached across calls: after cudaDeviceReset, or
//    when the host switches contexts, the address is looked up afresh.  After
//    the first call in a context this is a host-side table lookup.  The first
//    call in a context may load this library's device code into it; make that
//    first call before capturing any stream in that context.

#include "semicrf_internal.cuh"

namespace {

constexpr size_t kNoallocScratchBytes = size_t(2) << 20;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

// Device address of the scratch in the current context.
int noalloc_scratch(void** out) {
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr)
    return SEMICRF_ERR_CUDA;
  *out = ptr;
  return SEMICRF_OK;
}

}  // namespace

extern "C" int semicrf_forward_noalloc(const semicrf_problem* p, float* partition,
                                       void* stream) {
  if (!p) return SEMICRF_ERR_INVALID_ARGUMENT;
  // semicrf_forward checks every argument before it touches the device.  Given
  // no workspace it returns SEMICRF_OK for an empty batch, its validation
  // error for a bad problem, and otherwise stops at the workspace check.
  const int pre = semicrf_forward(p, partition, nullptr, 0, nullptr, nullptr, 0, stream);
  if (pre != SEMICRF_ERR_WORKSPACE) return pre;
  if (semicrf_forward_workspace_size(p) > kNoallocScratchBytes) return SEMICRF_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st != SEMICRF_OK) return st;
  return semicrf_forward(p, partition, nullptr, 0, nullptr, scratch, kNoallocScratchBytes,
                         stream);
}
