// moeb200_grouped_ffn_noalloc: the single-token grouped expert product (moeb200_grouped_ffn) with
// its scratch in a fixed device array instead of a caller-provided workspace.
//
// Who needs this: some callers have no way to hand the library a workspace. A host that binds the C
// ABI directly (a Go or Java service over cgo/JNI, a plain C program) may have no device allocator of
// its own; code inside a latency-critical decode loop must not call cudaMalloc, which can synchronise
// the whole device; and a process whose GPU memory is already budgeted by another framework's caching
// allocator should not take memory behind its back. For them the scratch is one static device array
// of kNoAllocScratchBytes per GPU, held from the moment this library's code is loaded on that GPU
// until the process exits. Nothing here calls cudaMalloc, cudaFree or any allocating routine.
//
// Rules of use:
//  - The first call on a device looks up the array's device address (cudaGetSymbolAddress) with that
//    device current and caches it; make that first call before any stream capture.
//  - Every call on a device shares the same array and finds the previous call's contents there. The
//    call clears what must start at zero (the status header; the fp32 combine buffer is zeroed by
//    the gate/up kernel), so sequential calls are independent, but calls that overlap on the GPU
//    (different streams, or different host threads without ordering) race on the scratch.
//  - Sizes whose scratch would exceed kNoAllocScratchBytes are refused with
//    MOEB200_ERR_UNSUPPORTED before anything is launched.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/moeb200.h"

namespace moeb200 {
int set_error(int code, const char* fmt, ...);
}

namespace {

constexpr size_t kNoAllocScratchBytes = MOEB200_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// The scratch itself. In host code this name is only a stand-in for the device array: its device
// address comes from cudaGetSymbolAddress below and is what the kernels receive.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {nullptr};

}  // namespace

extern "C" int moeb200_grouped_ffn_noalloc(const moeb200_layout* layout, const int64_t* tab, const float* w,
                                           int32_t n, const void* x, int32_t act_type, void* out, void* stream) {
  if (!layout) return moeb200::set_error(MOEB200_ERR_INVALID, "grouped_ffn_noalloc: null layout");
  const size_t need = moeb200_grouped_ffn_workspace(layout, n);
  if (need > kNoAllocScratchBytes)
    return moeb200::set_error(MOEB200_ERR_UNSUPPORTED,
                              "grouped_ffn_noalloc: this call needs %zu bytes of scratch, more than the fixed "
                              "%zu-byte device array (use moeb200_grouped_ffn with a workspace)",
                              need, kNoAllocScratchBytes);
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return moeb200::set_error(MOEB200_ERR_CUDA, "grouped_ffn_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return moeb200::set_error(MOEB200_ERR_UNSUPPORTED, "grouped_ffn_noalloc: device ordinal %d >= %d", dev, kMaxDevices);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_scratch_addr[dev] == nullptr) {  // once per device, with that device current
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr)
        return moeb200::set_error(MOEB200_ERR_CUDA, "grouped_ffn_noalloc: cudaGetSymbolAddress: %s",
                                  cudaGetErrorString(e));
      g_scratch_addr[dev] = p;
    }
    scratch = g_scratch_addr[dev];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the status header of the scratch must start at zero; the rest is rewritten by each call
  e = cudaMemsetAsync(scratch, 0, 256, s);
  if (e != cudaSuccess) return moeb200::set_error(MOEB200_ERR_CUDA, "grouped_ffn_noalloc: clearing scratch: %s", cudaGetErrorString(e));
  return moeb200_grouped_ffn(layout, tab, w, n, x, act_type, out, scratch, kNoAllocScratchBytes, stream);
}
