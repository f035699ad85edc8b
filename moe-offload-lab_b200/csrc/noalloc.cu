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
//  - The address is cached per device ordinal: the library assumes one context per device (the
//    primary context, as the CUDA runtime and torch use it). A process that creates further contexts
//    on the same device with the driver API must not call this entry point from them.
//  - Every call on a device shares the same array and finds the previous call's contents there. What
//    must start at zero is cleared on the device by the call's own kernels (the item count, the job
//    and split-K arrival counters by the items kernel, the fp32 combine buffer by the gate/up
//    kernel), so sequential calls are independent; calls that overlap on the GPU (different streams,
//    or different host threads without ordering) race on the scratch.
//  - The array starts zeroed when the library is loaded. Its first word is the device status word
//    (0 = OK, 1 = a bounded wait gave up, 2 = a bad index): kernels set it instead of hanging, calls
//    leave it as they find it, and moeb200_noalloc_check_status reads and clears it, so a failure in
//    any call since the last check is reported there.
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

// The scratch array's device address on the current device (looked up once per device, with that
// device current). Returns MOEB200_OK or an error code with the message set.
int scratch_address(const char* who, void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return moeb200::set_error(MOEB200_ERR_CUDA, "%s: cudaGetDevice: %s", who, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return moeb200::set_error(MOEB200_ERR_UNSUPPORTED, "%s: device ordinal %d >= %d", who, dev, kMaxDevices);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return moeb200::set_error(MOEB200_ERR_CUDA, "%s: cudaGetSymbolAddress: %s", who, cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return MOEB200_OK;
}

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
  void* scratch = nullptr;
  const int rc = scratch_address("grouped_ffn_noalloc", &scratch);
  if (rc != MOEB200_OK) return rc;
  return moeb200_grouped_ffn(layout, tab, w, n, x, act_type, out, scratch, kNoAllocScratchBytes, stream);
}

extern "C" int moeb200_noalloc_check_status(int32_t* status, void* stream) {
  if (!status) return moeb200::set_error(MOEB200_ERR_INVALID, "noalloc_check_status: null pointer");
  void* scratch = nullptr;
  const int rc = scratch_address("noalloc_check_status", &scratch);
  if (rc != MOEB200_OK) return rc;
  // the status word is the first field of the scratch's header (as in every workspace)
  return moeb200_check_workspace(scratch, status, stream);
}
