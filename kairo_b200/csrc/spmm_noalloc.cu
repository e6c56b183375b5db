// kairo_bsr_spmm_noalloc: the BSR SpMM without a caller workspace.
//
// Some callers cannot allocate device memory at the point where they need
// the product:
// - a host framework that owns all GPU memory through its own pool and does
//   not let plugins call cudaMalloc;
// - a code path that must not stall the device, since cudaMalloc and cudaFree
//   may synchronize;
// - a stateless C callback that has nowhere to keep a workspace alive between
//   calls.
// This entry point serves them.  It runs exactly the launch of kairo_bsr_spmm,
// with its scratch (error word, split-row counters, partial tiles) taken from
// a fixed array compiled into this library.  Every GPU that loads the library
// keeps the array (kNoAllocScratchBytes) until the process exits.
//
// The array is one per device and shared by every call on that device.  It
// keeps whatever the previous call left there.  Each call therefore clears
// the part that must start at zero (error word and counter banks) on its own
// stream before the kernel.  Calls whose launches overlap on the GPU (e.g.
// two streams at once) would race on the array: callers must order them.
// The device error word of the last call stays in the array until the next
// call clears it; kairo_noalloc_error reads it.
//
// Set-up: host code cannot use the array's name as a device address.  So
// the first call on each device looks the address up with
// cudaGetSymbolAddress, with that device current, and caches it together
// with the CUDA context that was current.  A later call under another
// context (a non-primary driver context, or the primary context re-created
// after cudaDeviceReset under a new handle) looks the address up again.
// Make the first call on a device before any stream capture.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <sstream>

#include "internal.h"

namespace kairo {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB per device

static __device__ __align__(256) unsigned char g_spmm_scratch[kNoAllocScratchBytes];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// cuCtxGetCurrent, resolved once through the runtime's driver entry-point
// query (the library links against the CUDA runtime only).
CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

// Device address of g_spmm_scratch on `device` under the current context
// (looked up once per device and context).
kairo_status scratch_address(int device, void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  static CUcontext owner[64] = {nullptr};
  if (device < 0 || device >= 64) return fail(KAIRO_STATUS_NOT_SUPPORTED, "device index out of range");
  CtxGetCurrentFn get = ctx_get_current_fn();
  if (!get) return fail(KAIRO_STATUS_CUDA_ERROR, "cuCtxGetCurrent is not available from the driver");
  CUcontext ctx = nullptr;
  if (get(&ctx) != CUDA_SUCCESS) return fail(KAIRO_STATUS_CUDA_ERROR, "cuCtxGetCurrent failed");
  if (!ctx) {
    // No context bound to this thread yet: cudaSetDevice makes the
    // device's primary context current (CUDA 12 and later).
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    if (get(&ctx) != CUDA_SUCCESS || !ctx) return fail(KAIRO_STATUS_CUDA_ERROR, "no current CUDA context");
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[device] || owner[device] != ctx) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_spmm_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(scratch)");
    if (!p) return fail(KAIRO_STATUS_CUDA_ERROR, "cudaGetSymbolAddress returned a null scratch address");
    addr[device] = p;
    owner[device] = ctx;
  }
  *out = addr[device];
  return KAIRO_STATUS_SUCCESS;
}

kairo_status current_scratch(void** out) {
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  return scratch_address(device, out);
}

}  // namespace
}  // namespace kairo

using namespace kairo;

extern "C" kairo_status kairo_bsr_spmm_noalloc(const kairo_bsr* a, const void* b, int64_t ldb, int32_t layout,
                                               int64_t n, void* c, int64_t ldc, kairo_dtype c_dtype,
                                               const kairo_spmm_config* cfg, void* stream) {
  if (!a) return fail(KAIRO_STATUS_INVALID_VALUE, "null BSR descriptor");
  size_t need = 0;
  kairo_status st = kairo_bsr_spmm_workspace_size(a, layout, n, cfg, &need);
  if (st) return st;
  if (need > kNoAllocScratchBytes) {
    std::ostringstream os;
    os << "this problem needs " << need << " bytes of scratch; kairo_bsr_spmm_noalloc has "
       << kNoAllocScratchBytes << " (use kairo_bsr_spmm with a caller workspace)";
    return fail(KAIRO_STATUS_NOT_SUPPORTED, os.str());
  }
  void* scratch = nullptr;
  st = current_scratch(&scratch);
  if (st) return st;
  // Error word and both counter banks start at zero for every call.
  const size_t clear = kWorkspaceHeaderBytes + kCounterRegionBytes;
  cudaError_t e = cudaMemsetAsync(scratch, 0, clear, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(scratch header)");
  return kairo_bsr_spmm(a, b, ldb, layout, n, c, ldc, c_dtype, cfg, scratch, kNoAllocScratchBytes, stream);
}

extern "C" kairo_status kairo_noalloc_error(int32_t clear, uint32_t* code, void* stream) {
  if (!code) return fail(KAIRO_STATUS_INVALID_VALUE, "null code");
  void* scratch = nullptr;
  kairo_status st = current_scratch(&scratch);
  if (st) return st;
  return kairo_workspace_error(scratch, clear, code, stream);
}
