// Diagnostics: the L2 -> SM bulk-copy throughput of the current GPU.
//
// Every tcgen05 kernel of this library gathers one B panel (or X / dY box)
// per nonzero block, mostly from L2, with TMA.  Their ceiling is therefore
// the rate at which the SMs can pull bulk copies out of L2, not the HBM
// bandwidth.  kairo_gather_probe measures that rate: one CTA per SM, two
// issuing warps (a single thread serialises its bulk copies), a ring of six
// 32 KiB stages, each filled by bulk copies of `load_bytes` from
// pseudo-random aligned offsets of a caller buffer (L2-resident when it is
// smaller than the L2).  The caller's stream is synchronised.
#include <cuda_runtime.h>

#include <algorithm>

#include "internal.h"
#include "ptx.cuh"

namespace kairo {
namespace {

constexpr int kProbeStages = 6;
constexpr int kProbeSlot = 32 * 1024;
constexpr int kProbeIssuers = 2;  // issuing warps (lane 0 of warps 0 and 1); warp 2 consumes
constexpr long long kProbeWait = 2000000000LL;

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352dU;
  x ^= x >> 15;
  x *= 0x846ca68bU;
  x ^= x >> 16;
  return x;
}

__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   ptx::smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(ptx::smem_u32(bar))
               : "memory");
}

__global__ void __launch_bounds__(96, 1) k_gather_probe(const uint8_t* __restrict__ buf, uint64_t nloads_in_buf,
                                                        uint32_t load_bytes, int iters, unsigned* err) {
  extern __shared__ uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kProbeStages * kProbeSlot);
  uint64_t* empty = full + kProbeStages;
  int* issued = reinterpret_cast<int*>(empty + kProbeStages);
  int* abort_flag = issued + kProbeStages;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kProbeStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
      issued[s] = 0;
    }
    *abort_flag = 0;
    ptx::mbar_init_fence();
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = kProbeSlot / static_cast<int>(load_bytes);
  volatile int* vabort = abort_flag;
  if (warp < kProbeIssuers && lane == 0) {
    for (int it = 0; it < iters; ++it) {
      const int s = it % kProbeStages;
      if (it >= kProbeStages &&
          !ptx::wait_parity(&empty[s], ((it / kProbeStages) - 1) & 1, vabort, err, 1, kProbeWait))
        break;
      if (warp == 0) {
        ptx::mbar_arrive_expect_tx(&full[s], kProbeSlot);
        issued[s] = it + 1;
      }
      for (int q = warp; q < per; q += kProbeIssuers) {
        const uint32_t h = mix32(blockIdx.x * 7919u + static_cast<uint32_t>(it) * 131u + static_cast<uint32_t>(q));
        bulk_copy(sm + s * kProbeSlot + q * load_bytes, buf + (h % nloads_in_buf) * load_bytes, load_bytes,
                  &full[s]);
      }
    }
  } else if (warp == kProbeIssuers && lane == 0) {
    for (int it = 0; it < iters; ++it) {
      const int s = it % kProbeStages;
      if (!ptx::wait_parity(&full[s], (it / kProbeStages) & 1, vabort, err, 2, kProbeWait)) break;
      ptx::mbar_arrive(&empty[s]);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Every copy issued has landed before the CTA exits.
    int dummy = 0;
    for (int s = 0; s < kProbeStages; ++s)
      if (issued[s])
        ptx::wait_parity(&full[s], ((issued[s] - 1) / kProbeStages) & 1, reinterpret_cast<volatile int*>(&dummy),
                         err, 3, kProbeWait);
  }
}

}  // namespace
}  // namespace kairo

using namespace kairo;

extern "C" kairo_status kairo_gather_probe(const void* buffer, size_t buffer_bytes, uint32_t load_bytes,
                                           int32_t iterations, double* gb_per_s, void* stream) {
  if (!buffer || !gb_per_s) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  if (load_bytes < 16 || load_bytes > static_cast<uint32_t>(kProbeSlot) || load_bytes % 16 != 0 ||
      kProbeSlot % load_bytes != 0)
    return fail(KAIRO_STATUS_INVALID_VALUE, "load_bytes must be a multiple of 16 dividing 32768");
  if (buffer_bytes < load_bytes || reinterpret_cast<uintptr_t>(buffer) % 16 != 0)
    return fail(KAIRO_STATUS_INVALID_VALUE, "buffer too small or not 16-byte aligned");
  if (iterations < 1) return fail(KAIRO_STATUS_INVALID_VALUE, "iterations must be positive");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int dev = current_device();
  const int sms = device_sm_count(dev);
  unsigned* err = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&err), sizeof(unsigned), s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMallocAsync(probe error word)");
  const size_t smem = static_cast<size_t>(kProbeStages) * kProbeSlot + 1024 + 256;
  cudaEvent_t t0 = nullptr, t1 = nullptr;
  e = cudaMemsetAsync(err, 0, sizeof(unsigned), s);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&k_gather_probe),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess) e = cudaEventCreate(&t0);
  if (e == cudaSuccess) e = cudaEventCreate(&t1);
  float ms = 0.f;
  unsigned code = 0;
  if (e == cudaSuccess) {
    const uint64_t nloads = buffer_bytes / load_bytes;
    // One untimed launch, then the timed one.
    for (int rep = 0; rep < 2 && e == cudaSuccess; ++rep) {
      if (rep == 1) e = cudaEventRecord(t0, s);
      if (e == cudaSuccess)
        k_gather_probe<<<sms, 96, smem, s>>>(static_cast<const uint8_t*>(buffer), nloads, load_bytes, iterations,
                                             err);
      if (e == cudaSuccess) e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaEventRecord(t1, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&code, err, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, t0, t1);
  }
  if (t0) cudaEventDestroy(t0);
  if (t1) cudaEventDestroy(t1);
  cudaFreeAsync(err, s);
  if (e != cudaSuccess) return cuda_fail(e, "gather probe");
  if (code) return fail(KAIRO_STATUS_DEVICE_ERROR, "gather probe: a wait timed out");
  const double bytes = static_cast<double>(sms) * iterations * kProbeSlot;
  *gb_per_s = bytes / (static_cast<double>(ms) * 1e-3) / 1e9;
  return KAIRO_STATUS_SUCCESS;
}
