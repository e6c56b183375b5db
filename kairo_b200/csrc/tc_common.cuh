// Device helpers shared by the tcgen05 SpMM kernels (row-split and band
// schedules): CTA shape, wait bounds, and the epilogue's stores of TMEM
// results into C (STANDARD layout) or Y (LINEAR layout).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "../../include/kairo_spmm.h"

namespace kairo {

constexpr int kThreads = 192;                    // warp 0 producer, warp 1 MMA, warps 2..5 epilogue
constexpr long long kWaitCycles = 8000000000LL;  // per-wait bound in SM cycles (about 4 s at 2 GHz)
constexpr int kMaxSmem = 227 * 1024;

// Wait-site tags recorded with a timeout (bits 8..15 of the error word),
// the KAIRO_WAIT_SITE_* values of the C ABI.
enum : uint32_t {
  kTagEmpty = KAIRO_WAIT_SITE_EMPTY,
  kTagFull = KAIRO_WAIT_SITE_FULL,
  kTagTmemEmpty = KAIRO_WAIT_SITE_TMEM_EMPTY,
  kTagTmemFull = KAIRO_WAIT_SITE_TMEM_FULL,
  kTagDrain = KAIRO_WAIT_SITE_DRAIN
};

// Wait bound of a launch: the config's wait_kcycles (thousands of cycles)
// or the default.
inline long long wait_bound_cycles(const kairo_spmm_config* cfg) {
  return (cfg && cfg->wait_kcycles > 0) ? static_cast<long long>(cfg->wait_kcycles) * 1000LL : kWaitCycles;
}

// Bytes of one pipeline slot: the B panel (NT sub-tiles of 128 x bk) and the
// block (bm x bk; rg blocks side by side for row groups), padded to 1 KiB for
// the swizzle atom.
constexpr int stage_bytes(int bm, int bk, int nt, int rg = 1) {
  return nt * 128 * bk * 2 + (rg * bm * bk * 2 + 1023) / 1024 * 1024;
}

// Bytes of one stage of `group` blocks of the row-split tcgen05 kernel:
// `group` slots of one B panel and rg blocks (stage_bytes each), or, packed
// (rg = 1), the group's panels and then its blocks side by side, rounded up
// to 1 KiB.
__host__ __device__ constexpr int tc_stage_bytes(int bm, int bk, int nt, int rg, int group, bool packed) {
  return packed ? (group * (nt * 128 * bk * 2 + bm * bk * 2) + 1023) / 1024 * 1024
                : group * (nt * 128 * bk * 2 + (rg * bm * bk * 2 + 1023) / 1024 * 1024);
}

template <typename TOut>
__device__ __forceinline__ void store_scalar(TOut* p, float v);
template <>
__device__ __forceinline__ void store_scalar<float>(float* p, float v) { __stcs(p, v); }
template <>
__device__ __forceinline__ void store_scalar<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ void store_scalar<__half>(__half* p, float v) { *p = __float2half_rn(v); }

// Writes 16 accumulator values of one epilogue thread: rows j0..j0+15 of
// block-row i, at column `col` of C (STANDARD) or row `col` of Y (LINEAR).
// `Args` supplies c, ldc, m, n and vec_store.
template <bool LINEAR, typename TOut, class Args>
__device__ __forceinline__ void store16(const Args& a, int i, int bm, int j0, int col, const float* v) {
  if (col >= a.n) return;
  const int row0 = i * bm + j0;
  if (!LINEAR) {
    float* c = static_cast<float*>(a.c);
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
      const int r = row0 + jj;
      if (r < a.m) __stcs(c + static_cast<int64_t>(r) * a.ldc + col, v[jj]);
    }
  } else {
    TOut* y = static_cast<TOut*>(a.c) + static_cast<int64_t>(col) * a.ldc + row0;
    if (a.vec_store && row0 + 16 <= a.m) {
      if constexpr (sizeof(TOut) == 4) {
        float4* y4 = reinterpret_cast<float4*>(y);
#pragma unroll
        for (int q = 0; q < 4; ++q) y4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      } else {
        uint32_t w[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          TOut lo, hi;
          store_scalar<TOut>(&lo, v[2 * q]);
          store_scalar<TOut>(&hi, v[2 * q + 1]);
          w[q] = static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&lo)) |
                 (static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&hi)) << 16);
        }
        uint4* y4 = reinterpret_cast<uint4*>(y);
        y4[0] = make_uint4(w[0], w[1], w[2], w[3]);
        y4[1] = make_uint4(w[4], w[5], w[6], w[7]);
      }
    } else {
#pragma unroll
      for (int jj = 0; jj < 16; ++jj)
        if (row0 + jj < a.m) store_scalar<TOut>(y + jj, v[jj]);
    }
  }
}

// Block indices (column, stored block) of BSR positions for the producer
// warp, held in registers ahead of use.  Three 32-position windows: lane l
// of window w holds position base + 32*w + l.  A batch of up to 32 positions
// starting at pb (base <= pb < base + 32) is served from windows 0 and 1;
// window 2 is in flight.  Positions are consumed in increasing order, and
// once a batch starts past window 0 the windows shift and the loads of the
// next window are issued, so every index load has a whole window of blocks
// to land before it is read.  A jump backwards or by more than a window
// reloads all three (one wait).
struct IndexWindow {
  int64_t base = -(int64_t(1) << 40);
  int c0 = 0, b0 = 0, c1 = 0, b1 = 0, c2 = 0, b2 = 0;

  __device__ __forceinline__ static void fetch(const int32_t* __restrict__ col_idx,
                                               const int32_t* __restrict__ blk_idx, int64_t nnzb, int64_t p,
                                               int& c, int& b) {
    if (p < nnzb) {
      c = __ldg(col_idx + p);
      b = blk_idx ? __ldg(blk_idx + p) : static_cast<int>(p);
    } else {
      c = 0;
      b = 0;
    }
  }

  // Makes positions [pb, pb + 32) available.
  __device__ __forceinline__ void ensure(const int32_t* __restrict__ col_idx, const int32_t* __restrict__ blk_idx,
                                         int64_t nnzb, int64_t pb, int lane) {
    if (pb < base || pb >= base + 64) {
      base = pb;
      fetch(col_idx, blk_idx, nnzb, base + lane, c0, b0);
      fetch(col_idx, blk_idx, nnzb, base + 32 + lane, c1, b1);
      fetch(col_idx, blk_idx, nnzb, base + 64 + lane, c2, b2);
    } else if (pb >= base + 32) {
      c0 = c1;
      b0 = b1;
      c1 = c2;
      b1 = b2;
      base += 32;
      fetch(col_idx, blk_idx, nnzb, base + 64 + lane, c2, b2);
    }
  }

  // Entry of position p (base <= p < base + 64; other lanes get junk).
  // Every lane of the warp must call this.
  __device__ __forceinline__ void get(int64_t p, int& c, int& b) const {
    const int d = static_cast<int>(p - base);
    const int src = d & 31;
    const int xc0 = __shfl_sync(0xffffffffu, c0, src), xc1 = __shfl_sync(0xffffffffu, c1, src);
    const int xb0 = __shfl_sync(0xffffffffu, b0, src), xb1 = __shfl_sync(0xffffffffu, b1, src);
    c = d < 32 ? xc0 : xc1;
    b = d < 32 ? xb0 : xb1;
  }
};

// Named barrier 1 over the 128 epilogue threads.
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// OR of `pred` over the 128 epilogue threads (named barrier 1).  Used so that
// the four epilogue warps always leave the work loop at the same item; a warp
// that left alone would strand the others at the next named barrier.
__device__ __forceinline__ bool epi_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t"
      ".reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t"
      "}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred))
      : "memory");
  return r != 0;
}

}  // namespace kairo
