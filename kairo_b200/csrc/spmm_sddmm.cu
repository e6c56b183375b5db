// Weight gradient of the block-sparse linear layer: a block-sampled
// dense x dense product (SDDMM) on sm_100a.
//
//   Y  = X * W^T                 (forward, LINEAR layout of kairo_bsr_spmm)
//   dW[p] = dY[:, i*bm : (i+1)*bm]^T * X[:, j*bk : (j+1)*bk]
// for every nonzero block p = (block-row i, block-column j) of W, summed over
// the N batch rows; dY is (N x M) and X is (N x K), both row-major.  The
// reference has no SpMM backward; the math is that of torch's autograd of
// Y = X @ W.T restricted to W's nonzero blocks.
//
// Work.  Blocks are visited by block-column j (the transposed structure from
// kairo_bsr_transpose).  A work item is up to U stacks of S = 128 / bm
// blocks of one column, all sharing one X panel: every batch slab loads the
// item's dY boxes and ONE X box, so the L2 -> SM gathers (which bound this
// kernel) are 1 + 1/(S*U) boxes per block instead of 1 + 1/S.  One stack
// is one MMA tile: M = S * bm rows (the stacked dY panels, transposed),
// N = bk, K = the batch, streamed in slabs of KB rows:
//   operand A = S dY boxes (bm columns x KB rows each), MN-major;
//   operand B = the X box  (bk columns x KB rows),      MN-major;
//   D in TMEM = 128 lanes (block rows of the S blocks) x bk fp32 columns,
//               one accumulator per stack, two sets of U (512 columns).
// Rows of a stack beyond the item's last block repeat that block and are
// not written.
//
// Roles (192 threads, persistent): warp 0 TMA producer, warp 1 TMEM
// allocator + MMA issuer, warps 2..5 epilogue (TMEM -> dW).  Every mbarrier
// wait is bounded as in spmm_tc.cu.
//
// A CUDA-core kernel covers the other block sizes and fp32.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <sstream>

#include "internal.h"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace kairo {
namespace {

constexpr int kSddKB = 64;          // batch rows per pipeline stage
constexpr int kSddU = 4;            // stacks (MMA tiles) per work item, sharing the X box
constexpr int kItemScanThreads = 1024;

struct SddItem {
  int32_t q0;    // first transposed position of the stack
  int32_t cnt;   // blocks in the item (1..S*U)
  int32_t col;   // block-column j
  int32_t pad;
};

// Workspace: header (error word at 0, item count at 64), then the items.
struct SddWs {
  unsigned* err;
  int* nitems;
  SddItem* items;
};

SddWs carve_sdd(void* ws) {
  uint8_t* p = static_cast<uint8_t*>(ws);
  return SddWs{reinterpret_cast<unsigned*>(p), reinterpret_cast<int*>(p + 64),
               reinterpret_cast<SddItem*>(p + kWorkspaceHeaderBytes)};
}

size_t sdd_ws_bytes(int64_t nnzb, int64_t nbc, int S) {
  const int64_t max_items = nnzb / S + nbc + 1;
  return kWorkspaceHeaderBytes + static_cast<size_t>(max_items) * sizeof(SddItem);
}

// One CTA: for every block-column, ceil(len / S) items of up to S blocks;
// exclusive scan of the item counts, then the item list.
__global__ void __launch_bounds__(kItemScanThreads) k_sdd_items(const int32_t* __restrict__ row_ptr_t, int32_t nbc,
                                                                int S, SddItem* __restrict__ items, int* nitems) {
  __shared__ int warp_sums[kItemScanThreads / 32];
  __shared__ int carry_s;
  if (threadIdx.x == 0) carry_s = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = 0; base < nbc; base += kItemScanThreads) {
    const int j = base + threadIdx.x;
    int len = 0;
    if (j < nbc) len = max(0, row_ptr_t[j + 1] - row_ptr_t[j]);
    const int v = (len + S - 1) / S;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int s = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      warp_sums[lane] = s;
    }
    __syncthreads();
    const int carry = carry_s;
    const int incl = x + (warp > 0 ? warp_sums[warp - 1] : 0) + carry;
    const int first = incl - v;
    for (int s = 0; s < v; ++s) {
      SddItem it;
      it.q0 = row_ptr_t[j] + s * S;
      it.cnt = min(S, len - s * S);
      it.col = j;
      it.pad = 0;
      items[first + s] = it;
    }
    __syncthreads();
    if (threadIdx.x == kItemScanThreads - 1) carry_s = incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) *nitems = carry_s;
}

struct SddArgs {
  const SddItem* items;
  const int* nitems;
  const int32_t* col_idx_t;  // block-row of every transposed position
  const int32_t* perm_t;     // W position of every transposed position
  void* dblocks;             // (nnzb, bm, bk)
  unsigned* err;
  int64_t n;                 // batch rows
  int32_t nbr;
  int32_t nnzb;
  int32_t stages;
};

template <typename TOut>
__device__ __forceinline__ void store_row16(TOut* dst, const float* v);
template <>
__device__ __forceinline__ void store_row16<float>(float* dst, const float* v) {
  float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}
template <typename T16>
__device__ __forceinline__ void store_row16_16bit(T16* dst, const float* v) {
  uint32_t w[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    T16 lo, hi;
    store_scalar<T16>(&lo, v[2 * q]);
    store_scalar<T16>(&hi, v[2 * q + 1]);
    w[q] = static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&lo)) |
           (static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&hi)) << 16);
  }
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
  d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
}
template <>
__device__ __forceinline__ void store_row16<__half>(__half* dst, const float* v) {
  store_row16_16bit(dst, v);
}
template <>
__device__ __forceinline__ void store_row16<__nv_bfloat16>(__nv_bfloat16* dst, const float* v) {
  store_row16_16bit(dst, v);
}

// tcgen05 kernel for bm = bk = 64 (S = 2 blocks per stack, U stacks per item).
template <int IN_FMT, typename TOut>
__global__ void __launch_bounds__(kThreads, 1)
    bsr_sddmm_tc_kernel(const __grid_constant__ CUtensorMap tmap_dy, const __grid_constant__ CUtensorMap tmap_x,
                        const SddArgs args) {
  constexpr int BS = 64;
  constexpr int S = 128 / BS;
  constexpr int U = kSddU;
  constexpr int SU = S * U;                          // blocks per item
  constexpr int KB = kSddKB;
  constexpr int BOX_BYTES = BS * KB * 2;             // one 64-column box of KB rows
  constexpr int STAGE_BYTES = (SU + 1) * BOX_BYTES;  // SU dY boxes, then the X box
  constexpr uint32_t IDESC = ptx::make_idesc_f16(IN_FMT, 1u, 1u, 128u, BS);
  constexpr uint32_t SET_COLS = U * BS;              // one accumulator set: U stacks
  constexpr uint32_t TMEM_COLS = 2 * SET_COLS;       // two sets (512 columns)
  static_assert(TMEM_COLS <= 512, "TMEM budget");
  constexpr uint32_t KSTEP16 = (16 * 128) >> 4;      // 16 batch rows of a 128-byte atom row

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ST = args.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ST * STAGE_BYTES);
  uint64_t* empty = full + ST;
  uint64_t* tfull = empty + ST;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  int* misc = reinterpret_cast<int*>(mma_done + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 0);
  volatile int* abort_flag = misc + 1;
  int* issued = misc + 4;  // [ST]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
      issued[s] = 0;
    }
    for (int k = 0; k < 2; ++k) {
      ptx::mbar_init(&tfull[k], 1);
      ptx::mbar_init(&tempty[k], 4);
    }
    ptx::mbar_init(mma_done, 1);
    misc[1] = 0;
    ptx::mbar_init_fence();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_dy);
    ptx::prefetch_tmap(&tmap_x);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, TMEM_COLS);
    ptx::tmem_relinquish();
  }
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nitems = *args.nitems;
  const int G = gridDim.x;
  const int nslabs = static_cast<int>((args.n + KB - 1) / KB);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol_dy = ptx::policy_evict_last();
    const uint64_t pol_x = ptx::policy_evict_first();
    int sidx = 0;
    uint32_t sph = 0;
    bool alive = true;
    for (int t = blockIdx.x; t < nitems && alive; t += G) {
      const SddItem it = args.items[t];
      const int nst = (it.cnt + S - 1) / S;  // stacks in this item
      const uint32_t tx = static_cast<uint32_t>(nst * S + 1) * BOX_BYTES;
      // lane l < nst*S: block-row of item slot l (the last block repeated)
      int row = 0;
      if (lane < nst * S) {
        const int q = it.q0 + min(lane, it.cnt - 1);
        row = (q >= 0 && q < args.nnzb) ? __ldg(args.col_idx_t + q) : -1;
        if (row < 0 || row >= args.nbr) {
          atomicCAS(args.err, 0u, KAIRO_DEVERR_BAD_INDEX);
          row = 0;
        }
      }
      for (int slab = 0; slab < nslabs; ++slab) {
        int ok = ptx::wait_parity(&empty[sidx], sph ^ 1u, abort_flag, args.err, kTagEmpty, kWaitCycles);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          alive = false;
          break;
        }
        if (lane == 0) issued[sidx] = static_cast<int>(sph) + 1;
        uint8_t* st = smem + sidx * STAGE_BYTES;
        const int y = slab * KB;
        ptx::mbar_expect_tx_if(lane == 0 ? 1u : 0u, &full[sidx], tx);
        ptx::tma_load_2d_if(lane < nst * S ? 1u : 0u, st + lane * BOX_BYTES, &tmap_dy, row * BS, y, &full[sidx],
                            pol_dy);
        ptx::tma_load_2d_if(lane == 31 ? 1u : 0u, st + SU * BOX_BYTES, &tmap_x, it.col * BS, y, &full[sidx], pol_x);
        __syncwarp();
        ptx::mbar_arrive_if(lane == 0 ? 1u : 0u, &full[sidx]);
        if (++sidx == ST) {
          sidx = 0;
          sph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t leader = lane == 0 ? 1u : 0u;
    const uint32_t sbase = ptx::smem_u32(smem);
    // A: S dY boxes side by side along M (atom stride BOX_BYTES); B: the X box.
    const uint64_t adesc0 = ptx::make_smem_desc(sbase, BOX_BYTES, 1024, 2u);
    const uint64_t bdesc0 = ptx::make_smem_desc(sbase + SU * BOX_BYTES, BOX_BYTES, 1024, 2u);
    const uint32_t a_lo0 = static_cast<uint32_t>(adesc0), a_hi = static_cast<uint32_t>(adesc0 >> 32);
    const uint32_t b_lo0 = static_cast<uint32_t>(bdesc0), b_hi = static_cast<uint32_t>(bdesc0 >> 32);
    constexpr uint32_t STAGE16 = STAGE_BYTES >> 4;
    int sidx = 0;
    uint32_t sph = 0;
    int slot = 0;
    uint32_t aphase = 0;
    bool alive = true;
    for (int t = blockIdx.x; t < nitems && alive; t += G) {
      const int nst = (args.items[t].cnt + S - 1) / S;
      int ok = ptx::wait_parity(&tempty[slot], aphase ^ 1u, abort_flag, args.err, kTagTmemEmpty, kWaitCycles);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      ptx::tc_fence_after();
      const uint32_t d = tmem_base + static_cast<uint32_t>(slot) * SET_COLS;
      for (int slab = 0; slab < nslabs; ++slab) {
        ok = ptx::wait_parity(&full[sidx], sph, abort_flag, args.err, kTagFull, kWaitCycles);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          alive = false;
          break;
        }
        const uint32_t s16 = static_cast<uint32_t>(sidx) * STAGE16;
        for (int u = 0; u < nst; ++u) {
          const uint32_t u16 = static_cast<uint32_t>(u * S * BOX_BYTES) >> 4;
#pragma unroll
          for (int kk = 0; kk < KB / 16; ++kk) {
            ptx::mma_f16_ss_if(leader, d + static_cast<uint32_t>(u * BS), a_lo0 + s16 + u16 + kk * KSTEP16, a_hi,
                               b_lo0 + s16 + kk * KSTEP16, b_hi, IDESC, (slab > 0 || kk > 0) ? 1u : 0u);
          }
        }
        ptx::mma_commit_if(leader, &empty[sidx]);
        if (++sidx == ST) {
          sidx = 0;
          sph ^= 1u;
        }
      }
      if (!alive) break;
      ptx::mma_commit_if(leader, &tfull[slot]);
      slot ^= 1;
      if (slot == 0) aphase ^= 1u;
    }
    ptx::mma_commit_if(leader, mma_done);
    int dummy = 0;
    ptx::wait_parity(mma_done, 0, reinterpret_cast<volatile int*>(&dummy), args.err, kTagDrain, kWaitCycles);
    __syncwarp();
  } else if (warp >= 2 && warp <= 5) {
    // ------------------------------------------------------------ epilogue
    const int qtr = warp & 3;
    const int e = qtr * 32 + lane;  // TMEM lane: row e % BS of slot e / BS of a stack
    const int sslot = e / BS, r = e % BS;
    const uint32_t lane_addr = static_cast<uint32_t>(qtr * 32) << 16;
    int slot = 0;
    uint32_t aphase = 0;
    for (int t = blockIdx.x; t < nitems; t += G) {
      const SddItem it = args.items[t];
      int ok = ptx::wait_parity(&tfull[slot], aphase, abort_flag, args.err, kTagTmemFull, kWaitCycles, 200);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (epi_any(!ok)) break;
      ptx::tc_fence_after();
      const int nst = (it.cnt + S - 1) / S;
      for (int u = 0; u < nst; ++u) {
        const int bi = u * S + sslot;  // block of the item in this lane's TMEM rows
        int p = -1;
        if (bi < it.cnt) {
          const int q = it.q0 + bi;
          p = (q >= 0 && q < args.nnzb) ? __ldg(args.perm_t + q) : -1;
          if (p >= args.nnzb) p = -1;
        }
        TOut* dst = p >= 0 ? static_cast<TOut*>(args.dblocks) + (static_cast<int64_t>(p) * BS + r) * BS : nullptr;
        const uint32_t cols = static_cast<uint32_t>(slot) * SET_COLS + static_cast<uint32_t>(u * BS);
#pragma unroll
        for (int c0 = 0; c0 < BS; c0 += 16) {
          float v[16];
          ptx::tmem_ld16(tmem_base + lane_addr + cols + static_cast<uint32_t>(c0), v);
          ptx::tmem_wait_ld();
          if (dst) store_row16<TOut>(dst + c0, v);
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&tempty[slot]);
      slot ^= 1;
      if (slot == 0) aphase ^= 1u;
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    int dummy = 0;
    for (int s = 0; s < ST; ++s)
      if (issued[s])
        ptx::wait_parity(&full[s], static_cast<uint32_t>(issued[s] - 1), reinterpret_cast<volatile int*>(&dummy),
                         args.err, kTagDrain, kWaitCycles);
  }
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// CUDA-core kernel for every shape: one CTA per transposed position q
// computes dW[perm_t[q]] (bm x bk) over the batch in slabs of 32 rows staged
// in shared memory; each thread owns (bm * bk) / 256 outputs.
template <typename TIn, typename TOut>
__global__ void __launch_bounds__(256) bsr_sddmm_simt_kernel(
    const TIn* __restrict__ dy, int64_t lddy, const TIn* __restrict__ x, int64_t ldx, int64_t n, int64_t m, int64_t k,
    const int32_t* __restrict__ col_idx, const int32_t* __restrict__ col_idx_t, const int32_t* __restrict__ perm_t,
    int32_t nnzb, int32_t nbr, int32_t nbc, int32_t bm, int32_t bk, TOut* __restrict__ dblocks, unsigned* err) {
  __shared__ float sdy[32][65];
  __shared__ float sx[32][65];
  for (int q = blockIdx.x; q < nnzb; q += gridDim.x) {
    const int p = perm_t[q];
    const int i = col_idx_t[q];
    const bool ok = p >= 0 && p < nnzb && i >= 0 && i < nbr && col_idx[p] >= 0 && col_idx[p] < nbc;
    if (!ok) {
      if (threadIdx.x == 0) atomicCAS(err, 0u, KAIRO_DEVERR_BAD_INDEX);
      continue;
    }
    const int j = col_idx[p];
    float acc[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) acc[u] = 0.f;
    const int outs = bm * bk;
    for (int64_t n0 = 0; n0 < n; n0 += 32) {
      __syncthreads();
      for (int e = threadIdx.x; e < 32 * bm; e += blockDim.x) {
        const int rr = e / bm, c = e - rr * bm;
        const int64_t row = n0 + rr, col = static_cast<int64_t>(i) * bm + c;
        sdy[rr][c] = (row < n && col < m) ? static_cast<float>(dy[row * lddy + col]) : 0.f;
      }
      for (int e = threadIdx.x; e < 32 * bk; e += blockDim.x) {
        const int rr = e / bk, c = e - rr * bk;
        const int64_t row = n0 + rr, col = static_cast<int64_t>(j) * bk + c;
        sx[rr][c] = (row < n && col < k) ? static_cast<float>(x[row * ldx + col]) : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int o = threadIdx.x + u * 256;
        if (o < outs) {
          const int r = o / bk, c = o - r * bk;
          float s = acc[u];
#pragma unroll 8
          for (int rr = 0; rr < 32; ++rr) s += sdy[rr][r] * sx[rr][c];
          acc[u] = s;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int o = threadIdx.x + u * 256;
      if (o < outs) store_scalar<TOut>(dblocks + static_cast<int64_t>(p) * outs + o, acc[u]);
    }
  }
}

template <typename TIn, typename TOut>
kairo_status launch_simt(const kairo_bsr* a, const int32_t* col_idx_t, const int32_t* perm_t, const void* dy,
                         int64_t lddy, const void* x, int64_t ldx, int64_t n, void* dblocks, unsigned* err,
                         cudaStream_t s) {
  const int nbc = static_cast<int>(ceil_div64(a->cols, a->bk));
  const int g = static_cast<int>(std::min<int64_t>(a->nnzb, static_cast<int64_t>(device_sm_count(current_device())) * 8));
  bsr_sddmm_simt_kernel<TIn, TOut><<<g, 256, 0, s>>>(
      static_cast<const TIn*>(dy), lddy, static_cast<const TIn*>(x), ldx, n, a->rows, a->cols, a->col_idx, col_idx_t,
      perm_t, static_cast<int32_t>(a->nnzb), a->nbr, nbc, a->bm, a->bk, static_cast<TOut*>(dblocks), err);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the CUDA-core SDDMM kernel");
  return KAIRO_STATUS_SUCCESS;
}

using SddFn = void (*)(CUtensorMap, CUtensorMap, SddArgs);

SddFn pick_sdd(kairo_dtype in, kairo_dtype out) {
  if (in == KAIRO_DTYPE_F16) {
    if (out == KAIRO_DTYPE_F32) return reinterpret_cast<SddFn>(&bsr_sddmm_tc_kernel<0, float>);
    if (out == KAIRO_DTYPE_F16) return reinterpret_cast<SddFn>(&bsr_sddmm_tc_kernel<0, __half>);
  } else if (in == KAIRO_DTYPE_BF16) {
    if (out == KAIRO_DTYPE_F32) return reinterpret_cast<SddFn>(&bsr_sddmm_tc_kernel<1, float>);
    if (out == KAIRO_DTYPE_BF16) return reinterpret_cast<SddFn>(&bsr_sddmm_tc_kernel<1, __nv_bfloat16>);
  }
  return nullptr;
}

bool sdd_tc_ok(const kairo_bsr* a, const void* dy, int64_t lddy, const void* x, int64_t ldx, kairo_dtype out) {
  if (a->bm != 64 || a->bk != 64) return false;
  if (!pick_sdd(a->dtype, out)) return false;
  if ((lddy % 8) || (ldx % 8)) return false;
  if ((reinterpret_cast<uintptr_t>(dy) & 15u) || (reinterpret_cast<uintptr_t>(x) & 15u)) return false;
  return true;
}

}  // namespace
}  // namespace kairo

using namespace kairo;

extern "C" kairo_status kairo_bsr_sddmm_workspace_size(const kairo_bsr* a, size_t* bytes) {
  if (!a || !bytes) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  const int64_t nbc = ceil_div64(a->cols, a->bk);
  *bytes = sdd_ws_bytes(a->nnzb, nbc, std::max(1, 128 / std::max(1, a->bm)));
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_bsr_sddmm(const kairo_bsr* a, const int32_t* row_ptr_t, const int32_t* col_idx_t,
                                        const int32_t* perm_t, const void* dy, int64_t lddy, const void* x,
                                        int64_t ldx, int64_t n, void* dblocks, kairo_dtype out_dtype,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  if (!a) return fail(KAIRO_STATUS_INVALID_VALUE, "null BSR descriptor");
  if (a->rows < 0 || a->cols < 0 || a->nnzb < 0 || a->bm <= 0 || a->bk <= 0 || n < 0)
    return fail(KAIRO_STATUS_INVALID_VALUE, "invalid size");
  if (a->nnzb > 0x7fffffffLL) return fail(KAIRO_STATUS_NOT_SUPPORTED, "more than 2^31-1 blocks");
  if (a->dtype != KAIRO_DTYPE_F32 && a->dtype != KAIRO_DTYPE_F16 && a->dtype != KAIRO_DTYPE_BF16)
    return fail(KAIRO_STATUS_INVALID_VALUE, "unknown dtype");
  if (out_dtype != KAIRO_DTYPE_F32 && out_dtype != a->dtype)
    return fail(KAIRO_STATUS_INVALID_VALUE, "dW dtype must be fp32 or the input dtype");
  if (lddy < a->rows || ldx < a->cols) return fail(KAIRO_STATUS_INVALID_VALUE, "leading dimension too small");
  if (a->nnzb == 0) return KAIRO_STATUS_SUCCESS;
  if (!row_ptr_t || !col_idx_t || !perm_t || !a->col_idx || !dblocks || !workspace || (n > 0 && (!dy || !x)))
    return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  size_t need = 0;
  kairo_status st = kairo_bsr_sddmm_workspace_size(a, &need);
  if (st) return st;
  if (workspace_bytes < need) return fail(KAIRO_STATUS_WORKSPACE_TOO_SMALL, "SDDMM workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SddWs w = carve_sdd(workspace);
  cudaError_t e = cudaMemsetAsync(workspace, 0, kWorkspaceHeaderBytes, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(SDDMM workspace)");
  const size_t osz = out_dtype == KAIRO_DTYPE_F32 ? 4 : 2;
  if (n == 0) {
    e = cudaMemsetAsync(dblocks, 0, static_cast<size_t>(a->nnzb) * a->bm * a->bk * osz, s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(dW)");
    return KAIRO_STATUS_SUCCESS;
  }
  const bool tc = sdd_tc_ok(a, dy, lddy, x, ldx, out_dtype) && n <= 0x7fffffffLL && a->rows <= 0x7fffffffLL &&
                  a->cols <= 0x7fffffffLL;
  if (!tc) {
    switch (a->dtype) {
      case KAIRO_DTYPE_F32:
        return launch_simt<float, float>(a, col_idx_t, perm_t, dy, lddy, x, ldx, n, dblocks, w.err, s);
      case KAIRO_DTYPE_F16:
        return out_dtype == KAIRO_DTYPE_F32
                   ? launch_simt<__half, float>(a, col_idx_t, perm_t, dy, lddy, x, ldx, n, dblocks, w.err, s)
                   : launch_simt<__half, __half>(a, col_idx_t, perm_t, dy, lddy, x, ldx, n, dblocks, w.err, s);
      default:
        return out_dtype == KAIRO_DTYPE_F32
                   ? launch_simt<__nv_bfloat16, float>(a, col_idx_t, perm_t, dy, lddy, x, ldx, n, dblocks, w.err, s)
                   : launch_simt<__nv_bfloat16, __nv_bfloat16>(a, col_idx_t, perm_t, dy, lddy, x, ldx, n, dblocks,
                                                               w.err, s);
    }
  }
  const int nbc = static_cast<int>(ceil_div64(a->cols, a->bk));
  k_sdd_items<<<1, kItemScanThreads, 0, s>>>(row_ptr_t, nbc, 2 * kSddU, w.items, w.nitems);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the SDDMM item kernel");
  const CUtensorMapDataType dt =
      a->dtype == KAIRO_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap map_dy, map_x;
  st = make_map_2d(&map_dy, dy, dt, 2, static_cast<uint64_t>(a->rows), static_cast<uint64_t>(n),
                   static_cast<uint64_t>(lddy), 64, kSddKB, "dY");
  if (st) return st;
  st = make_map_2d(&map_x, x, dt, 2, static_cast<uint64_t>(a->cols), static_cast<uint64_t>(n),
                   static_cast<uint64_t>(ldx), 64, kSddKB, "X");
  if (st) return st;
  constexpr int stage_bytes = (2 * kSddU + 1) * 64 * kSddKB * 2;
  const int budget = kMaxSmem - 1024 - 1024;
  const int stages = std::min(8, budget / stage_bytes);
  SddArgs args{};
  args.items = w.items;
  args.nitems = w.nitems;
  args.col_idx_t = col_idx_t;
  args.perm_t = perm_t;
  args.dblocks = dblocks;
  args.err = w.err;
  args.n = n;
  args.nbr = a->nbr;
  args.nnzb = static_cast<int32_t>(a->nnzb);
  args.stages = stages;
  SddFn fn = pick_sdd(a->dtype, out_dtype);
  const size_t smem = static_cast<size_t>(stages) * stage_bytes + 2048;
  e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  const int64_t max_items = a->nnzb / (2 * kSddU) + nbc;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(device_sm_count(current_device()), max_items)));
  fn<<<grid, kThreads, smem, s>>>(map_dy, map_x, args);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the tcgen05 SDDMM kernel");
  return KAIRO_STATUS_SUCCESS;
}
