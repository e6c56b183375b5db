// fp32 BSR SpMM on the tcgen05 kernel by a bf16 split (opt-in kernel
// KAIRO_KERNEL_SPLIT_BF16; no counterpart in the reference, whose fp32 path
// is the scalar kernel of csrc/acc_spmm_kernel.cu:115-152).
//
// Every fp32 value v is written as hi + lo with hi = bf16(v) and
// lo = bf16(v - hi).  The product is taken as
//   A·B ≈ A_hi·B_hi + A_hi·B_lo + A_lo·B_hi
// (the dropped A_lo·B_lo term and lo's own rounding are about 2^-16 of each
// product), with the products exact in fp32 and accumulated in fp32 by the
// tensor cores.  All three terms are one SpMM over a derived bf16 matrix:
//   block q of A      -> blocks 3q, 3q+1, 3q+2 = (hi, hi, lo), block-columns
//                        3c, 3c+1, 3c+2 for A's block-column c;
//   block-row c of B  -> block-rows 3c, 3c+1, 3c+2 = (hi, lo, hi) of a
//                        (3 * nbc * bk) x N bf16 B.
// One kernel builds the derived operands in the caller's workspace; the
// tcgen05 kernel then runs on them unchanged.
#include <cuda_bf16.h>

#include <algorithm>

#include "internal.h"

namespace kairo {
namespace {

__device__ __forceinline__ void split_bf16(float v, __nv_bfloat16* hi, __nv_bfloat16* lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  const float hf = __bfloat162float(h);
  *hi = h;
  // An infinite or NaN hi (v not finite, or rounded past the largest
  // finite bf16) keeps lo at zero so that hi alone carries the value.
  *lo = isfinite(hf) ? __float2bfloat16_rn(v - hf) : __float2bfloat16_rn(0.f);
}

// CTAs for `items` threads of work: at most 8 resident CTAs per SM of the
// current device.
int grid_for(int64_t items, int threads) {
  const int64_t cap = static_cast<int64_t>(device_sm_count(current_device())) * 8;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((items + threads - 1) / threads, cap)));
}

__device__ __forceinline__ uint2 pack4(__nv_bfloat16 a, __nv_bfloat16 b, __nv_bfloat16 c, __nv_bfloat16 d) {
  __nv_bfloat162 lo2, hi2;
  lo2.x = a;
  lo2.y = b;
  hi2.x = c;
  hi2.y = d;
  uint2 r;
  r.x = *reinterpret_cast<uint32_t*>(&lo2);
  r.y = *reinterpret_cast<uint32_t*>(&hi2);
  return r;
}

// Derived blocks, block-column indices and row pointers, one warp per block
// (elems is bm * bk with bk a multiple of 16, so a block is whole float4s).
// A block whose storage index is out of range becomes a zero block with
// column -1, which the tcgen05 kernel reports as KAIRO_DEVERR_BAD_INDEX; an
// out-of-range block-column maps to an out-of-range derived column, reported
// the same way.
__device__ void split_blocks_part(int64_t cta, int64_t ncta, const float* __restrict__ blocks,
                                  const int32_t* __restrict__ blk_idx, int64_t nblocks_stored,
                                  const int32_t* __restrict__ col_idx, const int32_t* __restrict__ row_ptr,
                                  int32_t nbr, int64_t nnzb, int32_t elems, __nv_bfloat16* __restrict__ out,
                                  int32_t* __restrict__ col_out, int32_t* __restrict__ row_ptr_out) {
  const int64_t tstride = ncta * blockDim.x;
  for (int64_t i = cta * blockDim.x + threadIdx.x; i <= nbr; i += tstride) row_ptr_out[i] = 3 * row_ptr[i];
  const int lane = threadIdx.x & 31;
  const int64_t warps = tstride / 32;
  const int vecs = elems / 4;
  for (int64_t q = (cta * blockDim.x + threadIdx.x) / 32; q < nnzb; q += warps) {
    const int64_t blk = blk_idx ? static_cast<int64_t>(blk_idx[q]) : q;
    const int64_t c3 = 3 * static_cast<int64_t>(col_idx[q]);
    const bool in_store = blk >= 0 && blk < nblocks_stored;
    const bool ok = in_store && c3 >= 0 && c3 + 2 <= INT32_MAX;
    if (lane < 3) col_out[3 * q + lane] = ok ? static_cast<int32_t>(c3 + lane) : -1;
    const float4* src = reinterpret_cast<const float4*>(blocks + (in_store ? blk : 0) * elems);
    uint2* o0 = reinterpret_cast<uint2*>(out + (3 * q + 0) * elems);
    uint2* o1 = reinterpret_cast<uint2*>(out + (3 * q + 1) * elems);
    uint2* o2 = reinterpret_cast<uint2*>(out + (3 * q + 2) * elems);
    for (int v = lane; v < vecs; v += 32) {
      const float4 f = in_store ? src[v] : make_float4(0.f, 0.f, 0.f, 0.f);
      __nv_bfloat16 h0, h1, h2, h3, l0, l1, l2, l3;
      split_bf16(f.x, &h0, &l0);
      split_bf16(f.y, &h1, &l1);
      split_bf16(f.z, &h2, &l2);
      split_bf16(f.w, &h3, &l3);
      const uint2 hv = pack4(h0, h1, h2, h3);
      o0[v] = hv;
      o1[v] = hv;
      o2[v] = pack4(l0, l1, l2, l3);
    }
  }
}

// Derived B: row (3c + t) * bk + kk holds B's row c * bk + kk as hi (t = 0,
// 2) or lo (t = 1); rows past K are zero.  Threads run over the columns of
// kRowsPerPass source rows at a time (gridDim.y strides the row groups), so
// each thread has that many independent loads in flight and no per-element
// index is divided.
constexpr int kRowsPerPass = 4;

__device__ void split_b_part(int64_t cx, int64_t ncx, int64_t cy, int64_t ncy, const float* __restrict__ b,
                             int64_t ldb, int64_t k, int64_t n, int32_t bk, int64_t k_src, int64_t ldb_out,
                             __nv_bfloat16* __restrict__ out) {
  for (int64_t r0 = cy * kRowsPerPass; r0 < k_src; r0 += ncy * kRowsPerPass) {
    for (int64_t col = cx * blockDim.x + threadIdx.x; col < n; col += ncx * blockDim.x) {
      float v[kRowsPerPass];
#pragma unroll
      for (int u = 0; u < kRowsPerPass; ++u) {
        const int64_t r = r0 + u;
        v[u] = (r < k) ? b[r * ldb + col] : 0.f;  // rows in [k, k_src) are the zero padding
      }
#pragma unroll
      for (int u = 0; u < kRowsPerPass; ++u) {
        const int64_t r = r0 + u;
        if (r >= k_src) break;
        const int64_t c = r / bk;
        const int64_t kk = r - c * bk;
        __nv_bfloat16 hi, lo;
        split_bf16(v[u], &hi, &lo);
        out[((3 * c + 0) * bk + kk) * ldb_out + col] = hi;
        out[((3 * c + 1) * bk + kk) * ldb_out + col] = lo;
        out[((3 * c + 2) * bk + kk) * ldb_out + col] = hi;
      }
    }
  }
}

// Both splits in one launch: CTAs [0, nb_ctas) split the blocks, the rest
// split B as a (bx_ctas x by_ctas) grid of column chunks x row groups.
__global__ void __launch_bounds__(256) k_split(const float* __restrict__ blocks, const int32_t* __restrict__ blk_idx,
                                               int64_t nblocks_stored, const int32_t* __restrict__ col_idx,
                                               const int32_t* __restrict__ row_ptr, int32_t nbr, int64_t nnzb,
                                               int32_t elems, __nv_bfloat16* __restrict__ blocks_out,
                                               int32_t* __restrict__ col_out, int32_t* __restrict__ row_ptr_out,
                                               const float* __restrict__ b, int64_t ldb, int64_t k, int64_t n,
                                               int32_t bk, int64_t k_src, int64_t ldb_out,
                                               __nv_bfloat16* __restrict__ b_out, int32_t nb_ctas, int32_t bx_ctas,
                                               int32_t by_ctas) {
  const int64_t cta = blockIdx.x;
  if (cta < nb_ctas) {
    split_blocks_part(cta, nb_ctas, blocks, blk_idx, nblocks_stored, col_idx, row_ptr, nbr, nnzb, elems, blocks_out,
                      col_out, row_ptr_out);
  } else {
    const int64_t bc = cta - nb_ctas;
    const int64_t cy = bc / bx_ctas;
    split_b_part(bc - cy * bx_ctas, bx_ctas, cy, by_ctas, b, ldb, k, n, bk, k_src, ldb_out, b_out);
  }
}

constexpr size_t kAlign = 256;

size_t up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

}  // namespace

SplitLayout split_bf16_layout(const kairo_bsr* a, int64_t n) {
  SplitLayout l{};
  const int64_t nbc = ceil_div64(a->cols, a->bk);
  const int64_t elems = static_cast<int64_t>(a->bm) * a->bk;
  l.ldb = (n + 7) / 8 * 8;
  l.k = 3 * nbc * a->bk;
  l.blocks_off = 0;
  l.col_idx_off = up(static_cast<size_t>(3 * a->nnzb * elems) * 2);
  l.row_ptr_off = l.col_idx_off + up(static_cast<size_t>(3 * a->nnzb) * 4);
  l.b_off = l.row_ptr_off + up(static_cast<size_t>(a->nbr + 1) * 4);
  l.bytes = l.b_off + up(static_cast<size_t>(l.k) * static_cast<size_t>(l.ldb) * 2);
  return l;
}

kairo_bsr split_bf16_desc(const kairo_bsr* a, const SplitLayout& l, void* base) {
  kairo_bsr d = *a;
  d.cols = l.k;
  d.nnzb = 3 * a->nnzb;
  d.nblocks_stored = 3 * a->nnzb;
  d.blk_idx = nullptr;
  d.dtype = KAIRO_DTYPE_BF16;
  d.max_row_blocks = a->max_row_blocks > 0 ? 3 * a->max_row_blocks : 0;
  uint8_t* p = static_cast<uint8_t*>(base);
  d.blocks = p + l.blocks_off;
  d.col_idx = reinterpret_cast<const int32_t*>(p + l.col_idx_off);
  d.row_ptr = reinterpret_cast<const int32_t*>(p + l.row_ptr_off);
  return d;
}

kairo_status split_bf16_prepare(const kairo_bsr* a, const void* b, int64_t ldb, int64_t n, const SplitLayout& l,
                                void* base, cudaStream_t s) {
  uint8_t* p = static_cast<uint8_t*>(base);
  const int32_t elems = a->bm * a->bk;
  const int64_t k_src = l.k / 3;  // nbc * bk source rows, the last slab zero-padded past K
  const int nb_ctas = grid_for(std::max<int64_t>(a->nnzb * 32, a->nbr + 1), 256);
  const int bx_ctas = static_cast<int>(std::min<int64_t>((n + 255) / 256, 64));
  const int by_ctas = static_cast<int>(std::min<int64_t>((k_src + kRowsPerPass - 1) / kRowsPerPass,
                                                          static_cast<int64_t>(device_sm_count(current_device())) * 4));
  k_split<<<nb_ctas + bx_ctas * by_ctas, 256, 0, s>>>(
      static_cast<const float*>(a->blocks), a->blk_idx, a->nblocks_stored, a->col_idx, a->row_ptr, a->nbr, a->nnzb,
      elems, reinterpret_cast<__nv_bfloat16*>(p + l.blocks_off), reinterpret_cast<int32_t*>(p + l.col_idx_off),
      reinterpret_cast<int32_t*>(p + l.row_ptr_off), static_cast<const float*>(b), ldb, a->cols, n, a->bk, k_src,
      l.ldb, reinterpret_cast<__nv_bfloat16*>(p + l.b_off), nb_ctas, bx_ctas, by_ctas);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the split-bf16 kernel");
  return KAIRO_STATUS_SUCCESS;
}

}  // namespace kairo
