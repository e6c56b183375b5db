// Block-granular pruning support: block L2 norms and a deterministic top-k.
//
// The reference prunes element by element (kairo/training/sparse_rec/
// topology.py:50-118: scores = |w| of the active positions, keep the
// largest with topk, indices sorted).  At block granularity the score of a
// block is its L2 norm, and the same selection picks whole blocks; the
// linear-layer workload's mask is built this way (top 20 % of 64 x 64 blocks
// of an N(0, 0.02^2) weight by norm, indices sorted).
//
// kairo_topk_indices returns the indices of the `count` largest scores in
// ascending index order, ties at the threshold broken by lower index, so the
// result equals "topk, then sort" whenever scores are distinct and is fully
// deterministic otherwise.  It is a radix select over order-preserving
// 32-bit keys (four 8-bit digits, most significant first) followed by an
// order-preserving compaction; NaN scores rank below every number.
// Everything is asynchronous on the caller's stream.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "internal.h"

namespace kairo {
namespace {

constexpr int kNormThreads = 256;
constexpr int kSelThreads = 256;
constexpr int kChunk = 4096;  // scores per compaction CTA

template <typename T>
__device__ __forceinline__ float to_f(T v) {
  return static_cast<float>(v);
}
template <>
__device__ __forceinline__ float to_f<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

// One warp per block of a dense (m x k) matrix: norms[i * nbc + j].
template <typename T>
__global__ void __launch_bounds__(kNormThreads) k_dense_block_norms(const T* __restrict__ a, int64_t m, int64_t k,
                                                                    int64_t lda, int32_t bm, int32_t bk, int64_t nbc,
                                                                    int64_t nblocks, float* __restrict__ norms) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kNormThreads / 32);
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * (kNormThreads / 32) + (threadIdx.x >> 5); b < nblocks;
       b += warps) {
    const int64_t i = b / nbc, j = b - i * nbc;
    const int64_t r0 = i * bm, c0 = j * bk;
    const int rows = static_cast<int>(min(static_cast<int64_t>(bm), m - r0));
    const int cols = static_cast<int>(min(static_cast<int64_t>(bk), k - c0));
    float s = 0.f;
    for (int e = lane; e < rows * cols; e += 32) {
      const int r = e / cols, c = e - r * cols;
      const float v = to_f(a[(r0 + r) * lda + c0 + c]);
      s = fmaf(v, v, s);
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) norms[b] = sqrtf(s);
  }
}

// Sum of squares of the VE elements packed in a 16-byte vector.
template <typename T>
__device__ __forceinline__ float sumsq16(const uint4& v) {
  const T* e = reinterpret_cast<const T*>(&v);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < static_cast<int>(16 / sizeof(T)); ++i) {
    const float f = to_f(e[i]);
    s = fmaf(f, f, s);
  }
  return s;
}

// The same with 16-byte loads, for whole blocks whose rows start on 16-byte
// boundaries (bk and lda multiples of the vector, aligned base): a block row
// is vpr vectors, a warp covers 32 / vpr rows per step, so every step reads
// whole 16-byte-aligned row segments, coalesced.
template <typename T>
__global__ void __launch_bounds__(kNormThreads) k_dense_block_norms_vec(const T* __restrict__ a, int64_t lda,
                                                                        int32_t bm, int32_t bk, int64_t nbc,
                                                                        int64_t nblocks, float* __restrict__ norms) {
  constexpr int VE = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int vpr = bk / VE;  // vectors per block row (a power of two, <= 32)
  const int nvec = bm * vpr;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kNormThreads / 32);
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * (kNormThreads / 32) + (threadIdx.x >> 5); b < nblocks;
       b += warps) {
    const int64_t i = b / nbc, j = b - i * nbc;
    const T* base = a + i * bm * lda + j * bk;
    float s = 0.f;
#pragma unroll 4
    for (int e = lane; e < nvec; e += 32) {
      const int r = e / vpr, v = e - r * vpr;
      s += sumsq16<T>(*reinterpret_cast<const uint4*>(base + r * lda + v * VE));
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) norms[b] = sqrtf(s);
  }
}

// One warp per BSR position: norms[p] of block stored(p).
template <typename T>
__global__ void __launch_bounds__(kNormThreads) k_bsr_block_norms(const T* __restrict__ blocks,
                                                                  const int32_t* __restrict__ blk_idx, int64_t nnzb,
                                                                  int64_t nstored, int32_t elems,
                                                                  float* __restrict__ norms) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kNormThreads / 32);
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * (kNormThreads / 32) + (threadIdx.x >> 5); p < nnzb;
       p += warps) {
    const int64_t s = blk_idx ? static_cast<int64_t>(blk_idx[p]) : p;
    float acc = 0.f;
    if (s >= 0 && s < nstored) {
      const T* blk = blocks + s * elems;
      constexpr int VE = 16 / sizeof(T);
      if (elems % VE == 0 && (reinterpret_cast<uintptr_t>(blk) & 15u) == 0) {
        const uint4* b4 = reinterpret_cast<const uint4*>(blk);
#pragma unroll 4
        for (int e = lane; e < elems / VE; e += 32) acc += sumsq16<T>(b4[e]);
      } else {
        for (int e = lane; e < elems; e += 32) {
          const float v = to_f(blk[e]);
          acc = fmaf(v, v, acc);
        }
      }
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) norms[p] = (s >= 0 && s < nstored) ? sqrtf(acc) : __int_as_float(0x7fc00000);
  }
}

// Order-preserving key: larger float -> larger unsigned key; NaN -> 0.
__device__ __forceinline__ uint32_t score_key(float f) {
  if (f != f) return 0u;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Selection state in the workspace header.
struct SelState {
  uint32_t prefix;   // digits of the threshold key found so far
  uint32_t remain;   // keys equal to the prefix (at this digit) still to take
  uint32_t pad[2];
};

__global__ void k_sel_init(SelState* st, uint32_t count) {
  st->prefix = 0u;
  st->remain = count;
}

// Histogram of digit `shift` over keys whose higher digits equal the prefix.
__global__ void __launch_bounds__(kSelThreads) k_sel_hist(const float* __restrict__ scores, int64_t n, int shift,
                                                          const SelState* st, unsigned* __restrict__ hist) {
  __shared__ unsigned h[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const uint32_t prefix = st->prefix;
  const uint32_t hi_mask = shift >= 24 ? 0u : (0xffffffffu << (shift + 8));
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t key = score_key(scores[i]);
    if ((key & hi_mask) == (prefix & hi_mask)) atomicAdd(&h[(key >> shift) & 0xffu], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    if (h[i]) atomicAdd(&hist[i], h[i]);
}

// Picks the digit holding the remain-th largest key (counting from the top
// bucket down), updates the state and clears the histogram for the next pass.
__global__ void k_sel_pick(int shift, SelState* st, unsigned* hist) {
  if (threadIdx.x == 0) {
    uint32_t remain = st->remain;
    int digit = 0;
    for (int d = 255; d >= 0; --d) {
      const uint32_t c = hist[d];
      if (c >= remain) {
        digit = d;
        break;
      }
      remain -= c;
    }
    st->prefix |= static_cast<uint32_t>(digit) << shift;
    st->remain = remain;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
}

// Per chunk of kChunk scores: how many are selected (key > T), and how many
// equal T.
__global__ void __launch_bounds__(kSelThreads) k_sel_count(const float* __restrict__ scores, int64_t n,
                                                           const SelState* st, unsigned* __restrict__ gt_cnt,
                                                           unsigned* __restrict__ eq_cnt) {
  __shared__ unsigned sg, se;
  if (threadIdx.x == 0) sg = se = 0;
  __syncthreads();
  const uint32_t T = st->prefix;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kChunk;
  unsigned g = 0, e = 0;
  for (int64_t i = c0 + threadIdx.x; i < min(n, c0 + kChunk); i += blockDim.x) {
    const uint32_t key = score_key(scores[i]);
    g += key > T;
    e += key == T;
  }
  atomicAdd(&sg, g);
  atomicAdd(&se, e);
  __syncthreads();
  if (threadIdx.x == 0) {
    gt_cnt[blockIdx.x] = sg;
    eq_cnt[blockIdx.x] = se;
  }
}

// Exclusive scans of the per-chunk counts (one CTA, sequential over tiles).
__global__ void __launch_bounds__(1024) k_sel_scan(unsigned* __restrict__ gt_cnt, unsigned* __restrict__ eq_cnt,
                                                   int nchunks) {
  __shared__ unsigned sg[1024], se[1024];
  __shared__ unsigned carry_g, carry_e;
  if (threadIdx.x == 0) carry_g = carry_e = 0;
  __syncthreads();
  for (int base = 0; base < nchunks; base += 1024) {
    const int i = base + threadIdx.x;
    sg[threadIdx.x] = i < nchunks ? gt_cnt[i] : 0;
    se[threadIdx.x] = i < nchunks ? eq_cnt[i] : 0;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
      const unsigned ag = threadIdx.x >= o ? sg[threadIdx.x - o] : 0;
      const unsigned ae = threadIdx.x >= o ? se[threadIdx.x - o] : 0;
      __syncthreads();
      sg[threadIdx.x] += ag;
      se[threadIdx.x] += ae;
      __syncthreads();
    }
    if (i < nchunks) {
      const unsigned vg = gt_cnt[i], ve = eq_cnt[i];
      gt_cnt[i] = carry_g + sg[threadIdx.x] - vg;
      eq_cnt[i] = carry_e + se[threadIdx.x] - ve;
    }
    __syncthreads();
    if (threadIdx.x == 1023) {
      carry_g += sg[1023];
      carry_e += se[1023];
    }
    __syncthreads();
  }
}

// Writes the selected indices in ascending order: index i is selected if its
// key is above T, or equal to T and among the first `remain` such indices.
// Its output slot is (selected keys above T before it) + (selected equal
// keys before it).  One CTA per chunk; the chunk is walked in blockDim-sized
// tiles with a block-wide prefix count.
__global__ void __launch_bounds__(kSelThreads) k_sel_write(const float* __restrict__ scores, int64_t n,
                                                           const SelState* st, const unsigned* __restrict__ gt_off,
                                                           const unsigned* __restrict__ eq_off,
                                                           int64_t* __restrict__ out) {
  __shared__ unsigned wg[kSelThreads / 32], we[kSelThreads / 32];
  __shared__ unsigned run_g, run_e;
  const uint32_t T = st->prefix;
  const uint32_t take_eq = st->remain;
  if (threadIdx.x == 0) {
    run_g = gt_off[blockIdx.x];
    run_e = eq_off[blockIdx.x];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kChunk;
  const int64_t c1 = min(n, c0 + kChunk);
  for (int64_t base = c0; base < c1; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    uint32_t key = 0;
    bool valid = i < c1;
    if (valid) key = score_key(scores[i]);
    const bool g = valid && key > T;
    const bool e = valid && key == T;
    const unsigned bg = __ballot_sync(0xffffffffu, g), be = __ballot_sync(0xffffffffu, e);
    if (lane == 0) {
      wg[warp] = __popc(bg);
      we[warp] = __popc(be);
    }
    __syncthreads();
    unsigned pg = run_g, pe = run_e;
    for (int w = 0; w < warp; ++w) {
      pg += wg[w];
      pe += we[w];
    }
    const unsigned lt = (1u << lane) - 1u;
    const unsigned my_g = pg + __popc(bg & lt);
    const unsigned my_e = pe + __popc(be & lt);
    // slot = selected indices before i: all greater ones, plus equal ones
    // before i up to the quota.
    if (g || (e && my_e < take_eq)) out[my_g + min(my_e, take_eq)] = i;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned tg = 0, te = 0;
      for (int w = 0; w < kSelThreads / 32; ++w) {
        tg += wg[w];
        te += we[w];
      }
      run_g += tg;
      run_e += te;
    }
    __syncthreads();
  }
}

struct SelWs {
  unsigned* err;
  SelState* st;
  unsigned* hist;    // 256
  unsigned* gt_cnt;  // nchunks
  unsigned* eq_cnt;  // nchunks
};

int64_t sel_chunks(int64_t n) { return (n + kChunk - 1) / kChunk; }

size_t sel_ws_bytes(int64_t n) {
  return kWorkspaceHeaderBytes + 256 * sizeof(unsigned) + 2 * align_up(static_cast<size_t>(sel_chunks(n)), 64) * 4;
}

SelWs carve_sel(void* ws, int64_t n) {
  uint8_t* p = static_cast<uint8_t*>(ws);
  SelWs w;
  w.err = reinterpret_cast<unsigned*>(p);
  w.st = reinterpret_cast<SelState*>(p + 64);
  w.hist = reinterpret_cast<unsigned*>(p + kWorkspaceHeaderBytes);
  w.gt_cnt = w.hist + 256;
  w.eq_cnt = w.gt_cnt + align_up(static_cast<size_t>(sel_chunks(n)), 64);
  return w;
}

int grid_over(int64_t work, int per_cta) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + per_cta - 1) / per_cta, 148 * 16)));
}

}  // namespace
}  // namespace kairo

using namespace kairo;

extern "C" kairo_status kairo_block_norms(const void* a, int64_t m, int64_t k, int64_t lda, int32_t bm, int32_t bk,
                                          kairo_dtype dtype, float* norms, void* stream) {
  if (m < 0 || k < 0 || bm <= 0 || bk <= 0 || lda < k) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid size");
  const int64_t nbr = ceil_div64(m, bm), nbc = ceil_div64(k, bk), nb = nbr * nbc;
  if (nb == 0) return KAIRO_STATUS_SUCCESS;
  if (!a || !norms) return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int g = grid_over(nb, kNormThreads / 32);
  const int ve = dtype == KAIRO_DTYPE_F32 ? 4 : 8;
  const bool pow2 = bk >= ve && (bk / ve) <= 32 && ((bk / ve) & (bk / ve - 1)) == 0;
  const bool vec = pow2 && bk % ve == 0 && lda % ve == 0 && m % bm == 0 && k % bk == 0 &&
                   (reinterpret_cast<uintptr_t>(a) & 15u) == 0;
  if (vec) {
    switch (dtype) {
      case KAIRO_DTYPE_F32:
        k_dense_block_norms_vec<float><<<g, kNormThreads, 0, s>>>(static_cast<const float*>(a), lda, bm, bk, nbc, nb,
                                                                  norms);
        break;
      case KAIRO_DTYPE_F16:
        k_dense_block_norms_vec<__half><<<g, kNormThreads, 0, s>>>(static_cast<const __half*>(a), lda, bm, bk, nbc,
                                                                   nb, norms);
        break;
      case KAIRO_DTYPE_BF16:
        k_dense_block_norms_vec<__nv_bfloat16><<<g, kNormThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(a), lda,
                                                                          bm, bk, nbc, nb, norms);
        break;
      default:
        return fail(KAIRO_STATUS_INVALID_VALUE, "unknown dtype");
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch of the block-norm kernel");
    return KAIRO_STATUS_SUCCESS;
  }
  switch (dtype) {
    case KAIRO_DTYPE_F32:
      k_dense_block_norms<float><<<g, kNormThreads, 0, s>>>(static_cast<const float*>(a), m, k, lda, bm, bk, nbc, nb,
                                                            norms);
      break;
    case KAIRO_DTYPE_F16:
      k_dense_block_norms<__half><<<g, kNormThreads, 0, s>>>(static_cast<const __half*>(a), m, k, lda, bm, bk, nbc,
                                                             nb, norms);
      break;
    case KAIRO_DTYPE_BF16:
      k_dense_block_norms<__nv_bfloat16><<<g, kNormThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(a), m, k, lda,
                                                                    bm, bk, nbc, nb, norms);
      break;
    default:
      return fail(KAIRO_STATUS_INVALID_VALUE, "unknown dtype");
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the block-norm kernel");
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_bsr_block_norms(const kairo_bsr* a, float* norms, void* stream) {
  if (!a) return fail(KAIRO_STATUS_INVALID_VALUE, "null BSR descriptor");
  if (a->nnzb < 0 || a->bm <= 0 || a->bk <= 0) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid BSR size");
  if (a->nnzb == 0) return KAIRO_STATUS_SUCCESS;
  if (!norms || !a->blocks) return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int g = grid_over(a->nnzb, kNormThreads / 32);
  const int32_t elems = a->bm * a->bk;
  switch (a->dtype) {
    case KAIRO_DTYPE_F32:
      k_bsr_block_norms<float><<<g, kNormThreads, 0, s>>>(static_cast<const float*>(a->blocks), a->blk_idx, a->nnzb,
                                                          a->nblocks_stored, elems, norms);
      break;
    case KAIRO_DTYPE_F16:
      k_bsr_block_norms<__half><<<g, kNormThreads, 0, s>>>(static_cast<const __half*>(a->blocks), a->blk_idx,
                                                           a->nnzb, a->nblocks_stored, elems, norms);
      break;
    case KAIRO_DTYPE_BF16:
      k_bsr_block_norms<__nv_bfloat16><<<g, kNormThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(a->blocks),
                                                                  a->blk_idx, a->nnzb, a->nblocks_stored, elems,
                                                                  norms);
      break;
    default:
      return fail(KAIRO_STATUS_INVALID_VALUE, "unknown dtype");
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the BSR block-norm kernel");
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_topk_workspace_size(int64_t n, size_t* bytes) {
  if (!bytes || n < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid argument");
  *bytes = sel_ws_bytes(n);
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_topk_indices(const float* scores, int64_t n, int64_t count, int64_t* out,
                                           void* workspace, size_t workspace_bytes, void* stream) {
  if (n < 0 || count < 0 || count > n) return fail(KAIRO_STATUS_INVALID_VALUE, "count must be in [0, n]");
  if (n > 0xffffffffLL) return fail(KAIRO_STATUS_NOT_SUPPORTED, "more than 2^32-1 scores");
  if (count == 0) return KAIRO_STATUS_SUCCESS;
  if (!scores || !out || !workspace) return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  if (workspace_bytes < sel_ws_bytes(n)) return fail(KAIRO_STATUS_WORKSPACE_TOO_SMALL, "top-k workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SelWs w = carve_sel(workspace, n);
  cudaError_t e = cudaMemsetAsync(workspace, 0, kWorkspaceHeaderBytes + 256 * sizeof(unsigned), s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(top-k workspace)");
  k_sel_init<<<1, 1, 0, s>>>(w.st, static_cast<uint32_t>(count));
  const int g = grid_over(n, kSelThreads * 8);
  for (int shift = 24; shift >= 0; shift -= 8) {
    k_sel_hist<<<g, kSelThreads, 0, s>>>(scores, n, shift, w.st, w.hist);
    k_sel_pick<<<1, 256, 0, s>>>(shift, w.st, w.hist);
  }
  const int nch = static_cast<int>(sel_chunks(n));
  k_sel_count<<<nch, kSelThreads, 0, s>>>(scores, n, w.st, w.gt_cnt, w.eq_cnt);
  k_sel_scan<<<1, 1024, 0, s>>>(w.gt_cnt, w.eq_cnt, nch);
  k_sel_write<<<nch, kSelThreads, 0, s>>>(scores, n, w.st, w.gt_cnt, w.eq_cnt, out);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the top-k kernels");
  return KAIRO_STATUS_SUCCESS;
}
