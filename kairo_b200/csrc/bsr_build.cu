// Device-side COO tile list -> BSR conversion and dense -> tile gather.
//
// The BSR order is the reference's: a stable sort of the COO list by block
// row (kairo/ops/sparse_embedding.py:49-56, torch.argsort(stable=True)) and
// row offsets from per-row counts (sparse_embedding.py:23-46).  Stability is
// obtained without a global sort: tiles are scattered into their row's bucket
// with atomics (any order), then each bucket is sorted by original tile
// index, which is unique, so the result equals the stable order.  Input that
// is already row-sorted (the common case) skips both steps.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "internal.h"

namespace kairo {
namespace {

constexpr int kSortMax = kBucketSortMax;  // longest unsorted block-row sorted in shared memory
constexpr int kScanThreads = 1024;
constexpr int kScanTile = 4 * kScanThreads;  // counts per CTA of the multi-CTA scan
constexpr int kScanSingleMax = 16384;        // up to this many buckets the scan is one CTA
constexpr int kSegThreads = 1024;            // threads of the per-bucket sort
constexpr int kLaneSortMax = 8;              // buckets up to this long are sorted by one thread

// Build-workspace layout (after the 256-byte header holding the error word):
//   flags[0] = row list not sorted, flags[1] = longest row
struct BuildWs {
  unsigned* err;
  int* flags;
  int* counts;  // [nbr]
  int* fill;    // [nbr]
};

BuildWs carve(void* ws, int32_t nbr) {
  uint8_t* p = static_cast<uint8_t*>(ws);
  BuildWs w;
  w.err = reinterpret_cast<unsigned*>(p);
  w.flags = reinterpret_cast<int*>(p + 64);
  w.counts = reinterpret_cast<int*>(p + kWorkspaceHeaderBytes);
  w.fill = w.counts + align_up(static_cast<size_t>(nbr), 64);
  return w;
}

__global__ void k_count(const int32_t* __restrict__ rows, const int32_t* __restrict__ cols, int64_t nt, int32_t nbr,
                        int32_t nbc, int* counts, int* flags, unsigned* err) {
  __shared__ int descending;  // this CTA saw a row id below its predecessor
  if (threadIdx.x == 0) descending = 0;
  __syncthreads();
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < nt;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = rows[t];
    const int c = cols[t];
    if (r < 0 || r >= nbr || c < 0 || c >= nbc) {
      atomicCAS(err, 0u, KAIRO_DEVERR_BAD_INDEX);
      continue;
    }
    atomicAdd(counts + r, 1);
    if (t > 0 && rows[t - 1] > r) descending = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0 && descending) flags[0] = 1;  // one store per CTA, not per element
}

// Exclusive scan of counts into row_ptr (nbr + 1 entries) by one CTA, in
// tiles of kScanThreads; also records the longest row.
__global__ void __launch_bounds__(kScanThreads) k_scan(const int* __restrict__ counts, int32_t nbr,
                                                       int32_t* __restrict__ row_ptr, int* flags) {
  __shared__ int warp_sums[kScanThreads / 32];
  __shared__ int carry_s;
  if (threadIdx.x == 0) carry_s = 0;
  int longest = 0;
  __syncthreads();
  for (int base = 0; base < nbr; base += kScanThreads) {
    const int i = base + threadIdx.x;
    const int v = i < nbr ? counts[i] : 0;
    longest = max(longest, v);
    int x = v;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
    if (i < nbr) row_ptr[i] = incl - v;
    __syncthreads();
    if (threadIdx.x == kScanThreads - 1) carry_s = incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) row_ptr[nbr] = carry_s;
  // longest row
  for (int o = 16; o > 0; o >>= 1) longest = max(longest, __shfl_xor_sync(0xffffffffu, longest, o));
  if (flags && (threadIdx.x & 31) == 0) atomicMax(flags + 1, longest);
}

// Multi-CTA scan for many buckets: per-tile sums (and the longest count),
// one-CTA scan of the tile sums, then every tile scanned with its offset.
__global__ void __launch_bounds__(kScanThreads) k_tile_sums(const int* __restrict__ counts, int32_t n,
                                                            int* __restrict__ tile_sum, int* flags) {
  __shared__ int warp_sums[kScanThreads / 32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
  const int64_t end = min(static_cast<int64_t>(n), base + kScanTile);
  int sum = 0, longest = 0;
  for (int64_t i = base + threadIdx.x; i < end; i += kScanThreads) {
    const int v = counts[i];
    sum += v;
    longest = max(longest, v);
  }
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    longest = max(longest, __shfl_xor_sync(0xffffffffu, longest, o));
  }
  if ((threadIdx.x & 31) == 0) {
    warp_sums[threadIdx.x >> 5] = sum;
    if (flags) atomicMax(flags + 1, longest);
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    int t = warp_sums[threadIdx.x];
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) tile_sum[blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(kScanThreads) k_scan_apply(const int* __restrict__ counts, int32_t n,
                                                             const int* __restrict__ tile_off,
                                                             int32_t* __restrict__ out) {
  static_assert(kScanTile == 4 * kScanThreads, "four counts per thread");
  __shared__ int warp_sums[kScanThreads / 32];
  const int64_t i0 = static_cast<int64_t>(blockIdx.x) * kScanTile + 4 * threadIdx.x;
  int v[4];
  int t = 0;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    v[u] = i0 + u < n ? counts[i0 + u] : 0;
    t += v[u];
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = t;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  int excl = x - t + (warp > 0 ? warp_sums[warp - 1] : 0) + tile_off[blockIdx.x];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    if (i0 + u < n) out[i0 + u] = excl;
    excl += v[u];
  }
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) out[n] = tile_off[gridDim.x];
}

// Sorted input: identity permutation.  Unsorted input: scatter every tile
// into its row bucket (order inside the bucket fixed up by k_segsort).
__global__ void k_place(const int32_t* __restrict__ rows, const int32_t* __restrict__ cols, int64_t nt,
                        const int32_t* __restrict__ row_ptr, int* fill, int32_t* __restrict__ col_idx,
                        int32_t* __restrict__ perm, const int* flags, const unsigned* err) {
  if (*err) return;
  const bool unsorted = flags[0] != 0;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < nt;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (!unsorted) {
      perm[t] = static_cast<int32_t>(t);
      col_idx[t] = cols[t];
    } else {
      const int r = rows[t];
      const int pos = row_ptr[r] + atomicAdd(fill + r, 1);
      perm[pos] = static_cast<int32_t>(t);
    }
  }
}

// Ascending sort of one value per lane across a warp (bitonic network).
__device__ __forceinline__ int warp_sort_asc(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const int o = __shfl_xor_sync(0xffffffffu, v, j);
      const bool up = (lane & k) == 0;
      const bool lower = (lane & j) == 0;
      v = (lower == up) ? min(v, o) : max(v, o);
    }
  }
  return v;
}

// Sorts every unsorted bucket's tile indices (ascending, i.e. stable order)
// and writes col_idx from them.  Each CTA takes `chunk` consecutive buckets
// at a time, one per thread: buckets of up to kLaneSortMax entries are
// sorted by their thread, up to 32 by a warp in registers, longer ones (up
// to kSortMax) by the whole CTA in shared memory.
__global__ void __launch_bounds__(kSegThreads) k_segsort(const int32_t* __restrict__ cols,
                                                         const int32_t* __restrict__ row_ptr, int32_t nbr, int chunk,
                                                         int32_t* __restrict__ col_idx, int32_t* __restrict__ perm,
                                                         const int* flags, unsigned* err, bool long_rows_ok) {
  if (flags[0] == 0 || *err) return;
  extern __shared__ int keys[];
  __shared__ int big[kSegThreads];
  __shared__ int nbig;
  const int lane = threadIdx.x & 31;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * chunk; base < nbr;
       base += static_cast<int64_t>(gridDim.x) * chunk) {
    const int64_t r = base + threadIdx.x;
    int p0 = 0, len = 0;
    if (static_cast<int>(threadIdx.x) < chunk && r < nbr) {
      p0 = row_ptr[r];
      len = row_ptr[r + 1] - p0;
    }
    if (threadIdx.x == 0) nbig = 0;
    __syncthreads();
    if (len > 32) {
      if (len <= kSortMax) {
        big[atomicAdd(&nbig, 1)] = static_cast<int>(r);
      } else if (!long_rows_ok) {
        // Left unsorted; a caller that allows it orders such buckets itself.
        atomicCAS(err, 0u, KAIRO_DEVERR_ROW_TOO_LONG);
      }
    }
    if (len > 0 && len <= kLaneSortMax) {
      // Short bucket: sorted by its own lane in registers (odd-even
      // transposition network over kLaneSortMax slots).
      int a[kLaneSortMax];
#pragma unroll
      for (int i = 0; i < kLaneSortMax; ++i) a[i] = i < len ? perm[p0 + i] : 0x7fffffff;
      if (len > 1) {
#pragma unroll
        for (int round = 0; round < kLaneSortMax; ++round) {
#pragma unroll
          for (int i = round & 1; i + 1 < kLaneSortMax; i += 2) {
            const int lo = min(a[i], a[i + 1]);
            const int hi = max(a[i], a[i + 1]);
            a[i] = lo;
            a[i + 1] = hi;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kLaneSortMax; ++i) {
        if (i < len) {
          perm[p0 + i] = a[i];
          col_idx[p0 + i] = cols[a[i]];
        }
      }
    }
    unsigned todo = __ballot_sync(0xffffffffu, len > kLaneSortMax && len <= 32);
    while (todo) {
      const int j = __ffs(todo) - 1;
      todo &= todo - 1;
      const int q0 = __shfl_sync(0xffffffffu, p0, j);
      const int n = __shfl_sync(0xffffffffu, len, j);
      int v = lane < n ? perm[q0 + lane] : 0x7fffffff;
      v = warp_sort_asc(v);
      if (lane < n) {
        perm[q0 + lane] = v;
        col_idx[q0 + lane] = cols[v];
      }
    }
    __syncthreads();
    const int nb = nbig;
    for (int i = 0; i < nb; ++i) {
      const int rr = big[i];
      const int q0 = row_ptr[rr];
      const int n = row_ptr[rr + 1] - q0;
      int pw = 64;
      while (pw < n) pw <<= 1;
      for (int e = threadIdx.x; e < pw; e += kSegThreads) keys[e] = e < n ? perm[q0 + e] : 0x7fffffff;
      __syncthreads();
      for (int k = 2; k <= pw; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
          for (int e = threadIdx.x; e < pw; e += kSegThreads) {
            const int l = e ^ j;
            if (l > e) {
              const int a = keys[e], b = keys[l];
              const bool up = (e & k) == 0;
              if ((a > b) == up) {
                keys[e] = b;
                keys[l] = a;
              }
            }
          }
          __syncthreads();
        }
      }
      for (int e = threadIdx.x; e < n; e += kSegThreads) {
        const int t = keys[e];
        perm[q0 + e] = t;
        col_idx[q0 + e] = cols[t];
      }
      __syncthreads();
    }
  }
}

// Block-row of every BSR position (out[p] = i for row_ptr[i] <= p < row_ptr[i+1]).
// One warp per block-row; positions outside [0, nnzb) are skipped.
__global__ void k_expand_rows(const int32_t* __restrict__ row_ptr, int32_t nbr, int64_t nnzb,
                              int32_t* __restrict__ out) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t r = blockIdx.x * static_cast<int64_t>(warps) + (threadIdx.x >> 5); r < nbr;
       r += static_cast<int64_t>(gridDim.x) * warps) {
    const int64_t p0 = max(static_cast<int64_t>(0), static_cast<int64_t>(row_ptr[r]));
    const int64_t p1 = min(nnzb, static_cast<int64_t>(row_ptr[r + 1]));
    for (int64_t p = p0 + lane; p < p1; p += 32) out[p] = static_cast<int32_t>(r);
  }
}

// blocks_t[q] = transpose(blocks[stored(perm_t[q])]) for q < nnzb, through a
// shared-memory tile so that both the read and the write are coalesced.
// One CTA per output block (grid-stride); bm, bk <= 64.
template <typename T>
__global__ void __launch_bounds__(256) k_transpose_blocks(const T* __restrict__ blocks, const int32_t* __restrict__ blk_idx,
                                                          const int32_t* __restrict__ perm_t, int64_t nnzb,
                                                          int64_t nstored, int32_t bm, int32_t bk,
                                                          T* __restrict__ out, unsigned* err) {
  __shared__ T tile[64][65];
  for (int64_t q = blockIdx.x; q < nnzb; q += gridDim.x) {
    const int64_t p = perm_t[q];
    int64_t s = (p >= 0 && p < nnzb) ? (blk_idx ? static_cast<int64_t>(blk_idx[p]) : p) : -1;
    const bool ok = s >= 0 && s < nstored;
    if (!ok && threadIdx.x == 0) atomicCAS(err, 0u, KAIRO_DEVERR_BAD_INDEX);
    const T* src = blocks + (ok ? s : 0) * bm * bk;
    for (int e = threadIdx.x; e < bm * bk; e += blockDim.x) {
      const int r = e / bk, c = e - r * bk;
      T v;
      if (ok)
        v = src[e];
      else
        memset(&v, 0, sizeof(T));
      tile[r][c] = v;
    }
    __syncthreads();
    T* dst = out + q * bm * bk;  // (bk x bm) row-major
    for (int e = threadIdx.x; e < bm * bk; e += blockDim.x) {
      const int c = e / bm, r = e - c * bm;
      dst[e] = tile[r][c];
    }
    __syncthreads();
  }
}

// The same with 16-byte vectors (VE elements) on both sides: rows of bk and
// bm elements are multiples of VE, blocks 16-byte aligned.  A block is read
// as row vectors into a padded shared tile, and written as row vectors of
// the transposed block gathered down the tile's columns (the padding puts
// the rows of one column in different banks).
template <typename T>
__global__ void __launch_bounds__(256) k_transpose_blocks_vec(const T* __restrict__ blocks,
                                                              const int32_t* __restrict__ blk_idx,
                                                              const int32_t* __restrict__ perm_t, int64_t nnzb,
                                                              int64_t nstored, int32_t bm, int32_t bk,
                                                              T* __restrict__ out, unsigned* err) {
  constexpr int VE = 16 / sizeof(T);
  constexpr int kPitch = 64 + 4 / sizeof(T);  // elements per tile row: an odd number of 4-byte words
  __shared__ __align__(16) T tile[64 * kPitch];
  const int row_vecs = bk / VE;       // input vectors per block row
  const int out_vecs = bm / VE;       // output vectors per transposed row
  const int nvec = bm * row_vecs;     // vectors per block
  for (int64_t q = blockIdx.x; q < nnzb; q += gridDim.x) {
    const int64_t p = perm_t[q];
    const int64_t sidx = (p >= 0 && p < nnzb) ? (blk_idx ? static_cast<int64_t>(blk_idx[p]) : p) : -1;
    const bool ok = sidx >= 0 && sidx < nstored;
    if (!ok && threadIdx.x == 0) atomicCAS(err, 0u, KAIRO_DEVERR_BAD_INDEX);
    const uint4* src = reinterpret_cast<const uint4*>(blocks + (ok ? sidx : 0) * bm * bk);
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
      const int r = v / row_vecs, c0 = (v - r * row_vecs) * VE;
      const uint4 x = ok ? src[v] : make_uint4(0u, 0u, 0u, 0u);
      const T* xe = reinterpret_cast<const T*>(&x);
#pragma unroll
      for (int i = 0; i < VE; ++i) tile[r * kPitch + c0 + i] = xe[i];
    }
    __syncthreads();
    uint4* dst = reinterpret_cast<uint4*>(out + q * bm * bk);  // (bk x bm) row-major
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
      const int c = v / out_vecs, r0 = (v - c * out_vecs) * VE;
      uint4 y;
      T* ye = reinterpret_cast<T*>(&y);
#pragma unroll
      for (int i = 0; i < VE; ++i) ye[i] = tile[(r0 + i) * kPitch + c];
      dst[v] = y;
    }
    __syncthreads();
  }
}

// Dense (M x K) -> tiles (num_tiles, tile, tile), zero-padded at the edges.
// One thread copies one tile row segment of up to 8 elements.
template <typename T>
__global__ void k_dense_to_tiles(const T* __restrict__ a, int64_t m, int64_t k, int64_t lda,
                                 const int32_t* __restrict__ rows, const int32_t* __restrict__ cols, int64_t nt,
                                 int32_t tile, int32_t nbr, int32_t nbc, T* __restrict__ tiles, unsigned* err) {
  const int segs = (tile + 7) / 8;
  const int64_t total = nt * tile * segs;
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = g / (static_cast<int64_t>(tile) * segs);
    const int rem = static_cast<int>(g - t * tile * segs);
    const int rr = rem / segs;
    const int c0 = (rem - rr * segs) * 8;
    const int br = rows[t], bc = cols[t];
    T* dst = tiles + (t * tile + rr) * tile;
    const bool ok = br >= 0 && br < nbr && bc >= 0 && bc < nbc;
    if (!ok && rr == 0 && c0 == 0 && err) atomicCAS(err, 0u, KAIRO_DEVERR_BAD_INDEX);
    const int64_t r = static_cast<int64_t>(br) * tile + rr;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int cc = c0 + q;
      if (cc >= tile) break;
      const int64_t c = static_cast<int64_t>(bc) * tile + cc;
      T v;
      if (ok && r < m && c < k)
        v = a[r * lda + c];
      else
        memset(&v, 0, sizeof(T));
      dst[cc] = v;
    }
  }
}

int grid_for(int64_t work, int threads) {
  const int64_t g = (work + threads - 1) / threads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(g, 148 * 32)));
}

// Tile sums and offsets of the multi-CTA scan (none when one CTA scans).
size_t scan_tile_ints(int32_t n) {
  return n > kScanSingleMax ? 2 * align_up(static_cast<size_t>((n + kScanTile - 1) / kScanTile + 1), 64) : 0;
}

// Counting workspace shared by the BSR build and the bucket sort: header
// (error word, flags), per-bucket counts and fill counters, scan tiles.
size_t count_ws_bytes(int32_t n) {
  return kWorkspaceHeaderBytes + (2 * align_up(static_cast<size_t>(n), 64) + scan_tile_ints(n)) * sizeof(int);
}

int* scan_tiles_of(int* counts, int32_t n) { return counts + 2 * align_up(static_cast<size_t>(n), 64); }

// Exclusive scan of n counts into out[0..n] (out[n] = total); flags[1]
// receives the longest count.
void launch_scan(const int* counts, int32_t n, int32_t* out, int* flags, int* tiles, cudaStream_t s) {
  if (n <= kScanSingleMax) {
    k_scan<<<1, kScanThreads, 0, s>>>(counts, n, out, flags);
    return;
  }
  const int nt = (n + kScanTile - 1) / kScanTile;
  int* tile_sum = tiles;
  int* tile_off = tiles + align_up(static_cast<size_t>(nt + 1), 64);
  k_tile_sums<<<nt, kScanThreads, 0, s>>>(counts, n, tile_sum, flags);
  k_scan<<<1, kScanThreads, 0, s>>>(tile_sum, nt, tile_off, nullptr);
  k_scan_apply<<<nt, kScanThreads, 0, s>>>(counts, n, tile_off, out);
}

kairo_status launch_segsort(const int32_t* cols, const int32_t* row_ptr, int32_t n, int32_t* col_idx, int32_t* perm,
                            const int* flags, unsigned* err, bool long_ok, cudaStream_t s) {
  static bool attr_set[64] = {false};
  const int dev = current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&k_segsort),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSortMax * static_cast<int>(sizeof(int)));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_segsort)");
    attr_set[dev] = true;
  }
  // Two CTAs per SM; each takes `chunk` buckets (a multiple of 32) at a time.
  constexpr int kCtas = 2 * 148;
  int64_t chunk = (static_cast<int64_t>(n) + kCtas - 1) / kCtas;
  chunk = std::min<int64_t>(kSegThreads, std::max<int64_t>(32, (chunk + 31) / 32 * 32));
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(kCtas, (n + chunk - 1) / chunk)));
  k_segsort<<<grid, kSegThreads, kSortMax * sizeof(int), s>>>(cols, row_ptr, n, static_cast<int>(chunk), col_idx,
                                                              perm, flags, err, long_ok);
  return KAIRO_STATUS_SUCCESS;
}

}  // namespace

size_t bsr_build_ws_bytes(int64_t num_tiles, int32_t nbr) {
  (void)num_tiles;
  return count_ws_bytes(nbr);
}

}  // namespace kairo

using namespace kairo;

extern "C" kairo_status kairo_bsr_build_workspace_size(int64_t num_tiles, int32_t nbr, size_t* bytes) {
  if (!bytes || num_tiles < 0 || nbr < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid argument");
  *bytes = bsr_build_ws_bytes(num_tiles, nbr);
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_bsr_build(const int32_t* tile_row_ids, const int32_t* tile_col_ids, int64_t num_tiles,
                                        int32_t nbr, int32_t nbc, int32_t* row_ptr, int32_t* col_idx, int32_t* perm,
                                        int32_t* is_identity, int32_t* max_row_blocks, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  if (num_tiles < 0 || nbr < 0 || nbc < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "negative size");
  if (num_tiles > 0x7fffffffLL) return fail(KAIRO_STATUS_NOT_SUPPORTED, "more than 2^31-1 tiles");
  if (!row_ptr || !workspace || (num_tiles > 0 && (!tile_row_ids || !tile_col_ids || !col_idx || !perm)))
    return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  if (workspace_bytes < bsr_build_ws_bytes(num_tiles, nbr))
    return fail(KAIRO_STATUS_WORKSPACE_TOO_SMALL, "build workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  BuildWs w = carve(workspace, nbr);
  cudaError_t e;
  // Zero the header flags and both per-row arrays.
  e = cudaMemsetAsync(workspace, 0, bsr_build_ws_bytes(num_tiles, nbr), s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(build workspace)");
  if (num_tiles > 0) k_count<<<grid_for(num_tiles, 256), 256, 0, s>>>(tile_row_ids, tile_col_ids, num_tiles, nbr, nbc, w.counts, w.flags, w.err);
  launch_scan(w.counts, nbr, row_ptr, w.flags, scan_tiles_of(w.counts, nbr), s);
  if (num_tiles > 0) {
    k_place<<<grid_for(num_tiles, 256), 256, 0, s>>>(tile_row_ids, tile_col_ids, num_tiles, row_ptr, w.fill, col_idx,
                                                     perm, w.flags, w.err);
    kairo_status st = launch_segsort(tile_col_ids, row_ptr, nbr, col_idx, perm, w.flags, w.err, false, s);
    if (st) return st;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the BSR build kernels");
  // One read-back: error word and the sorted flag.
  unsigned hdr[32];
  e = cudaMemcpyAsync(hdr, workspace, sizeof(hdr), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "reading the BSR build status");
  const unsigned code = hdr[0] & 0xffu;
  if (code == KAIRO_DEVERR_BAD_INDEX)
    return fail(KAIRO_STATUS_INVALID_VALUE, "tile row/column id outside the block grid");
  if (code == KAIRO_DEVERR_ROW_TOO_LONG)
    return fail(KAIRO_STATUS_NOT_SUPPORTED, "unsorted tile list with a block-row longer than 16384 tiles");
  if (code) return fail(KAIRO_STATUS_DEVICE_ERROR, "device error during BSR build");
  if (is_identity) *is_identity = (reinterpret_cast<int*>(hdr)[16] == 0) ? 1 : 0;
  if (max_row_blocks) *max_row_blocks = reinterpret_cast<int*>(hdr)[17];
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_dense_to_tiles(const void* a, int64_t m, int64_t k, int64_t lda,
                                             const int32_t* tile_row_ids, const int32_t* tile_col_ids,
                                             int64_t num_tiles, int32_t tile, kairo_dtype dtype, void* tiles,
                                             void* stream) {
  if (m < 0 || k < 0 || num_tiles < 0 || tile <= 0 || lda < k) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid size");
  if (num_tiles == 0) return KAIRO_STATUS_SUCCESS;
  if (!a || !tile_row_ids || !tile_col_ids || !tiles) return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int32_t nbr = static_cast<int32_t>(ceil_div64(m, tile));
  const int32_t nbc = static_cast<int32_t>(ceil_div64(k, tile));
  const int64_t work = num_tiles * tile * ((tile + 7) / 8);
  const int g = grid_for(work, 256);
  switch (dtype) {
    case KAIRO_DTYPE_F32:
      k_dense_to_tiles<float><<<g, 256, 0, s>>>(static_cast<const float*>(a), m, k, lda, tile_row_ids, tile_col_ids,
                                               num_tiles, tile, nbr, nbc, static_cast<float*>(tiles), nullptr);
      break;
    case KAIRO_DTYPE_F16:
    case KAIRO_DTYPE_BF16:
      k_dense_to_tiles<uint16_t><<<g, 256, 0, s>>>(static_cast<const uint16_t*>(a), m, k, lda, tile_row_ids,
                                                  tile_col_ids, num_tiles, tile, nbr, nbc,
                                                  static_cast<uint16_t*>(tiles), nullptr);
      break;
    default:
      return fail(KAIRO_STATUS_INVALID_VALUE, "unknown dtype");
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the dense-to-tiles kernel");
  return KAIRO_STATUS_SUCCESS;
}

// ------------------------------------------------------------ bucket sort

namespace kairo {

// Bucket-sort workspace: header (error word, flags), per-bucket counts and
// fill counters, scan tiles.
size_t bucket_sort_ws_bytes(int32_t nbuckets) { return count_ws_bytes(nbuckets); }

kairo_status bucket_sort(const int32_t* keys, const int32_t* vals, int32_t nvals, int64_t n, int32_t nbuckets,
                         int32_t* bucket_ptr, int32_t* perm, int32_t* vals_sorted, void* ws, cudaStream_t s,
                         bool long_buckets_ok) {
  uint8_t* p = static_cast<uint8_t*>(ws);
  unsigned* err = reinterpret_cast<unsigned*>(p);
  int* flags = reinterpret_cast<int*>(p + 64);
  int* counts = reinterpret_cast<int*>(p + kWorkspaceHeaderBytes);
  int* fill = counts + align_up(static_cast<size_t>(nbuckets), 64);
  cudaError_t e = cudaMemsetAsync(ws, 0, bucket_sort_ws_bytes(nbuckets), s);
  // flags[0] = 1: the key list is treated as unsorted, so every bucket is
  // filled by atomic scatter and then sorted by original index.
  if (e == cudaSuccess) e = cudaMemsetAsync(flags, 1, 1, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(bucket-sort workspace)");
  if (n > 0) k_count<<<grid_for(n, 256), 256, 0, s>>>(keys, vals, n, nbuckets, nvals, counts, flags, err);
  launch_scan(counts, nbuckets, bucket_ptr, flags, scan_tiles_of(counts, nbuckets), s);
  if (n > 0) {
    k_place<<<grid_for(n, 256), 256, 0, s>>>(keys, vals, n, bucket_ptr, fill, vals_sorted, perm, flags, err);
    kairo_status st = launch_segsort(vals, bucket_ptr, nbuckets, vals_sorted, perm, flags, err, long_buckets_ok, s);
    if (st) return st;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the bucket-sort kernels");
  return KAIRO_STATUS_SUCCESS;
}

}  // namespace kairo

// ------------------------------------------------------------ transpose

namespace kairo {
namespace {

// Transpose workspace: the bucket sort's, then the block-row of every BSR
// position.
size_t transpose_ws_bytes(int64_t nnzb, int32_t nbc) {
  return bucket_sort_ws_bytes(nbc) + align_up(static_cast<size_t>(nnzb), 64) * sizeof(int32_t);
}

kairo_status transpose_values(const kairo_bsr* a, const int32_t* perm_t, void* blocks_t, unsigned* err,
                              cudaStream_t s) {
  if (a->nnzb == 0) return KAIRO_STATUS_SUCCESS;
  if (a->bm > 64 || a->bk > 64) return fail(KAIRO_STATUS_NOT_SUPPORTED, "transpose supports blocks up to 64 x 64");
  const int g = static_cast<int>(std::min<int64_t>(a->nnzb, 148 * 16));
  const int ve = a->dtype == KAIRO_DTYPE_F32 ? 4 : 8;
  const bool vec = a->bm % ve == 0 && a->bk % ve == 0 && reinterpret_cast<uintptr_t>(a->blocks) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(blocks_t) % 16 == 0;
  if (vec) {
    switch (a->dtype) {
      case KAIRO_DTYPE_F32:
        k_transpose_blocks_vec<float><<<g, 256, 0, s>>>(static_cast<const float*>(a->blocks), a->blk_idx, perm_t,
                                                        a->nnzb, a->nblocks_stored, a->bm, a->bk,
                                                        static_cast<float*>(blocks_t), err);
        break;
      case KAIRO_DTYPE_F16:
        k_transpose_blocks_vec<__half><<<g, 256, 0, s>>>(static_cast<const __half*>(a->blocks), a->blk_idx, perm_t,
                                                         a->nnzb, a->nblocks_stored, a->bm, a->bk,
                                                         static_cast<__half*>(blocks_t), err);
        break;
      case KAIRO_DTYPE_BF16:
        k_transpose_blocks_vec<__nv_bfloat16><<<g, 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(a->blocks), a->blk_idx, perm_t, a->nnzb, a->nblocks_stored, a->bm,
            a->bk, static_cast<__nv_bfloat16*>(blocks_t), err);
        break;
      default:
        return fail(KAIRO_STATUS_INVALID_VALUE, "unknown dtype");
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "launch of the block transpose kernel");
    return KAIRO_STATUS_SUCCESS;
  }
  switch (a->dtype) {
    case KAIRO_DTYPE_F32:
      k_transpose_blocks<float><<<g, 256, 0, s>>>(static_cast<const float*>(a->blocks), a->blk_idx, perm_t, a->nnzb,
                                                  a->nblocks_stored, a->bm, a->bk, static_cast<float*>(blocks_t), err);
      break;
    case KAIRO_DTYPE_F16:
      k_transpose_blocks<__half><<<g, 256, 0, s>>>(static_cast<const __half*>(a->blocks), a->blk_idx, perm_t, a->nnzb,
                                                   a->nblocks_stored, a->bm, a->bk, static_cast<__half*>(blocks_t), err);
      break;
    case KAIRO_DTYPE_BF16:
      k_transpose_blocks<__nv_bfloat16><<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(a->blocks), a->blk_idx,
                                                          perm_t, a->nnzb, a->nblocks_stored, a->bm, a->bk,
                                                          static_cast<__nv_bfloat16*>(blocks_t), err);
      break;
    default:
      return fail(KAIRO_STATUS_INVALID_VALUE, "unknown dtype");
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the block transpose kernel");
  return KAIRO_STATUS_SUCCESS;
}

kairo_status check_transpose_args(const kairo_bsr* a) {
  if (!a) return fail(KAIRO_STATUS_INVALID_VALUE, "null BSR descriptor");
  if (a->nbr < 0 || a->nnzb < 0 || a->bm <= 0 || a->bk <= 0 || a->rows < 0 || a->cols < 0)
    return fail(KAIRO_STATUS_INVALID_VALUE, "invalid BSR size");
  if (a->nnzb > 0x7fffffffLL) return fail(KAIRO_STATUS_NOT_SUPPORTED, "more than 2^31-1 blocks");
  if (a->nbr > 0 && !a->row_ptr) return fail(KAIRO_STATUS_INVALID_VALUE, "null row_ptr");
  if (a->nnzb > 0 && !a->col_idx) return fail(KAIRO_STATUS_INVALID_VALUE, "null col_idx");
  return KAIRO_STATUS_SUCCESS;
}

}  // namespace
}  // namespace kairo

extern "C" kairo_status kairo_bsr_transpose_workspace_size(const kairo_bsr* a, size_t* bytes) {
  kairo_status st = check_transpose_args(a);
  if (st) return st;
  if (!bytes) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  *bytes = transpose_ws_bytes(a->nnzb, static_cast<int32_t>(ceil_div64(a->cols, a->bk)));
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_bsr_transpose(const kairo_bsr* a, int32_t* row_ptr_t, int32_t* col_idx_t,
                                            int32_t* perm_t, void* blocks_t, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  kairo_status st = check_transpose_args(a);
  if (st) return st;
  const int64_t nbc64 = ceil_div64(a->cols, a->bk);
  if (nbc64 > 0x7fffffffLL) return fail(KAIRO_STATUS_NOT_SUPPORTED, "too many block-columns");
  const int32_t nbc = static_cast<int32_t>(nbc64);
  if (!row_ptr_t || !workspace || (a->nnzb > 0 && (!col_idx_t || !perm_t)))
    return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  if (blocks_t && a->nnzb > 0 && !a->blocks) return fail(KAIRO_STATUS_INVALID_VALUE, "null blocks");
  if (workspace_bytes < transpose_ws_bytes(a->nnzb, nbc))
    return fail(KAIRO_STATUS_WORKSPACE_TOO_SMALL, "transpose workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // W^T order = W's positions bucketed by block-column, stable: the bucket
  // sort of keys col_idx[p], carrying each position's block-row.
  int32_t* rows_of_pos = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + bucket_sort_ws_bytes(nbc));
  if (a->nnzb > 0) {
    const int rows_grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((a->nbr + 7) / 8, 148 * 32)));
    k_expand_rows<<<rows_grid, 256, 0, s>>>(a->row_ptr, a->nbr, a->nnzb, rows_of_pos);
  }
  st = bucket_sort(a->col_idx, rows_of_pos, a->nbr, a->nnzb, nbc, row_ptr_t, perm_t, col_idx_t, workspace, s);
  if (st) return st;
  if (blocks_t) return transpose_values(a, perm_t, blocks_t, static_cast<unsigned*>(workspace), s);
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_bsr_transpose_values(const kairo_bsr* a, const int32_t* perm_t, void* blocks_t,
                                                   void* workspace, size_t workspace_bytes, void* stream) {
  kairo_status st = check_transpose_args(a);
  if (st) return st;
  if (a->nnzb == 0) return KAIRO_STATUS_SUCCESS;
  if (!perm_t || !blocks_t || !a->blocks || !workspace) return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  if (workspace_bytes < kWorkspaceHeaderBytes) return fail(KAIRO_STATUS_WORKSPACE_TOO_SMALL, "workspace too small");
  return transpose_values(a, perm_t, blocks_t, static_cast<unsigned*>(workspace), static_cast<cudaStream_t>(stream));
}
