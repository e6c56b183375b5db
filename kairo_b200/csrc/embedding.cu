// Masked embedding lookup and its gradient scatter: the reference's other
// CUDA path (csrc/sparse_embedding_kernel.cu, called from
// kairo/ops/sparse_embedding.py:59-160), rewritten for B200.
//
// gather   out[b, d] = weight[ids[b], d] if (ids[b], d) is active in the
//          mask, else 0; ids outside [0, N) give zero rows (as the
//          reference's kernel does).  One warp per id zeroes the output row
//          with wide stores, then writes the row's active values: O(D +
//          nnz_row) per id, where the reference's general kernel tests every
//          column against every active entry of the row (O(D * nnz_row)).
// scatter  grad_weight[r, :] = sum over b with batch_ids[b] == r of
//          grad_output[b, :] for every r in active_ids (sorted, unique), zero
//          elsewhere.  The reference gives every active row a CTA that scans
//          the whole batch (O(S * B)).  Here batch positions are bucketed by
//          their index in active_ids (binary search) with the device bucket
//          sort, and one warp per active row sums its gradient rows in
//          ascending batch order, so the result is deterministic and the
//          work is O(B log S + B * D).  A bucket too long to sort in shared
//          memory is summed by scanning the batch ids in order instead.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "internal.h"

namespace kairo {
namespace {

constexpr int kWarpsPerCta = 8;

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
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __half from_f<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <typename T>
__global__ void __launch_bounds__(kWarpsPerCta * 32) k_gather(const T* __restrict__ weight, int64_t n_rows,
                                                              int64_t dim, const int64_t* __restrict__ row_offsets,
                                                              const int64_t* __restrict__ mask_cols, int64_t nnz,
                                                              const int64_t* __restrict__ ids, int64_t nids,
                                                              T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarpsPerCta;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5); b < nids; b += warps) {
    T* orow = out + b * dim;
    const T zero = from_f<T>(0.f);
    for (int64_t d = lane; d < dim; d += 32) orow[d] = zero;
    __syncwarp();
    const int64_t row = ids[b];
    if (row < 0 || row >= n_rows) continue;
    const int64_t start = max(static_cast<int64_t>(0), row_offsets[row]);
    const int64_t end = min(nnz, row_offsets[row + 1]);
    const T* wrow = weight + row * dim;
    for (int64_t k = start + lane; k < end; k += 32) {
      const int64_t col = mask_cols[k];
      if (col >= 0 && col < dim) orow[col] = wrow[col];
    }
  }
}

// Row bitmask of a COO element mask: bit c % 32 of word c / 32 of row r is
// set when (r, c) is an entry.  Entries outside [0, n_rows) x [0, n_cols)
// are skipped.
__global__ void k_mask_bits(const int64_t* __restrict__ rows, const int64_t* __restrict__ cols, int64_t nnz,
                            int64_t n_rows, int64_t n_cols, int64_t words, uint32_t* __restrict__ bits) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nnz;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = rows[i], c = cols[i];
    if (r < 0 || r >= n_rows || c < 0 || c >= n_cols) continue;
    atomicOr(bits + r * words + (c >> 5), 1u << (c & 31));
  }
}

// Masked gather from the row bitmask.  A warp takes IDS ids at a time (one
// load by its first lanes) and then ROWS rows at once: each lane loads VEC
// consecutive columns of every row (16-byte vectors when rows are 16-byte
// aligned) and the mask word holding them, all in flight together, then
// stores the masked rows.  Every access is coalesced.  Large batches take 32
// ids per warp and 8 rows in flight; small ones 2 and 2, so that more warps
// share the batch (a sweep over batch shapes on B200 put both within a few
// percent of a device-to-device copy of the output's bytes).
constexpr int kSmallBatch = 16384;

template <int EB, int VEC>
struct GatherVec;
template <>
struct GatherVec<4, 4> {  // 4 x fp32
  using V = uint4;
  __device__ static V apply(V v, uint32_t m) {
    v.x = (m & 1u) ? v.x : 0u;
    v.y = (m & 2u) ? v.y : 0u;
    v.z = (m & 4u) ? v.z : 0u;
    v.w = (m & 8u) ? v.w : 0u;
    return v;
  }
};
template <>
struct GatherVec<2, 8> {  // 8 x 16-bit
  using V = uint4;
  __device__ static uint32_t pair(uint32_t w, uint32_t m2) {
    return w & (((m2 & 1u) ? 0x0000ffffu : 0u) | ((m2 & 2u) ? 0xffff0000u : 0u));
  }
  __device__ static V apply(V v, uint32_t m) {
    v.x = pair(v.x, m);
    v.y = pair(v.y, m >> 2);
    v.z = pair(v.z, m >> 4);
    v.w = pair(v.w, m >> 6);
    return v;
  }
};
template <>
struct GatherVec<4, 1> {
  using V = uint32_t;
  __device__ static V apply(V v, uint32_t m) { return (m & 1u) ? v : 0u; }
};
template <>
struct GatherVec<2, 1> {
  using V = uint16_t;
  __device__ static V apply(V v, uint32_t m) { return (m & 1u) ? v : static_cast<uint16_t>(0); }
};

template <int EB, int VEC, int IDS, int ROWS>
__global__ void __launch_bounds__(kWarpsPerCta * 32) k_gather_bits(const void* __restrict__ weight, int64_t n_rows,
                                                                   int64_t dim, const uint32_t* __restrict__ bits,
                                                                   int64_t words, const int64_t* __restrict__ ids,
                                                                   int64_t nids, void* __restrict__ out) {
  using G = GatherVec<EB, VEC>;
  using V = typename G::V;
  const V* w = static_cast<const V*>(weight);
  V* o = static_cast<V*>(out);
  const int64_t vdim = dim / VEC;  // vectors per row (dim is a multiple of VEC)
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarpsPerCta;
  for (int64_t b0 = (static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5)) * IDS; b0 < nids;
       b0 += warps * IDS) {
    long long mine = -1;  // lane l < IDS: row of id b0 + l, or -1 (missing / out of range)
    if (lane < IDS && b0 + lane < nids) {
      const int64_t r = ids[b0 + lane];
      mine = (r >= 0 && r < n_rows) ? r : -1;
    }
#pragma unroll 1
    for (int u0 = 0; u0 < IDS; u0 += ROWS) {
      const V* src[ROWS];         // weight row, or null for a zero row
      const uint32_t* mrow[ROWS];  // its mask words
#pragma unroll
      for (int u = 0; u < ROWS; ++u) {
        const long long r = __shfl_sync(0xffffffffu, mine, u0 + u);
        src[u] = r >= 0 ? w + r * vdim : nullptr;
        mrow[u] = bits + (r >= 0 ? r : 0) * words;
      }
      const int64_t nb = min(static_cast<int64_t>(ROWS), nids - (b0 + u0));  // rows to store
      V* dst = o + (b0 + u0) * vdim;
#pragma unroll 1
      for (int64_t v = lane; v < vdim; v += 32) {
        const int64_t c = v * VEC;  // first column of this lane's vector
        V val[ROWS];
        uint32_t m[ROWS];
#pragma unroll
        for (int u = 0; u < ROWS; ++u) {
          val[u] = src[u] ? src[u][v] : V{};
          m[u] = src[u] ? mrow[u][c >> 5] >> (c & 31) : 0u;
        }
#pragma unroll
        for (int u = 0; u < ROWS; ++u)
          if (u < nb) dst[u * vdim + v] = G::apply(val[u], m[u]);
      }
    }
  }
}

// Bucket of every batch position: the index of batch_ids[b] in the sorted
// active_ids, or nactive when it is not active.
__global__ void k_scatter_keys(const int64_t* __restrict__ active_ids, int64_t nactive,
                               const int64_t* __restrict__ batch_ids, int64_t nbatch, int32_t* __restrict__ keys) {
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nbatch;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t id = batch_ids[b];
    int64_t lo = 0, hi = nactive;  // first index with active_ids[index] >= id
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (active_ids[mid] < id) lo = mid + 1;
      else hi = mid;
    }
    keys[b] = static_cast<int32_t>((lo < nactive && active_ids[lo] == id) ? lo : nactive);
  }
}

// One warp per active row: the sum of its members' gradient rows in
// ascending batch order, written once (rows with no member stay zero).
template <typename T>
__global__ void __launch_bounds__(kWarpsPerCta * 32) k_scatter_sum(
    const T* __restrict__ grad, int64_t dim, const int64_t* __restrict__ active_ids, int64_t nactive, int64_t n_rows,
    const int32_t* __restrict__ bucket_ptr, const int32_t* __restrict__ members, const int32_t* __restrict__ keys,
    int64_t nbatch, T* __restrict__ grad_weight, unsigned* err) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarpsPerCta;
  for (int64_t a = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5); a < nactive; a += warps) {
    const int64_t row = active_ids[a];
    if (row < 0 || row >= n_rows) {
      if (lane == 0) atomicCAS(err, 0u, KAIRO_DEVERR_BAD_INDEX);
      continue;
    }
    const int p0 = bucket_ptr[a], p1 = bucket_ptr[a + 1];
    if (p1 <= p0) continue;
    const bool sorted = (p1 - p0) <= kBucketSortMax;
    for (int64_t d0 = 0; d0 < dim; d0 += 32 * 4) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (sorted) {
        for (int q = p0; q < p1; ++q) {
          const T* g = grad + static_cast<int64_t>(members[q]) * dim;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int64_t d = d0 + u * 32 + lane;
            if (d < dim) acc[u] += to_f(g[d]);
          }
        }
      } else {
        // Too long to have been sorted: walk the batch in order.
        for (int64_t b0 = 0; b0 < nbatch; b0 += 32) {
          const int64_t bl = b0 + lane;
          const bool mine = bl < nbatch && keys[bl] == static_cast<int32_t>(a);
          unsigned m = __ballot_sync(0xffffffffu, mine);
          while (m) {
            const int j = __ffs(m) - 1;
            m &= m - 1;
            const T* g = grad + (b0 + j) * dim;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int64_t d = d0 + u * 32 + lane;
              if (d < dim) acc[u] += to_f(g[d]);
            }
          }
        }
      }
      T* o = grad_weight + row * dim;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t d = d0 + u * 32 + lane;
        if (d < dim) o[d] = from_f<T>(acc[u]);
      }
    }
  }
}

// Mask rows/cols (int64) narrowed to the bucket sort's int32 keys and
// values; ids outside int32 become -1, which the sort reports as a bad index.
__global__ void k_narrow_coo(const int64_t* __restrict__ rows, const int64_t* __restrict__ cols, int64_t nnz,
                             int32_t* __restrict__ rows32, int32_t* __restrict__ cols32) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nnz;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = rows[i], c = cols[i];
    rows32[i] = (r >= 0 && r <= 0x7fffffffLL) ? static_cast<int32_t>(r) : -1;
    cols32[i] = (c >= 0 && c <= 0x7fffffffLL) ? static_cast<int32_t>(c) : -1;
  }
}

// row_offsets (int64) from the bucket pointers; sorted rows, cols and the
// permutation (int64) from the sort's permutation.
__global__ void k_widen_sorted(const int32_t* __restrict__ bucket_ptr, int64_t n_rows, const int32_t* __restrict__ perm,
                               const int64_t* __restrict__ rows, const int64_t* __restrict__ cols, int64_t nnz,
                               int64_t* __restrict__ row_offsets, int64_t* __restrict__ rows_sorted,
                               int64_t* __restrict__ cols_sorted, int64_t* __restrict__ perm64,
                               const unsigned* __restrict__ err) {
  if (*err) return;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  for (int64_t i = t0; i <= n_rows; i += stride) row_offsets[i] = bucket_ptr[i];
  for (int64_t p = t0; p < nnz; p += stride) {
    const int32_t src = perm[p];
    if (rows_sorted) rows_sorted[p] = rows[src];
    cols_sorted[p] = cols[src];
    if (perm64) perm64[p] = src;
  }
}

// Workspace of the mask row sort: the bucket sort's, then rows32, cols32,
// perm and the sorted cols32 (nnz int32 each) and the bucket pointers.
size_t coo_sort_ws_bytes(int64_t n_rows, int64_t nnz) {
  const size_t col = align_up(static_cast<size_t>(nnz), 64) * sizeof(int32_t);
  return bucket_sort_ws_bytes(static_cast<int32_t>(n_rows)) + 4 * col +
         align_up(static_cast<size_t>(n_rows + 1), 64) * sizeof(int32_t);
}

size_t dtype_bytes(kairo_dtype d) { return d == KAIRO_DTYPE_F32 ? 4 : 2; }

int warp_grid(int64_t items) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((items + kWarpsPerCta - 1) / kWarpsPerCta, 148 * 32)));
}

// Scatter workspace: the bucket sort's, then keys, members and a spare copy
// of the keys in bucket order (nbatch int32 each).
size_t scatter_ws_bytes(int64_t nactive, int64_t nbatch) {
  const size_t col = align_up(static_cast<size_t>(nbatch), 64) * sizeof(int32_t);
  return bucket_sort_ws_bytes(static_cast<int32_t>(nactive + 1)) + align_up(static_cast<size_t>(nactive + 2), 64) *
         sizeof(int32_t) + 3 * col;
}

}  // namespace
}  // namespace kairo

using namespace kairo;

extern "C" kairo_status kairo_sparse_gather(const void* weight, int64_t n_rows, int64_t dim, kairo_dtype dtype,
                                            const int64_t* row_offsets, const int64_t* mask_cols, int64_t nnz,
                                            const int64_t* ids, int64_t nids, void* out, void* stream) {
  if (n_rows < 0 || dim <= 0 || nnz < 0 || nids < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid size");
  if (nids == 0) return KAIRO_STATUS_SUCCESS;
  if (!weight || !row_offsets || !ids || !out || (nnz > 0 && !mask_cols))
    return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int g = warp_grid(nids);
  switch (dtype) {
    case KAIRO_DTYPE_F32:
      k_gather<float><<<g, kWarpsPerCta * 32, 0, s>>>(static_cast<const float*>(weight), n_rows, dim, row_offsets,
                                                      mask_cols, nnz, ids, nids, static_cast<float*>(out));
      break;
    case KAIRO_DTYPE_F16:
      k_gather<__half><<<g, kWarpsPerCta * 32, 0, s>>>(static_cast<const __half*>(weight), n_rows, dim, row_offsets,
                                                       mask_cols, nnz, ids, nids, static_cast<__half*>(out));
      break;
    case KAIRO_DTYPE_BF16:
      k_gather<__nv_bfloat16><<<g, kWarpsPerCta * 32, 0, s>>>(static_cast<const __nv_bfloat16*>(weight), n_rows, dim,
                                                              row_offsets, mask_cols, nnz, ids, nids,
                                                              static_cast<__nv_bfloat16*>(out));
      break;
    default:
      return fail(KAIRO_STATUS_INVALID_VALUE, "unknown dtype");
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the sparse gather kernel");
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_sparse_scatter_grad_workspace_size(int64_t nactive, int64_t nbatch, size_t* bytes) {
  if (!bytes || nactive < 0 || nbatch < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid argument");
  *bytes = scatter_ws_bytes(nactive, nbatch);
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_sparse_scatter_grad(const void* grad_output, kairo_dtype dtype,
                                                  const int64_t* active_ids, int64_t nactive,
                                                  const int64_t* batch_ids, int64_t nbatch, int64_t n_rows,
                                                  int64_t dim, void* grad_weight, void* workspace,
                                                  size_t workspace_bytes, void* stream) {
  if (n_rows <= 0 || dim <= 0 || nactive < 0 || nbatch < 0)
    return fail(KAIRO_STATUS_INVALID_VALUE, "N and D must be positive");
  if (nactive >= 0x7fffffffLL || nbatch > 0x7fffffffLL) return fail(KAIRO_STATUS_NOT_SUPPORTED, "too many ids");
  if (dtype != KAIRO_DTYPE_F32 && dtype != KAIRO_DTYPE_F16 && dtype != KAIRO_DTYPE_BF16)
    return fail(KAIRO_STATUS_INVALID_VALUE, "unknown dtype");
  if (!grad_weight) return fail(KAIRO_STATUS_INVALID_VALUE, "null grad_weight");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(grad_weight, 0, static_cast<size_t>(n_rows) * dim * dtype_bytes(dtype), s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(grad_weight)");
  if (nactive == 0 || nbatch == 0) return KAIRO_STATUS_SUCCESS;
  if (!grad_output || !active_ids || !batch_ids || !workspace)
    return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  if (workspace_bytes < scatter_ws_bytes(nactive, nbatch))
    return fail(KAIRO_STATUS_WORKSPACE_TOO_SMALL, "scatter workspace too small");
  const int32_t nb = static_cast<int32_t>(nactive + 1);  // last bucket: inactive positions
  uint8_t* p = static_cast<uint8_t*>(workspace) + bucket_sort_ws_bytes(nb);
  int32_t* bucket_ptr = reinterpret_cast<int32_t*>(p);
  p += align_up(static_cast<size_t>(nactive + 2), 64) * sizeof(int32_t);
  const size_t col = align_up(static_cast<size_t>(nbatch), 64) * sizeof(int32_t);
  int32_t* keys = reinterpret_cast<int32_t*>(p);
  int32_t* members = reinterpret_cast<int32_t*>(p + col);
  int32_t* keys_sorted = reinterpret_cast<int32_t*>(p + 2 * col);
  k_scatter_keys<<<std::max(1, static_cast<int>(std::min<int64_t>((nbatch + 255) / 256, 148 * 16))), 256, 0, s>>>(
      active_ids, nactive, batch_ids, nbatch, keys);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the scatter key kernel");
  kairo_status st = bucket_sort(keys, keys, nb, nbatch, nb, bucket_ptr, members, keys_sorted, workspace, s,
                                /*long_buckets_ok=*/true);
  if (st) return st;
  unsigned* err = static_cast<unsigned*>(workspace);
  const int g = warp_grid(nactive);
  switch (dtype) {
    case KAIRO_DTYPE_F32:
      k_scatter_sum<float><<<g, kWarpsPerCta * 32, 0, s>>>(static_cast<const float*>(grad_output), dim, active_ids,
                                                           nactive, n_rows, bucket_ptr, members, keys, nbatch,
                                                           static_cast<float*>(grad_weight), err);
      break;
    case KAIRO_DTYPE_F16:
      k_scatter_sum<__half><<<g, kWarpsPerCta * 32, 0, s>>>(static_cast<const __half*>(grad_output), dim, active_ids,
                                                            nactive, n_rows, bucket_ptr, members, keys, nbatch,
                                                            static_cast<__half*>(grad_weight), err);
      break;
    default:
      k_scatter_sum<__nv_bfloat16><<<g, kWarpsPerCta * 32, 0, s>>>(
          static_cast<const __nv_bfloat16*>(grad_output), dim, active_ids, nactive, n_rows, bucket_ptr, members, keys,
          nbatch, static_cast<__nv_bfloat16*>(grad_weight), err);
      break;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the scatter sum kernel");
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_coo_sort_rows_workspace_size(int64_t n_rows, int64_t nnz, size_t* bytes) {
  if (!bytes || n_rows < 0 || nnz < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid argument");
  if (n_rows >= 0x7fffffffLL || nnz >= 0x7fffffffLL) return fail(KAIRO_STATUS_NOT_SUPPORTED, "mask too large");
  *bytes = coo_sort_ws_bytes(n_rows, nnz);
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_coo_sort_rows(const int64_t* rows, const int64_t* cols, int64_t nnz, int64_t n_rows,
                                            int64_t n_cols, int64_t* row_offsets, int64_t* rows_sorted,
                                            int64_t* cols_sorted, int64_t* perm, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  if (n_rows < 0 || n_cols < 0 || nnz < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid size");
  if (n_rows >= 0x7fffffffLL || n_cols >= 0x7fffffffLL || nnz >= 0x7fffffffLL)
    return fail(KAIRO_STATUS_NOT_SUPPORTED, "mask too large");
  if (!row_offsets || !workspace || (nnz > 0 && (!rows || !cols || !cols_sorted)))
    return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  if (workspace_bytes < coo_sort_ws_bytes(n_rows, nnz))
    return fail(KAIRO_STATUS_WORKSPACE_TOO_SMALL, "mask sort workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int32_t nb = static_cast<int32_t>(n_rows);
  uint8_t* p = static_cast<uint8_t*>(workspace) + bucket_sort_ws_bytes(nb);
  const size_t col = align_up(static_cast<size_t>(nnz), 64) * sizeof(int32_t);
  int32_t* rows32 = reinterpret_cast<int32_t*>(p);
  int32_t* cols32 = reinterpret_cast<int32_t*>(p + col);
  int32_t* perm32 = reinterpret_cast<int32_t*>(p + 2 * col);
  int32_t* cols32_sorted = reinterpret_cast<int32_t*>(p + 3 * col);
  int32_t* bucket_ptr = reinterpret_cast<int32_t*>(p + 4 * col);
  const int g = std::max(1, static_cast<int>(std::min<int64_t>((std::max(nnz, n_rows + 1) + 255) / 256, 148 * 16)));
  if (nnz > 0) k_narrow_coo<<<g, 256, 0, s>>>(rows, cols, nnz, rows32, cols32);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the mask narrowing kernel");
  // Rows longer than the shared-memory sort keep their scatter order: the
  // gather's result does not depend on the order of a row's entries.
  kairo_status st = bucket_sort(rows32, cols32, static_cast<int32_t>(n_cols), nnz, nb, bucket_ptr, perm32,
                                cols32_sorted, workspace, s, /*long_buckets_ok=*/true);
  if (st) return st;
  k_widen_sorted<<<g, 256, 0, s>>>(bucket_ptr, n_rows, perm32, rows, cols, nnz, row_offsets, rows_sorted,
                                   cols_sorted, perm, static_cast<const unsigned*>(workspace));
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the mask widening kernel");
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_mask_bits(const int64_t* rows, const int64_t* cols, int64_t nnz, int64_t n_rows,
                                        int64_t n_cols, uint32_t* bits, void* stream) {
  if (n_rows < 0 || n_cols < 0 || nnz < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid size");
  if (!bits && n_rows > 0 && n_cols > 0) return fail(KAIRO_STATUS_INVALID_VALUE, "null bits");
  if (nnz > 0 && (!rows || !cols)) return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t words = (n_cols + 31) / 32;
  if (n_rows > 0 && words > 0) {
    cudaError_t e = cudaMemsetAsync(bits, 0, static_cast<size_t>(n_rows) * words * sizeof(uint32_t), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(mask bits)");
  }
  if (nnz > 0) {
    const int g = std::max(1, static_cast<int>(std::min<int64_t>((nnz + 255) / 256, 148 * 16)));
    k_mask_bits<<<g, 256, 0, s>>>(rows, cols, nnz, n_rows, n_cols, words, bits);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the mask bits kernel");
  return KAIRO_STATUS_SUCCESS;
}

extern "C" kairo_status kairo_sparse_gather_bits(const void* weight, int64_t n_rows, int64_t dim, kairo_dtype dtype,
                                                 const uint32_t* bits, const int64_t* ids, int64_t nids, void* out,
                                                 void* stream) {
  if (n_rows < 0 || dim <= 0 || nids < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid size");
  if (dtype != KAIRO_DTYPE_F32 && dtype != KAIRO_DTYPE_F16 && dtype != KAIRO_DTYPE_BF16)
    return fail(KAIRO_STATUS_INVALID_VALUE, "unknown dtype");
  if (nids == 0) return KAIRO_STATUS_SUCCESS;
  if (!weight || !bits || !ids || !out) return fail(KAIRO_STATUS_INVALID_VALUE, "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int eb = static_cast<int>(dtype_bytes(dtype));
  const int64_t words = (dim + 31) / 32;
  const bool vec = (dim * eb) % 16 == 0 && reinterpret_cast<uintptr_t>(weight) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0;
  if (nids < kSmallBatch) {
    const int g = warp_grid((nids + 1) / 2);
    if (eb == 4) {
      if (vec) k_gather_bits<4, 4, 2, 2><<<g, kWarpsPerCta * 32, 0, s>>>(weight, n_rows, dim, bits, words, ids, nids, out);
      else k_gather_bits<4, 1, 2, 2><<<g, kWarpsPerCta * 32, 0, s>>>(weight, n_rows, dim, bits, words, ids, nids, out);
    } else {
      if (vec) k_gather_bits<2, 8, 2, 2><<<g, kWarpsPerCta * 32, 0, s>>>(weight, n_rows, dim, bits, words, ids, nids, out);
      else k_gather_bits<2, 1, 2, 2><<<g, kWarpsPerCta * 32, 0, s>>>(weight, n_rows, dim, bits, words, ids, nids, out);
    }
  } else {
    const int g = warp_grid((nids + 31) / 32);
    if (eb == 4) {
      if (vec) k_gather_bits<4, 4, 32, 8><<<g, kWarpsPerCta * 32, 0, s>>>(weight, n_rows, dim, bits, words, ids, nids, out);
      else k_gather_bits<4, 1, 32, 8><<<g, kWarpsPerCta * 32, 0, s>>>(weight, n_rows, dim, bits, words, ids, nids, out);
    } else {
      if (vec) k_gather_bits<2, 8, 32, 8><<<g, kWarpsPerCta * 32, 0, s>>>(weight, n_rows, dim, bits, words, ids, nids, out);
      else k_gather_bits<2, 1, 32, 8><<<g, kWarpsPerCta * 32, 0, s>>>(weight, n_rows, dim, bits, words, ids, nids, out);
    }
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the sparse gather kernel");
  return KAIRO_STATUS_SUCCESS;
}
