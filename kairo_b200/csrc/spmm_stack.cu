// Row groups for the tcgen05 BSR SpMM (kairo_bsr_stack_build,
// kairo_bsr_spmm_stacked).
//
// On a skewed mask a few block-rows hold most blocks, and long rows share
// most of their columns.  Ordering the block-rows by length and taking them
// R at a time, the blocks of one group in one column-block need one B panel
// between them and, for group rows that are consecutive, one MMA: the stacked
// blocks form a K-major operand of (run * bm) rows, multiplied into
// consecutive accumulator columns (spmm_tc_kernel.cuh, RG > 1).  On the
// 65536^2 Zipf(1.1) mask with 16x16 blocks, R = 4 leaves 0.32 stacked blocks
// per block and 0.35x the MMA cycles.
//
// The group structure is built on the device by four small kernels:
//   order  one CTA: a bitonic sort of (length desc, row asc) -> row_map;
//   count  one CTA per group: a bitmask per column-block (bit r = group row
//          r has a block there) in shared memory; its nonzero columns;
//   scan   one CTA: exclusive sum of the counts -> group_ptr;
//   fill   one CTA per group: the bitmask again, its nonzero columns written
//          in ascending order (super_col, super_mask), then every block's
//          stored index at (its column's stacked block, its group row).
#include <algorithm>
#include <sstream>

#include "spmm_tc_kernel.cuh"

namespace kairo {
namespace {

constexpr int kStackMaxRows = 16384;  // block-rows (sort keys in shared memory)
constexpr int kStackMaxCols = 16384;  // block-columns (two int32 tables in shared memory)
constexpr unsigned kStackBadIndex = 1u;
constexpr unsigned kStackDuplicate = 2u;
constexpr unsigned kStackBadRowPtr = 4u;

__global__ void __launch_bounds__(1024) k_stack_order(const int32_t* __restrict__ row_ptr, int nbr, int rg,
                                                      int ngroups, int32_t* __restrict__ row_map,
                                                      unsigned* flags) {
  extern __shared__ unsigned long long keys[];
  int n2 = 1;
  while (n2 < nbr) n2 <<= 1;
  for (int i = threadIdx.x; i < n2; i += blockDim.x) {
    unsigned long long k = ~0ull;
    if (i < nbr) {
      int len = row_ptr[i + 1] - row_ptr[i];
      if (len < 0) {
        atomicOr(flags, kStackBadRowPtr);
        len = 0;
      }
      k = (static_cast<unsigned long long>(0x7fffffffu - static_cast<unsigned>(len)) << 32) |
          static_cast<unsigned>(i);
    }
    keys[i] = k;
  }
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const bool up = (i & k) == 0;
          const unsigned long long a = keys[i], b = keys[ixj];
          if ((a > b) == up) {
            keys[i] = b;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int s = threadIdx.x; s < ngroups * rg; s += blockDim.x)
    row_map[s] = s < nbr ? static_cast<int32_t>(keys[s] & 0xffffffffu) : -1;
}

// Bitmask of one group per column-block into mask[nbc] (bit r: group row r
// has a block there); flags out-of-range columns and repeated columns.
__device__ void stack_group_mask(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx, int nbc,
                                 int rg, const int32_t* __restrict__ rows, unsigned* mask, unsigned* flags) {
  for (int c = threadIdx.x; c < nbc; c += blockDim.x) mask[c] = 0u;
  __syncthreads();
  for (int r = 0; r < rg; ++r) {
    const int row = rows[r];
    if (row < 0) continue;
    const int p0 = row_ptr[row], p1 = row_ptr[row + 1];
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
      const int c = col_idx[p];
      if (static_cast<unsigned>(c) >= static_cast<unsigned>(nbc)) {
        atomicOr(flags, kStackBadIndex);
        continue;
      }
      const unsigned old = atomicOr(&mask[c], 1u << r);
      if (old & (1u << r)) atomicOr(flags, kStackDuplicate);
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(512) k_stack_count(const int32_t* __restrict__ row_ptr,
                                                     const int32_t* __restrict__ col_idx, int nbc, int rg,
                                                     const int32_t* __restrict__ row_map,
                                                     int32_t* __restrict__ counts, unsigned* flags) {
  extern __shared__ unsigned mask[];
  const int g = blockIdx.x;
  stack_group_mask(row_ptr, col_idx, nbc, rg, row_map + static_cast<int64_t>(g) * rg, mask, flags);
  int cnt = 0;
  for (int c0 = 0; c0 < nbc; c0 += blockDim.x) {
    const int c = c0 + threadIdx.x;
    cnt += __syncthreads_count(c < nbc && mask[c] != 0u);
  }
  if (threadIdx.x == 0) counts[g] = cnt;
}

__global__ void k_stack_scan(const int32_t* __restrict__ counts, int ngroups, int32_t* __restrict__ group_ptr) {
  if (threadIdx.x != 0) return;
  int32_t acc = 0;
  group_ptr[0] = 0;
  for (int g = 0; g < ngroups; ++g) {
    acc += counts[g];
    group_ptr[g + 1] = acc;
  }
}

__global__ void __launch_bounds__(512) k_stack_fill(const int32_t* __restrict__ row_ptr,
                                                    const int32_t* __restrict__ col_idx,
                                                    const int32_t* __restrict__ blk_idx, int nbc, int rg,
                                                    const int32_t* __restrict__ row_map,
                                                    const int32_t* __restrict__ group_ptr,
                                                    int32_t* __restrict__ super_col, int32_t* __restrict__ super_mask,
                                                    int32_t* __restrict__ super_blk, unsigned* flags) {
  extern __shared__ unsigned smem_u[];
  unsigned* mask = smem_u;
  int32_t* pos = reinterpret_cast<int32_t*>(smem_u + nbc);
  __shared__ int part[512];
  const int g = blockIdx.x;
  const int32_t* rows = row_map + static_cast<int64_t>(g) * rg;
  stack_group_mask(row_ptr, col_idx, nbc, rg, rows, mask, flags);
  // Ordered compaction of the nonzero columns: thread t owns a contiguous
  // run of columns; a serial scan of the per-thread counts gives offsets.
  const int per = (nbc + blockDim.x - 1) / blockDim.x;
  const int c_lo = min(nbc, static_cast<int>(threadIdx.x) * per), c_hi = min(nbc, c_lo + per);
  int cnt = 0;
  for (int c = c_lo; c < c_hi; ++c) cnt += mask[c] != 0u;
  part[threadIdx.x] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int t = 0; t < static_cast<int>(blockDim.x); ++t) {
      const int v = part[t];
      part[t] = acc;
      acc += v;
    }
  }
  __syncthreads();
  int q = group_ptr[g] + part[threadIdx.x];
  for (int c = c_lo; c < c_hi; ++c) {
    const unsigned m = mask[c];
    if (m) {
      super_col[q] = c;
      super_mask[q] = static_cast<int32_t>(m);
      pos[c] = q;
      ++q;
    }
  }
  __syncthreads();
  for (int r = 0; r < rg; ++r) {
    const int row = rows[r];
    if (row < 0) continue;
    const int p0 = row_ptr[row], p1 = row_ptr[row + 1];
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
      const int c = col_idx[p];
      if (static_cast<unsigned>(c) >= static_cast<unsigned>(nbc)) continue;
      super_blk[static_cast<int64_t>(pos[c]) * rg + r] = blk_idx ? blk_idx[p] : p;
    }
  }
}

struct StackLayout {
  int ngroups;
  size_t row_map, counts, group_ptr, super_col, super_mask, super_blk, flags, total;
};

size_t al256(size_t v) { return (v + 255) / 256 * 256; }

kairo_status stack_layout(const kairo_bsr* a, int rg, StackLayout* out) {
  if (!a || !out) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  if (rg != 2 && rg != 4 && rg != 8) return fail(KAIRO_STATUS_INVALID_VALUE, "rows_per_group must be 2, 4 or 8");
  if (a->nbr < 0 || a->nnzb < 0 || a->bk <= 0) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid BSR descriptor");
  if (a->nbr > kStackMaxRows) return fail(KAIRO_STATUS_NOT_SUPPORTED, "row groups support at most 16384 block-rows");
  if (ceil_div64(a->cols, a->bk) > kStackMaxCols)
    return fail(KAIRO_STATUS_NOT_SUPPORTED, "row groups support at most 16384 block-columns");
  StackLayout L{};
  L.ngroups = static_cast<int>(ceil_div64(a->nbr, rg));
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = al256(off + bytes);
    return at;
  };
  L.row_map = take(static_cast<size_t>(L.ngroups) * rg * 4);
  L.counts = take(static_cast<size_t>(L.ngroups) * 4);
  L.group_ptr = take(static_cast<size_t>(L.ngroups + 1) * 4);
  L.super_col = take(static_cast<size_t>(a->nnzb) * 4);
  L.super_mask = take(static_cast<size_t>(a->nnzb) * 4);
  L.super_blk = take(static_cast<size_t>(a->nnzb) * rg * 4);
  L.flags = take(4);
  L.total = off;
  *out = L;
  return KAIRO_STATUS_SUCCESS;
}

using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, TcArgs);

template <int BM, int NT, int IN_FMT, int RG>
KernelFn pick_rg4() {
  return reinterpret_cast<KernelFn>(&bsr_spmm_tc_kernel<BM, BM, NT, false, IN_FMT, float, RG>);
}

template <int IN_FMT>
KernelFn pick_rg(int bm, int nt, int rg) {
#define KAIRO_RG_CASE(B, T, R) \
  if (bm == B && nt == T && rg == R) return pick_rg4<B, T, IN_FMT, R>();
  KAIRO_RG_CASE(16, 1, 2)
  KAIRO_RG_CASE(16, 1, 4)
  KAIRO_RG_CASE(16, 1, 8)
  KAIRO_RG_CASE(16, 2, 2)
  KAIRO_RG_CASE(16, 2, 4)
  KAIRO_RG_CASE(32, 1, 2)
  KAIRO_RG_CASE(32, 1, 4)
  KAIRO_RG_CASE(32, 2, 2)
#undef KAIRO_RG_CASE
  return nullptr;
}

// The group descriptor as the kernel's BSR view: groups are its rows and
// stacked blocks its blocks (blk_idx carries the row masks).
kairo_bsr group_view(const kairo_bsr* a, const kairo_bsr_stack* s) {
  kairo_bsr v = *a;
  v.nbr = s->ngroups;
  v.nnzb = s->nsuper;
  v.row_ptr = s->group_ptr;
  v.col_idx = s->super_col;
  v.blk_idx = s->super_mask;
  return v;
}

struct StackChoice {
  bool nothing = false, zero = false;
  TcPlan plan{};
};

kairo_status stack_choose(const kairo_bsr* a, const kairo_bsr_stack* s, const void* b, int64_t ldb, int64_t n,
                          const void* c, int64_t ldc, const kairo_spmm_config* cfg, StackChoice* out) {
  if (!a || !s) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  const int rg = s->rows_per_group;
  if (rg != 2 && rg != 4 && rg != 8) return fail(KAIRO_STATUS_INVALID_VALUE, "rows_per_group must be 2, 4 or 8");
  if (a->nbr < 0 || a->bm <= 0 || a->nbr != ceil_div64(a->rows, a->bm))
    return fail(KAIRO_STATUS_INVALID_VALUE, "invalid BSR descriptor");
  if (s->ngroups != ceil_div64(a->nbr, rg)) return fail(KAIRO_STATUS_INVALID_VALUE, "group count does not match the BSR");
  if (s->nsuper < 0 || s->nsuper > a->nnzb) return fail(KAIRO_STATUS_INVALID_VALUE, "stacked block count out of range");
  if (n < 0 || ldb < n || ldc < n) return fail(KAIRO_STATUS_INVALID_VALUE, "negative N or leading dimension below N");
  StackChoice ch;
  if (a->rows == 0 || n == 0) {
    ch.nothing = true;
    *out = ch;
    return KAIRO_STATUS_SUCCESS;
  }
  if (!c) return fail(KAIRO_STATUS_INVALID_VALUE, "null C");
  if (a->nnzb == 0) {
    ch.zero = true;
    *out = ch;
    return KAIRO_STATUS_SUCCESS;
  }
  if (!b || !s->group_ptr || !s->super_col || !s->super_mask || !s->super_blk || !s->row_map)
    return fail(KAIRO_STATUS_INVALID_VALUE, "null operand or group table");
  std::string why;
  if (!tc_supported(a, KAIRO_LAYOUT_STANDARD, n, ldb, ldc, KAIRO_DTYPE_F32, b, c, &why))
    return fail(KAIRO_STATUS_NOT_SUPPORTED, why);
  if (a->bm > 32) return fail(KAIRO_STATUS_NOT_SUPPORTED, "row groups take blocks of 16 or 32");
  kairo_spmm_config cf = cfg ? *cfg : kairo_spmm_config{};
  if (cf.kernel != KAIRO_KERNEL_AUTO && cf.kernel != KAIRO_KERNEL_TCGEN05)
    return fail(KAIRO_STATUS_INVALID_VALUE, "row groups run on the tcgen05 kernel");
  if (cf.n_tile == 0) cf.n_tile = (n > 128 && rg * a->bm * 2 <= 128) ? 256 : 128;
  if (cf.n_tile != 128 && cf.n_tile != 256) return fail(KAIRO_STATUS_INVALID_VALUE, "n_tile must be 128 or 256");
  if (rg * a->bm * (cf.n_tile / 128) > 128)
    return fail(KAIRO_STATUS_NOT_SUPPORTED, "rows_per_group * bm * n_tile / 128 exceeds 128");
  const kairo_bsr v = group_view(a, s);
  kairo_status st = tc_plan(&v, KAIRO_LAYOUT_STANDARD, n, &cf, current_device(), &ch.plan, rg);
  if (st) return st;
  *out = ch;
  return KAIRO_STATUS_SUCCESS;
}

// The choice kairo_bsr_spmm_stacked would make, with aligned stand-in operands.
kairo_status stack_probe(const kairo_bsr* a, const kairo_bsr_stack* s, int64_t n, const kairo_spmm_config* cfg,
                         StackChoice* ch) {
  static const uint8_t dummy[16] __attribute__((aligned(16))) = {0};
  if (!a || !s) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  kairo_bsr probe = *a;
  if (!probe.blocks) probe.blocks = dummy;
  kairo_bsr_stack ps = *s;
  const int32_t* d32 = reinterpret_cast<const int32_t*>(dummy);
  if (!ps.group_ptr) ps.group_ptr = d32;
  if (!ps.super_col) ps.super_col = d32;
  if (!ps.super_mask) ps.super_mask = d32;
  if (!ps.super_blk) ps.super_blk = d32;
  if (!ps.row_map) ps.row_map = d32;
  return stack_choose(&probe, &ps, dummy, ((n + 7) / 8) * 8, n, dummy, n, cfg, ch);
}

}  // namespace
}  // namespace kairo

using namespace kairo;

extern "C" {

kairo_status kairo_bsr_stack_size(const kairo_bsr* a, int32_t rows_per_group, size_t* bytes) {
  if (!bytes) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  StackLayout L;
  kairo_status st = stack_layout(a, rows_per_group, &L);
  if (st) return st;
  *bytes = L.total;
  return KAIRO_STATUS_SUCCESS;
}

kairo_status kairo_bsr_stack_build(const kairo_bsr* a, int32_t rows_per_group, void* mem, size_t mem_bytes,
                                   kairo_bsr_stack* out, void* stream) {
  if (!out) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  StackLayout L;
  kairo_status st = stack_layout(a, rows_per_group, &L);
  if (st) return st;
  if (!mem) return fail(KAIRO_STATUS_INVALID_VALUE, "null group memory");
  if (mem_bytes < L.total) return fail(KAIRO_STATUS_WORKSPACE_TOO_SMALL, "group memory smaller than kairo_bsr_stack_size");
  if (a->nbr > 0 && !a->row_ptr) return fail(KAIRO_STATUS_INVALID_VALUE, "null row_ptr");
  if (a->nnzb > 0 && !a->col_idx) return fail(KAIRO_STATUS_INVALID_VALUE, "null col_idx");
  const int rg = rows_per_group;
  uint8_t* m = static_cast<uint8_t*>(mem);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t* row_map = reinterpret_cast<int32_t*>(m + L.row_map);
  int32_t* counts = reinterpret_cast<int32_t*>(m + L.counts);
  int32_t* group_ptr = reinterpret_cast<int32_t*>(m + L.group_ptr);
  int32_t* super_col = reinterpret_cast<int32_t*>(m + L.super_col);
  int32_t* super_mask = reinterpret_cast<int32_t*>(m + L.super_mask);
  int32_t* super_blk = reinterpret_cast<int32_t*>(m + L.super_blk);
  unsigned* flags = reinterpret_cast<unsigned*>(m + L.flags);
  const int nbc = static_cast<int>(ceil_div64(a->cols, a->bk));
  cudaError_t e = cudaMemsetAsync(flags, 0, sizeof(unsigned), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(group_ptr, 0, sizeof(int32_t), s);
  if (e == cudaSuccess && a->nbr > 0) {
    int n2 = 1;
    while (n2 < a->nbr) n2 <<= 1;
    const size_t sort_smem = static_cast<size_t>(n2) * 8;
    const size_t col_smem = static_cast<size_t>(std::max(nbc, 1)) * 8;
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&k_stack_order), cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sort_smem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&k_stack_fill),
                               cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(col_smem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&k_stack_count),
                               cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(col_smem / 2));
    if (e == cudaSuccess) {
      k_stack_order<<<1, 1024, sort_smem, s>>>(a->row_ptr, a->nbr, rg, L.ngroups, row_map, flags);
      k_stack_count<<<L.ngroups, 512, col_smem / 2, s>>>(a->row_ptr, a->col_idx, nbc, rg, row_map, counts, flags);
      k_stack_scan<<<1, 32, 0, s>>>(counts, L.ngroups, group_ptr);
      k_stack_fill<<<L.ngroups, 512, col_smem, s>>>(a->row_ptr, a->col_idx, a->blk_idx, nbc, rg, row_map, group_ptr,
                                                    super_col, super_mask, super_blk, flags);
      e = cudaGetLastError();
    }
  }
  int32_t nsuper = 0;
  unsigned fl = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&nsuper, group_ptr + L.ngroups, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&fl, flags, sizeof(unsigned), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "building row groups");
  if (fl & (kStackBadIndex | kStackBadRowPtr))
    return fail(KAIRO_STATUS_INVALID_VALUE, "row groups: a column index or row pointer is out of range");
  if (fl & kStackDuplicate)
    return fail(KAIRO_STATUS_NOT_SUPPORTED, "row groups: a block-row holds two blocks in one column");
  kairo_bsr_stack r{};
  r.rows_per_group = rg;
  r.ngroups = L.ngroups;
  r.nsuper = nsuper;
  r.group_ptr = group_ptr;
  r.super_col = super_col;
  r.super_mask = super_mask;
  r.super_blk = super_blk;
  r.row_map = row_map;
  *out = r;
  return KAIRO_STATUS_SUCCESS;
}

kairo_status kairo_bsr_spmm_stacked_workspace_size(const kairo_bsr* a, const kairo_bsr_stack* s, int64_t n,
                                                   const kairo_spmm_config* cfg, size_t* bytes) {
  if (!bytes) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  StackChoice ch;
  kairo_status st = stack_probe(a, s, n, cfg, &ch);
  if (st) return st;
  *bytes = (ch.nothing || ch.zero) ? kWorkspaceHeaderBytes + kCounterRegionBytes : ch.plan.workspace_bytes;
  return KAIRO_STATUS_SUCCESS;
}

kairo_status kairo_bsr_spmm_stacked_describe(const kairo_bsr* a, const kairo_bsr_stack* s, int64_t n,
                                             const kairo_spmm_config* cfg, kairo_spmm_plan* out) {
  if (!out) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  StackChoice ch;
  kairo_status st = stack_probe(a, s, n, cfg, &ch);
  if (st) return st;
  kairo_spmm_plan p{};
  p.workspace_bytes = (ch.nothing || ch.zero) ? kWorkspaceHeaderBytes + kCounterRegionBytes : ch.plan.workspace_bytes;
  if (ch.zero) p.launches = 1;
  if (!ch.nothing && !ch.zero) {
    p.kernel = KAIRO_KERNEL_TCGEN05;
    p.schedule = KAIRO_SCHEDULE_GROUPS;
    p.launches = 1;
    p.grid = ch.plan.grid;
    p.n_tile = 128 * ch.plan.nt;
    p.stages = ch.plan.stages;
    p.group_blocks = ch.plan.group;
    p.rows = ch.plan.rg;
  }
  *out = p;
  return KAIRO_STATUS_SUCCESS;
}

kairo_status kairo_bsr_spmm_stacked(const kairo_bsr* a, const kairo_bsr_stack* s, const void* b, int64_t ldb,
                                    int64_t n, void* c, int64_t ldc, const kairo_spmm_config* cfg, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  StackChoice ch;
  kairo_status st = stack_choose(a, s, b, ldb, n, c, ldc, cfg, &ch);
  if (st) return st;
  cudaStream_t strm = static_cast<cudaStream_t>(stream);
  if (ch.nothing) return KAIRO_STATUS_SUCCESS;
  if (ch.zero) {
    cudaError_t e = cudaMemset2DAsync(c, static_cast<size_t>(ldc) * 4, 0, static_cast<size_t>(n) * 4,
                                      static_cast<size_t>(a->rows), strm);
    return e == cudaSuccess ? KAIRO_STATUS_SUCCESS : cuda_fail(e, "cudaMemset2DAsync(C)");
  }
  const TcPlan& plan = ch.plan;
  if (!workspace) return fail(KAIRO_STATUS_INVALID_VALUE, "null workspace");
  if (workspace_bytes < plan.workspace_bytes) {
    std::ostringstream os;
    os << "workspace of " << workspace_bytes << " bytes, " << plan.workspace_bytes << " needed";
    return fail(KAIRO_STATUS_WORKSPACE_TOO_SMALL, os.str());
  }
  KernelFn fn = a->dtype == KAIRO_DTYPE_F16 ? pick_rg<0>(plan.bm, plan.nt, plan.rg) : pick_rg<1>(plan.bm, plan.nt, plan.rg);
  if (!fn) return fail(KAIRO_STATUS_NOT_SUPPORTED, "no row-group kernel for this block size / n_tile / group size");
  CUtensorMap map_a, map_b;
  int b_box3d = 0;
  st = make_operand_maps(a, b, ldb, false, n, plan.nt, &map_a, &map_b, &b_box3d);
  if (st) return st;
  const kairo_bsr v = group_view(a, s);
  TcArgs args{};
  args.row_ptr = v.row_ptr;
  args.col_idx = v.col_idx;
  args.blk_idx = v.blk_idx;
  args.c = c;
  args.ldc = ldc;
  args.w = plan.w;
  args.nblocks_stored = a->nblocks_stored;
  args.nnzb = v.nnzb;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  args.err = reinterpret_cast<unsigned*>(ws);
  const int bank = tc_next_counter_bank(workspace);
  unsigned* banks = reinterpret_cast<unsigned*>(ws + plan.counters_offset);
  args.counters = banks + bank * kCounterBankEntries;
  args.counters_other = banks + (1 - bank) * kCounterBankEntries;
  args.partials = reinterpret_cast<float*>(ws + plan.partials_offset);
  args.m = static_cast<int32_t>(a->rows);
  args.n = static_cast<int32_t>(n);
  args.nbr = v.nbr;
  args.nbc = static_cast<int32_t>(ceil_div64(a->cols, a->bk));
  args.chunk_group = plan.chunk_group;
  args.ngroups = plan.ngroups;
  args.row_cost = plan.row_cost;
  args.stages = plan.stages;
  args.group = plan.group;
  args.tmem_cols = plan.tmem_cols;
  args.b_box3d = b_box3d;
  args.hold_stage = plan.hold_stage;
  args.wait_cycles = plan.wait_cycles;
  args.vec_store = 0;
  args.stack_blk = s->super_blk;
  args.row_map = s->row_map;
  args.c_vec4 = ((reinterpret_cast<uintptr_t>(c) & 15u) == 0) && (ldc % 4 == 0) ? 1 : 0;
  args.packed = 0;
  args.a_batch = 0;
  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(plan.smem_bytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  fn<<<plan.grid, kThreads, plan.smem_bytes, strm>>>(map_a, map_b, map_a, args);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the row-group tcgen05 SpMM kernel");
  return KAIRO_STATUS_SUCCESS;
}

}  // extern "C"
