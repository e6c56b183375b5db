// Internal declarations shared by the translation units of libkairo_spmm.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/kairo_spmm.h"

namespace kairo {

// Per-thread message behind kairo_last_error_message().
void set_error(const std::string& msg);
kairo_status fail(kairo_status s, const std::string& msg);
kairo_status cuda_fail(cudaError_t e, const char* what);

int device_sm_count(int device);
int current_device();

inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

constexpr size_t kWorkspaceHeaderBytes = 256;  // error word + reserved

// Split-row arrival counters of the tcgen05 kernel live in a region of fixed
// size right after the header, so that no launch configuration ever places
// partial tiles over another configuration's counters.  Two banks alternate
// between launches on one workspace; each launch zeroes the bank it does not
// use, which also clears counters left behind by an aborted launch.
constexpr int kCounterBankEntries = 16384;
constexpr size_t kCounterRegionBytes = 2 * kCounterBankEntries * sizeof(unsigned);

// Blocks per pipeline stage when the caller leaves it to the library.  On
// B200, TMA gathers of B panels into shared memory run faster in fewer,
// larger stage groups while their data is in L2 (16 KB panels: 40, 49, 55 and
// 60 B/clk per SM with groups of 2, 3, 4 and 6 blocks), whereas gathers that
// miss L2 are bound by HBM and gain from more stages in flight instead.  So:
// four stages when the B slice of one chunk exceeds half of L2; otherwise
// three stages of the largest group that fits, or two when fewer than nine
// block slots fit.
// With several CTAs per SM the stages of all of them are in flight at once;
// each CTA then keeps three stages (measured best at two CTAs per SM on the
// 262144^2, 16384^2 and Zipf workloads).
inline int default_group_blocks(int slots, bool b_slice_exceeds_half_l2, int ctas_per_sm = 1) {
  const int stages = ctas_per_sm > 1 ? 3 : (b_slice_exceeds_half_l2 ? 4 : (slots >= 9 ? 3 : 2));
  int g = slots / stages;
  if (g > 32) g = 32;
  if (g < 1) g = 1;
  return g;
}

// Shared memory of one SM and the part the driver reserves per resident CTA
// (sm_100: 228 KiB and 1 KiB).
constexpr int kSmemPerSm = 228 * 1024;
constexpr int kSmemReservedPerCta = 1024;

// Resident CTAs per SM of the row-split tcgen05 kernel when the caller
// leaves it to the library.
int default_ctas_per_sm(const kairo_bsr* a, int nt, int sms);

// Bytes of the B (or X) columns one chunk of 128 * nt output columns reads.
inline double b_slice_bytes(const kairo_bsr* a, int nt) { return static_cast<double>(a->cols) * 128.0 * nt * 2.0; }

// L2 size of `device` in bytes (126 MB if the query fails).
int device_l2_bytes(int device);

// Scheduling plan of one tcgen05 launch (host side).
struct TcPlan {
  int bm, bk, nt;          // block size, 128-column sub-tiles per work item
  int nchunks;             // ceil(N / (128 * nt))
  int chunk_group;         // chunks processed as one merge-path segment (divides nchunks)
  int ngroups;             // nchunks / chunk_group; ngroups * grid <= kCounterBankEntries
  int row_cost;            // R
  int64_t w;               // path length of one chunk: nnzb + R * nbr
  int grid;                // persistent CTAs
  int stages;              // stage groups
  int group;               // blocks per stage group
  uint32_t tmem_cols;      // TMEM columns allocated per CTA
  size_t smem_bytes;
  size_t counters_offset, counters_bytes;
  size_t partials_offset, partials_bytes;
  size_t workspace_bytes;
  long long wait_cycles;   // bound of every mbarrier wait (kairo_spmm_config.wait_kcycles)
  int hold_stage;          // kairo_spmm_config.debug_hold_stage
  int ctas_per_sm;         // resident CTAs per SM the shared-memory budget was split for
  int rg;                  // block-rows per item (1, or the row-group size)
  int packed;              // stages hold their panels, then their blocks packed (rg = 1, 16-row blocks)
};

// TMA tensor maps (tma_maps.cu).  make_operand_maps builds the block-storage
// map and the B map (3D MN-major panel view when N % 64 == 0, else 2D) or,
// for the LINEAR layout, the X map; *b_box3d tells which B map was built.
kairo_status make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                         uint64_t inner, uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner,
                         uint32_t box_outer, const char* what);
kairo_status make_map_b3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t n, uint64_t k,
                          uint64_t ldb, uint32_t bk, uint32_t atoms);
// The block storage as runs of `blocks` consecutive blocks (one box of
// blocks * bm rows, at most 256), for copying a stage of consecutive blocks.
kairo_status make_block_run_map(const kairo_bsr* a, int blocks, CUtensorMap* map);
kairo_status make_operand_maps(const kairo_bsr* a, const void* b, int64_t ldb, bool linear, int64_t n, int nt,
                               CUtensorMap* map_a, CUtensorMap* map_b, int* b_box3d);

// Scheduling plan of one band-schedule launch (host side).  An item is
// (chunk of 128*nt columns of C, group of `rows` consecutive block-rows); its
// blocks are visited in column order (a per-launch sort into `order`) so
// that all CTAs sweep the B panels of a chunk together.
struct BandPlan {
  int bm, bk, nt;
  int nchunks;
  int rows;                // block-rows per item (R)
  int row_groups;          // ceil(nbr / R)
  int64_t nitems;          // nchunks * row_groups
  int acc_slots;           // TMEM accumulator sets (2 = epilogue overlaps the next item)
  int grid;
  int stages;
  int group;
  int serpentine;          // odd item waves visit their blocks in descending column order
  uint32_t tmem_cols;
  size_t smem_bytes;
  size_t order_offset, order_bytes;
  size_t workspace_bytes;
  long long wait_cycles;   // bound of every mbarrier wait (kairo_spmm_config.wait_kcycles)
};

// Band schedule (spmm_band.cu)
bool band_supported(const kairo_bsr* a, std::string* why);
bool band_preferred(const kairo_bsr* a, int64_t n, int device);
kairo_status band_plan(const kairo_bsr* a, int32_t layout, int64_t n, const kairo_spmm_config* cfg,
                       int device, BandPlan* plan);
kairo_status band_launch(const kairo_bsr* a, const void* b, int64_t ldb, int32_t layout, int64_t n,
                         void* c, int64_t ldc, kairo_dtype c_dtype, const BandPlan& plan,
                         void* workspace, cudaStream_t stream);

// tcgen05 path (spmm_tc.cu)
bool tc_supported(const kairo_bsr* a, int32_t layout, int64_t n, int64_t ldb, int64_t ldc,
                  kairo_dtype c_dtype, const void* b, const void* c, std::string* why);
// rg > 1 plans a row-group launch: `a` then describes the groups (nbr =
// groups, nnzb = stacked blocks), and slots, accumulators and partial tiles
// hold rg blocks' rows.
kairo_status tc_plan(const kairo_bsr* a, int32_t layout, int64_t n, const kairo_spmm_config* cfg,
                     int device, TcPlan* plan, int rg = 1);
// Counter bank (0 or 1) of the next row-split launch on `workspace`; the
// banks alternate per workspace (spmm_tc.cu).
int tc_next_counter_bank(void* workspace);
kairo_status tc_launch(const kairo_bsr* a, const void* b, int64_t ldb, int32_t layout, int64_t n,
                       void* c, int64_t ldc, kairo_dtype c_dtype, const TcPlan& plan,
                       void* workspace, cudaStream_t stream);

// fp32 on the tcgen05 kernel by a bf16 hi/lo split (spmm_split.cu).  The
// derived operands occupy `bytes` of workspace: blocks (3 nnzb, bm, bk)
// bf16, block-column indices, row pointers, and a (k, ldb) bf16 B.
struct SplitLayout {
  int64_t ldb;  // leading dimension of the derived B (N rounded up to 8)
  int64_t k;    // rows of the derived B: 3 * nbc * bk
  size_t blocks_off, col_idx_off, row_ptr_off, b_off, bytes;
};
SplitLayout split_bf16_layout(const kairo_bsr* a, int64_t n);
kairo_bsr split_bf16_desc(const kairo_bsr* a, const SplitLayout& l, void* base);
kairo_status split_bf16_prepare(const kairo_bsr* a, const void* b, int64_t ldb, int64_t n, const SplitLayout& l,
                                void* base, cudaStream_t s);

// SIMT path (spmm_simt.cu)
bool simt_supported(const kairo_bsr* a, int32_t layout, kairo_dtype c_dtype, std::string* why);
kairo_status simt_launch(const kairo_bsr* a, const void* b, int64_t ldb, int64_t n, void* c,
                         int64_t ldc, void* workspace, cudaStream_t stream);

// BSR construction (bsr_build.cu)
size_t bsr_build_ws_bytes(int64_t num_tiles, int32_t nbr);

// Stable bucket sort on the device, asynchronously (bsr_build.cu).  For t in
// [0, n): keys[t] in [0, nbuckets), vals[t] in [0, nvals) (anything else is
// recorded as KAIRO_DEVERR_BAD_INDEX in the workspace error word).  Writes
// bucket_ptr (nbuckets + 1 offsets), perm (the original index of every
// sorted position, ascending inside a bucket) and vals_sorted[q] =
// vals[perm[q]].  A bucket of more than kBucketSortMax entries is left in
// arbitrary order and records KAIRO_DEVERR_ROW_TOO_LONG unless
// long_buckets_ok.  ws needs bucket_sort_ws_bytes(nbuckets) bytes and starts
// with the error word.
constexpr int kBucketSortMax = 16384;
size_t bucket_sort_ws_bytes(int32_t nbuckets);
kairo_status bucket_sort(const int32_t* keys, const int32_t* vals, int32_t nvals, int64_t n, int32_t nbuckets,
                         int32_t* bucket_ptr, int32_t* perm, int32_t* vals_sorted, void* ws, cudaStream_t s,
                         bool long_buckets_ok = false);

}  // namespace kairo
