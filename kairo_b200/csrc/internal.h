// Internal declarations shared by the translation units of libkairo_spmm.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

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
};

// tcgen05 path (spmm_tc.cu)
bool tc_supported(const kairo_bsr* a, int32_t layout, int64_t n, int64_t ldb, int64_t ldc,
                  kairo_dtype c_dtype, const void* b, const void* c, std::string* why);
kairo_status tc_plan(const kairo_bsr* a, int32_t layout, int64_t n, const kairo_spmm_config* cfg,
                     int device, TcPlan* plan);
kairo_status tc_launch(const kairo_bsr* a, const void* b, int64_t ldb, int32_t layout, int64_t n,
                       void* c, int64_t ldc, kairo_dtype c_dtype, const TcPlan& plan,
                       void* workspace, cudaStream_t stream);

// SIMT path (spmm_simt.cu)
bool simt_supported(const kairo_bsr* a, int32_t layout, kairo_dtype c_dtype, std::string* why);
kairo_status simt_launch(const kairo_bsr* a, const void* b, int64_t ldb, int64_t n, void* c,
                         int64_t ldc, void* workspace, cudaStream_t stream);

// BSR construction (bsr_build.cu)
size_t bsr_build_ws_bytes(int64_t num_tiles, int32_t nbr);

}  // namespace kairo
