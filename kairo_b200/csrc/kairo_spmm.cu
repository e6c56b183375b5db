// C-ABI entry points of libkairo_spmm (declared in include/kairo_spmm.h):
// argument validation with the reference's error conventions, kernel
// selection, workspace carving, and the acc_spmm_forward composition
// (COO tiles -> BSR -> SpMM) that replaces csrc/acc_spmm_kernel.cu:158-207.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <sstream>
#include <string>

#include "internal.h"

namespace kairo {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) { g_last_error = msg; }

kairo_status fail(kairo_status s, const std::string& msg) {
  set_error(msg);
  return s;
}

kairo_status cuda_fail(cudaError_t e, const char* what) {
  std::ostringstream os;
  os << what << ": " << cudaGetErrorName(e) << " (" << cudaGetErrorString(e) << ")";
  return fail(KAIRO_STATUS_CUDA_ERROR, os.str());
}

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

int device_sm_count(int device) {
  static std::mutex mu;
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
    cache[device] = v;
  }
  return cache[device];
}

int device_l2_bytes(int device) {
  static std::mutex mu;
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 126 << 20;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrL2CacheSize, device) != cudaSuccess || v <= 0) v = 126 << 20;
    cache[device] = v;
  }
  return cache[device];
}

namespace {

kairo_status validate_bsr(const kairo_bsr* a) {
  if (!a) return fail(KAIRO_STATUS_INVALID_VALUE, "null BSR descriptor");
  if (a->rows < 0 || a->cols < 0 || a->nnzb < 0 || a->nbr < 0)
    return fail(KAIRO_STATUS_INVALID_VALUE, "negative BSR size");
  if (a->bm <= 0 || a->bk <= 0) return fail(KAIRO_STATUS_INVALID_VALUE, "block size must be positive");
  if (a->nbr != ceil_div64(a->rows, a->bm)) return fail(KAIRO_STATUS_INVALID_VALUE, "nbr must equal ceil(rows / bm)");
  if (a->dtype != KAIRO_DTYPE_F32 && a->dtype != KAIRO_DTYPE_F16 && a->dtype != KAIRO_DTYPE_BF16)
    return fail(KAIRO_STATUS_INVALID_VALUE, "unknown dtype");
  if (a->nnzb > 0x7fffffffLL) return fail(KAIRO_STATUS_NOT_SUPPORTED, "more than 2^31-1 nonzero blocks");
  if (a->nbr > 0 && !a->row_ptr) return fail(KAIRO_STATUS_INVALID_VALUE, "null row_ptr");
  if (a->nnzb > 0 && (!a->col_idx || !a->blocks)) return fail(KAIRO_STATUS_INVALID_VALUE, "null col_idx or blocks");
  if (a->blk_idx == nullptr && a->nblocks_stored < a->nnzb)
    return fail(KAIRO_STATUS_INVALID_VALUE, "nblocks_stored < nnzb with identity block order");
  return KAIRO_STATUS_SUCCESS;
}

enum class Path { kNone, kZero, kSimt, kTc, kBand, kSplit };

struct Choice {
  Path path = Path::kNone;
  TcPlan plan{};
  BandPlan band{};
  SplitLayout split{};  // kSplit: derived operands after the tcgen05 workspace
  size_t split_base = 0;
};

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

kairo_status choose(const kairo_bsr* a, const void* b, int64_t ldb, int32_t layout, int64_t n, const void* c,
                    int64_t ldc, kairo_dtype c_dtype, const kairo_spmm_config* cfg, Choice* out) {
  kairo_status st = validate_bsr(a);
  if (st) return st;
  if (layout != KAIRO_LAYOUT_STANDARD && layout != KAIRO_LAYOUT_LINEAR)
    return fail(KAIRO_STATUS_INVALID_VALUE, "unknown layout");
  if (n < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "negative N");
  if (layout == KAIRO_LAYOUT_STANDARD) {
    if (ldb < n || ldc < n) return fail(KAIRO_STATUS_INVALID_VALUE, "leading dimension smaller than N");
  } else {
    if (ldb < a->cols || ldc < a->rows) return fail(KAIRO_STATUS_INVALID_VALUE, "leading dimension smaller than K or M");
  }
  Choice ch;
  if (a->rows == 0 || n == 0) {
    ch.path = Path::kNone;
    *out = ch;
    return KAIRO_STATUS_SUCCESS;
  }
  if (!c) return fail(KAIRO_STATUS_INVALID_VALUE, "null C");
  if (a->nnzb == 0) {
    ch.path = Path::kZero;
    *out = ch;
    return KAIRO_STATUS_SUCCESS;
  }
  if (!b) return fail(KAIRO_STATUS_INVALID_VALUE, "null B");
  const int kernel = cfg ? cfg->kernel : KAIRO_KERNEL_AUTO;
  std::string why_tc, why_simt;
  const bool tc_ok = tc_supported(a, layout, n, ldb, ldc, c_dtype, b, c, &why_tc);
  const bool simt_ok = simt_supported(a, layout, c_dtype, &why_simt);
  const int schedule = cfg ? cfg->schedule : KAIRO_SCHEDULE_AUTO;
  if (schedule != KAIRO_SCHEDULE_AUTO && schedule != KAIRO_SCHEDULE_ROWS && schedule != KAIRO_SCHEDULE_BANDS)
    return fail(KAIRO_STATUS_INVALID_VALUE, "unknown schedule selector");
  if (schedule == KAIRO_SCHEDULE_BANDS && (kernel == KAIRO_KERNEL_SIMT || kernel == KAIRO_KERNEL_SPLIT_BF16))
    return fail(KAIRO_STATUS_INVALID_VALUE, "the band schedule runs on the tcgen05 kernel only");
  if (kernel == KAIRO_KERNEL_SPLIT_BF16) {
    if (a->dtype != KAIRO_DTYPE_F32) return fail(KAIRO_STATUS_NOT_SUPPORTED, "the split-bf16 kernel takes fp32 input");
    if (layout != KAIRO_LAYOUT_STANDARD)
      return fail(KAIRO_STATUS_NOT_SUPPORTED, "the split-bf16 kernel implements the STANDARD layout only");
    if (3 * a->nnzb > INT32_MAX) return fail(KAIRO_STATUS_NOT_SUPPORTED, "too many blocks for the split-bf16 kernel");
    if (reinterpret_cast<uintptr_t>(a->blocks) & 15u)
      return fail(KAIRO_STATUS_NOT_SUPPORTED, "the split-bf16 kernel needs 16-byte aligned block storage");
    // Plan on the derived bf16 operands, with aligned stand-in pointers.
    static const uint8_t dummy[16] __attribute__((aligned(16))) = {0};
    ch.split = split_bf16_layout(a, n);
    kairo_bsr d = split_bf16_desc(a, ch.split, const_cast<uint8_t*>(dummy));
    d.blocks = dummy;
    std::string why;
    if (!tc_supported(&d, layout, n, ch.split.ldb, ldc, c_dtype, dummy, c, &why))
      return fail(KAIRO_STATUS_NOT_SUPPORTED, why);
    ch.path = Path::kSplit;
    st = tc_plan(&d, layout, n, cfg, current_device(), &ch.plan);
    if (st) return st;
    ch.split_base = align256(ch.plan.workspace_bytes);
  } else if (kernel == KAIRO_KERNEL_TCGEN05 || (kernel == KAIRO_KERNEL_AUTO && tc_ok)) {
    if (!tc_ok) return fail(KAIRO_STATUS_NOT_SUPPORTED, why_tc);
    const int dev = current_device();
    std::string why_band;
    const bool band_ok = band_supported(a, &why_band);
    if (schedule == KAIRO_SCHEDULE_BANDS && !band_ok) return fail(KAIRO_STATUS_NOT_SUPPORTED, why_band);
    if (schedule == KAIRO_SCHEDULE_BANDS || (schedule == KAIRO_SCHEDULE_AUTO && band_ok && band_preferred(a, n, dev))) {
      ch.path = Path::kBand;
      st = band_plan(a, layout, n, cfg, dev, &ch.band);
    } else {
      ch.path = Path::kTc;
      st = tc_plan(a, layout, n, cfg, dev, &ch.plan);
    }
    if (st) return st;
  } else if (kernel == KAIRO_KERNEL_SIMT || kernel == KAIRO_KERNEL_AUTO) {
    if (!simt_ok) return fail(KAIRO_STATUS_NOT_SUPPORTED, kernel == KAIRO_KERNEL_AUTO ? why_tc + "; " + why_simt : why_simt);
    ch.path = Path::kSimt;
  } else {
    return fail(KAIRO_STATUS_INVALID_VALUE, "unknown kernel selector");
  }
  *out = ch;
  return KAIRO_STATUS_SUCCESS;
}

// Every workspace reserves the tcgen05 counter region, whichever kernel runs,
// so memory that one call uses for other data is never another call's counter.
size_t ws_bytes_for(const Choice& ch) {
  if (ch.path == Path::kTc) return ch.plan.workspace_bytes;
  if (ch.path == Path::kBand) return ch.band.workspace_bytes;
  if (ch.path == Path::kSplit) return ch.split_base + ch.split.bytes;
  return kWorkspaceHeaderBytes + kCounterRegionBytes;
}

size_t dtype_size(kairo_dtype d) { return d == KAIRO_DTYPE_F32 ? 4 : 2; }

kairo_status zero_c(const kairo_bsr* a, int32_t layout, int64_t n, void* c, int64_t ldc, kairo_dtype c_dtype,
                    cudaStream_t s) {
  const size_t es = dtype_size(c_dtype);
  const int64_t rows = layout == KAIRO_LAYOUT_STANDARD ? a->rows : n;
  const int64_t cols = layout == KAIRO_LAYOUT_STANDARD ? n : a->rows;
  cudaError_t e = cudaMemset2DAsync(c, static_cast<size_t>(ldc) * es, 0, static_cast<size_t>(cols) * es,
                                    static_cast<size_t>(rows), s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemset2DAsync(C)");
  return KAIRO_STATUS_SUCCESS;
}

}  // namespace
}  // namespace kairo

using namespace kairo;

extern "C" {

const char* kairo_status_string(kairo_status s) {
  switch (s) {
    case KAIRO_STATUS_SUCCESS: return "success";
    case KAIRO_STATUS_INVALID_VALUE: return "invalid value";
    case KAIRO_STATUS_NOT_SUPPORTED: return "not supported";
    case KAIRO_STATUS_CUDA_ERROR: return "CUDA error";
    case KAIRO_STATUS_WORKSPACE_TOO_SMALL: return "workspace too small";
    case KAIRO_STATUS_DEVICE_ERROR: return "device error";
  }
  return "unknown status";
}

const char* kairo_last_error_message(void) { return g_last_error.c_str(); }

int32_t kairo_abi_version(void) { return KAIRO_ABI_VERSION; }

namespace {

// The path kairo_bsr_spmm would take for `a`, with aligned dummy operands.
kairo_status probe_choice(const kairo_bsr* a, int32_t layout, int64_t n, const kairo_spmm_config* cfg, Choice* ch) {
  // Pointer-alignment checks cannot be made without the operands; assume
  // aligned operands (the size only grows on the tcgen05 path).
  kairo_bsr probe = *a;
  static const uint8_t dummy[16] __attribute__((aligned(16))) = {0};
  if (!probe.blocks) probe.blocks = dummy;
  if (!probe.row_ptr) probe.row_ptr = reinterpret_cast<const int32_t*>(dummy);
  if (!probe.col_idx) probe.col_idx = reinterpret_cast<const int32_t*>(dummy);
  const int64_t ldb = layout == KAIRO_LAYOUT_STANDARD ? ((n + 7) / 8) * 8 : ((a->cols + 7) / 8) * 8;
  const int64_t ldc = layout == KAIRO_LAYOUT_STANDARD ? n : a->rows;
  const kairo_dtype c_dtype = KAIRO_DTYPE_F32;
  return choose(&probe, dummy, ldb, layout, n, dummy, ldc, c_dtype, cfg, ch);
}

}  // namespace

kairo_status kairo_bsr_spmm_workspace_size(const kairo_bsr* a, int32_t layout, int64_t n,
                                           const kairo_spmm_config* cfg, size_t* bytes) {
  if (!bytes || !a) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  Choice ch;
  kairo_status st = probe_choice(a, layout, n, cfg, &ch);
  if (st) return st;
  *bytes = ws_bytes_for(ch);
  return KAIRO_STATUS_SUCCESS;
}

kairo_status kairo_bsr_spmm_describe(const kairo_bsr* a, int32_t layout, int64_t n, const kairo_spmm_config* cfg,
                                     kairo_spmm_plan* out) {
  if (!out || !a) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  Choice ch;
  kairo_status st = probe_choice(a, layout, n, cfg, &ch);
  if (st) return st;
  kairo_spmm_plan p{};
  p.workspace_bytes = ws_bytes_for(ch);
  switch (ch.path) {
    case Path::kNone:
      break;
    case Path::kZero:
      p.launches = 1;
      break;
    case Path::kSimt:
      p.kernel = KAIRO_KERNEL_SIMT;
      p.launches = 1;
      p.n_tile = 128;
      break;
    case Path::kTc:
      p.kernel = KAIRO_KERNEL_TCGEN05;
      p.schedule = KAIRO_SCHEDULE_ROWS;
      p.launches = 1;
      p.grid = ch.plan.grid;
      p.n_tile = 128 * ch.plan.nt;
      p.stages = ch.plan.stages;
      p.group_blocks = ch.plan.group;
      p.rows = ch.plan.row_cost;
      break;
    case Path::kSplit:
      p.kernel = KAIRO_KERNEL_SPLIT_BF16;
      p.schedule = KAIRO_SCHEDULE_ROWS;
      p.launches = 2;
      p.grid = ch.plan.grid;
      p.n_tile = 128 * ch.plan.nt;
      p.stages = ch.plan.stages;
      p.group_blocks = ch.plan.group;
      p.rows = ch.plan.row_cost;
      break;
    case Path::kBand:
      p.kernel = KAIRO_KERNEL_TCGEN05;
      p.schedule = KAIRO_SCHEDULE_BANDS;
      p.launches = 2;
      p.grid = ch.band.grid;
      p.n_tile = 128 * ch.band.nt;
      p.stages = ch.band.stages;
      p.group_blocks = ch.band.group;
      p.rows = ch.band.rows;
      break;
  }
  *out = p;
  return KAIRO_STATUS_SUCCESS;
}

kairo_status kairo_bsr_spmm(const kairo_bsr* a, const void* b, int64_t ldb, int32_t layout, int64_t n, void* c,
                            int64_t ldc, kairo_dtype c_dtype, const kairo_spmm_config* cfg, void* workspace,
                            size_t workspace_bytes, void* stream) {
  Choice ch;
  kairo_status st = choose(a, b, ldb, layout, n, c, ldc, c_dtype, cfg, &ch);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (ch.path) {
    case Path::kNone:
      return KAIRO_STATUS_SUCCESS;
    case Path::kZero:
      return zero_c(a, layout, n, c, ldc, c_dtype, s);
    default:
      break;
  }
  if (!workspace) return fail(KAIRO_STATUS_INVALID_VALUE, "null workspace");
  if (workspace_bytes < ws_bytes_for(ch)) {
    std::ostringstream os;
    os << "workspace of " << workspace_bytes << " bytes, " << ws_bytes_for(ch) << " needed";
    return fail(KAIRO_STATUS_WORKSPACE_TOO_SMALL, os.str());
  }
  if (ch.path == Path::kTc) return tc_launch(a, b, ldb, layout, n, c, ldc, c_dtype, ch.plan, workspace, s);
  if (ch.path == Path::kBand) return band_launch(a, b, ldb, layout, n, c, ldc, c_dtype, ch.band, workspace, s);
  if (ch.path == Path::kSplit) {
    void* base = static_cast<uint8_t*>(workspace) + ch.split_base;
    st = split_bf16_prepare(a, b, ldb, n, ch.split, base, s);
    if (st) return st;
    const kairo_bsr d = split_bf16_desc(a, ch.split, base);
    return tc_launch(&d, static_cast<uint8_t*>(base) + ch.split.b_off, ch.split.ldb, layout, n, c, ldc, c_dtype,
                     ch.plan, workspace, s);
  }
  return simt_launch(a, b, ldb, n, c, ldc, workspace, s);
}

// ------------------------------------------------------------ acc_spmm_forward

namespace {

struct ForwardLayout {
  int32_t nbr, nbc;
  size_t row_ptr_off, col_idx_off, perm_off, build_off, spmm_off, total;
};

kairo_status forward_layout(int32_t m, int32_t k, int32_t n, int32_t num_tiles, int32_t tile_m, int32_t tile_k,
                            kairo_dtype dtype, ForwardLayout* out, Choice* ch_out) {
  // bindings.cpp:92-100: positive dimensions, int32 ids (contiguity is a
  // property of the caller's buffers here).
  if (m <= 0 || k <= 0 || n <= 0) return fail(KAIRO_STATUS_INVALID_VALUE, "dimensions must be positive");
  if (num_tiles < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "num_tiles must be non-negative");
  if (tile_m <= 0 || tile_k <= 0) return fail(KAIRO_STATUS_INVALID_VALUE, "tile sizes must be positive");
  ForwardLayout L{};
  L.nbr = static_cast<int32_t>(ceil_div64(m, tile_m));
  L.nbc = static_cast<int32_t>(ceil_div64(k, tile_k));
  kairo_bsr a{};
  a.rows = m;
  a.cols = k;
  a.bm = tile_m;
  a.bk = tile_k;
  a.nbr = L.nbr;
  a.nnzb = num_tiles;
  a.nblocks_stored = num_tiles;
  a.dtype = dtype;
  static const uint8_t dummy[16] __attribute__((aligned(16))) = {0};
  a.row_ptr = reinterpret_cast<const int32_t*>(dummy);
  a.col_idx = reinterpret_cast<const int32_t*>(dummy);
  a.blk_idx = reinterpret_cast<const int32_t*>(dummy);
  a.blocks = dummy;
  Choice ch;
  kairo_status st = choose(&a, dummy, n, KAIRO_LAYOUT_STANDARD, n, dummy, n, KAIRO_DTYPE_F32, nullptr, &ch);
  if (st) return st;
  // The SpMM workspace comes first so that its error word is the error word
  // of the whole acc_spmm_forward workspace (kairo_workspace_error).
  size_t off = 0;
  L.spmm_off = off;
  off += align_up(ws_bytes_for(ch), 256);
  L.row_ptr_off = off;
  off += align_up((static_cast<size_t>(L.nbr) + 1) * 4, 256);
  L.col_idx_off = off;
  off += align_up(static_cast<size_t>(num_tiles) * 4, 256);
  L.perm_off = off;
  off += align_up(static_cast<size_t>(num_tiles) * 4, 256);
  L.build_off = off;
  off += align_up(bsr_build_ws_bytes(num_tiles, L.nbr), 256);
  L.total = off;
  *out = L;
  if (ch_out) *ch_out = ch;
  return KAIRO_STATUS_SUCCESS;
}

}  // namespace

kairo_status kairo_acc_spmm_forward_workspace_size(int32_t m, int32_t k, int32_t n, int32_t num_tiles, int32_t tile_m,
                                                   int32_t tile_k, kairo_dtype dtype, size_t* bytes) {
  if (!bytes) return fail(KAIRO_STATUS_INVALID_VALUE, "null bytes");
  ForwardLayout L;
  kairo_status st = forward_layout(m, k, n, num_tiles, tile_m, tile_k, dtype, &L, nullptr);
  if (st) return st;
  *bytes = L.total;
  return KAIRO_STATUS_SUCCESS;
}

kairo_status kairo_acc_spmm_forward(const void* a_tiles, const int32_t* tile_row_ids, const int32_t* tile_col_ids,
                                    const void* b, float* c, int32_t m, int32_t k, int32_t n, int32_t num_tiles,
                                    int32_t tile_m, int32_t tile_k, kairo_dtype dtype, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  ForwardLayout L;
  kairo_status st = forward_layout(m, k, n, num_tiles, tile_m, tile_k, dtype, &L, nullptr);
  if (st) return st;
  if (!c || !b) return fail(KAIRO_STATUS_INVALID_VALUE, "null B or C");
  if (num_tiles > 0 && (!a_tiles || !tile_row_ids || !tile_col_ids))
    return fail(KAIRO_STATUS_INVALID_VALUE, "null tile arrays");
  if (!workspace) return fail(KAIRO_STATUS_INVALID_VALUE, "null workspace");
  if (workspace_bytes < L.total) return fail(KAIRO_STATUS_WORKSPACE_TOO_SMALL, "acc_spmm_forward workspace too small");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* row_ptr = reinterpret_cast<int32_t*>(ws + L.row_ptr_off);
  int32_t* col_idx = reinterpret_cast<int32_t*>(ws + L.col_idx_off);
  int32_t* perm = reinterpret_cast<int32_t*>(ws + L.perm_off);
  int32_t identity = 0;
  // max_row_blocks stays 0 (row-split schedule): the workspace was sized before
  // the build, without knowing the row lengths.
  st = kairo_bsr_build(tile_row_ids, tile_col_ids, num_tiles, L.nbr, L.nbc, row_ptr, col_idx, perm, &identity,
                       nullptr, ws + L.build_off, L.total - L.build_off, stream);
  if (st) return st;
  kairo_bsr a{};
  a.rows = m;
  a.cols = k;
  a.bm = tile_m;
  a.bk = tile_k;
  a.nbr = L.nbr;
  a.nnzb = num_tiles;
  a.nblocks_stored = num_tiles;
  a.row_ptr = row_ptr;
  a.col_idx = col_idx;
  a.blk_idx = identity ? nullptr : perm;
  a.blocks = a_tiles;
  a.dtype = dtype;
  return kairo_bsr_spmm(&a, b, n, KAIRO_LAYOUT_STANDARD, n, c, n, KAIRO_DTYPE_F32, nullptr, ws + L.spmm_off,
                        L.row_ptr_off - L.spmm_off, stream);
}

// ------------------------------------------------------------ host helpers

kairo_status kairo_partition_rows(const int64_t* row_ptr, int32_t nbr, int32_t parts, int32_t* bounds) {
  if (!row_ptr || !bounds || nbr < 0 || parts <= 0) return fail(KAIRO_STATUS_INVALID_VALUE, "invalid argument");
  const int64_t nnzb = row_ptr[nbr];
  bounds[0] = 0;
  for (int32_t p = 1; p < parts; ++p) {
    const int64_t target = nnzb * p / parts;
    // first row whose prefix reaches the target
    const int64_t* it = std::lower_bound(row_ptr, row_ptr + nbr + 1, target);
    int32_t r = static_cast<int32_t>(it - row_ptr);
    r = std::min(std::max(r, bounds[p - 1]), nbr);
    bounds[p] = r;
  }
  bounds[parts] = nbr;
  return KAIRO_STATUS_SUCCESS;
}

kairo_status kairo_workspace_error(void* workspace, int32_t clear, uint32_t* code, void* stream) {
  if (!workspace || !code) return fail(KAIRO_STATUS_INVALID_VALUE, "null argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(workspace, 0, sizeof(uint32_t), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "reading the workspace error word");
  *code = v;
  return KAIRO_STATUS_SUCCESS;
}

}  // extern "C"
