// Host side of the row-split tcgen05 BSR SpMM: plan, kernel selection and
// launch.  The kernel itself (formulation, roles, scheduler, bounded waits)
// is described in spmm_tc_kernel.cuh.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <sstream>
#include <unordered_map>

#include "spmm_tc_kernel.cuh"

namespace kairo {
namespace {

// ---------------------------------------------------------------- host side

using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, TcArgs);

template <int BM, int NT, bool LINEAR, int IN_FMT, typename TOut>
KernelFn pick4() {
  return reinterpret_cast<KernelFn>(&bsr_spmm_tc_kernel<BM, BM, NT, LINEAR, IN_FMT, TOut>);
}

template <bool LINEAR, int IN_FMT, typename TOut>
KernelFn pick3(int bm, int nt) {
#define KAIRO_TC_CASE(B, T) \
  if (bm == B && nt == T) return pick4<B, T, LINEAR, IN_FMT, TOut>();
  KAIRO_TC_CASE(16, 1)
  KAIRO_TC_CASE(16, 2)
  KAIRO_TC_CASE(32, 1)
  KAIRO_TC_CASE(32, 2)
  KAIRO_TC_CASE(64, 1)
  KAIRO_TC_CASE(64, 2)
#undef KAIRO_TC_CASE
  return nullptr;
}

KernelFn pick_kernel(int bm, int nt, bool linear, kairo_dtype in, kairo_dtype out) {
  if (!linear) {
    if (out != KAIRO_DTYPE_F32) return nullptr;
    return in == KAIRO_DTYPE_F16 ? pick3<false, 0, float>(bm, nt) : pick3<false, 1, float>(bm, nt);
  }
  if (in == KAIRO_DTYPE_F16) {
    if (out == KAIRO_DTYPE_F32) return pick3<true, 0, float>(bm, nt);
    if (out == KAIRO_DTYPE_F16) return pick3<true, 0, __half>(bm, nt);
  } else {
    if (out == KAIRO_DTYPE_F32) return pick3<true, 1, float>(bm, nt);
    if (out == KAIRO_DTYPE_BF16) return pick3<true, 1, __nv_bfloat16>(bm, nt);
  }
  return nullptr;
}

size_t elem_size(kairo_dtype d) { return d == KAIRO_DTYPE_F32 ? 4 : 2; }

}  // namespace

// Counter bank of the next launch on `workspace` (alternates per workspace).
// The map is bounded: past kMaxTrackedWorkspaces entries it is cleared, and
// the next launch on a forgotten workspace uses bank 0.  That is safe after
// a launch that completed, which leaves both banks at zero (it zeroed the
// other bank and reset its own counters).  Only after an aborted launch
// (a recorded device error) can bank 0 still hold counters, which is why
// the banks alternate at all.
int tc_next_counter_bank(void* workspace) {
  constexpr size_t kMaxTrackedWorkspaces = 4096;
  static std::mutex mu;
  static std::unordered_map<void*, int> parity;
  std::lock_guard<std::mutex> lock(mu);
  if (parity.size() >= kMaxTrackedWorkspaces && parity.find(workspace) == parity.end()) parity.clear();
  int& b = parity[workspace];
  const int use = b;
  b ^= 1;
  return use;
}


// Two resident CTAs per SM for blocks of up to 32 rows.  Measured on B200
// (median of 10 launches, L2 flushed; 1 CTA of 3-4 stages against 2 CTAs of
// 3 stages each): 262144^2 bf16 with 32x32 blocks 2.38 -> 2.22 ms, 16384^2
// fp16 with 32x32 blocks 0.068 -> 0.055 ms, the 65536^2 Zipf mask with 16x16
// blocks 0.165 -> 0.102 ms.  Three or four CTAs per SM were no faster; 64x64
// blocks (one stage holds two 40 KB slots) gained nothing.
int default_ctas_per_sm(const kairo_bsr* a, int nt, int sms) {
  (void)nt;
  (void)sms;
  return a->bm <= 32 ? 2 : 1;
}

bool tc_supported(const kairo_bsr* a, int32_t layout, int64_t n, int64_t ldb, int64_t ldc, kairo_dtype c_dtype,
                  const void* b, const void* c, std::string* why) {
  auto no = [&](const char* w) {
    if (why) *why = w;
    return false;
  };
  if (a->dtype != KAIRO_DTYPE_F16 && a->dtype != KAIRO_DTYPE_BF16) return no("tcgen05 path needs f16 or bf16 input");
  if (a->bm != a->bk) return no("tcgen05 path needs square blocks");
  if (a->bm != 16 && a->bm != 32 && a->bm != 64) return no("tcgen05 path supports blocks of 16, 32 or 64");
  if (ldb % 8 != 0) return no("B leading dimension must be a multiple of 8 elements (16-byte TMA stride)");
  if ((reinterpret_cast<uintptr_t>(b) & 15u) || (reinterpret_cast<uintptr_t>(a->blocks) & 15u))
    return no("B and block storage must be 16-byte aligned");
  if (a->nblocks_stored * a->bm > INT32_MAX || a->cols > INT32_MAX || n > INT32_MAX || a->rows > INT32_MAX)
    return no("problem exceeds 32-bit TMA coordinates");
  if (layout == KAIRO_LAYOUT_STANDARD) {
    if (c_dtype != KAIRO_DTYPE_F32) return no("STANDARD layout writes fp32 C");
  } else {
    if (c_dtype != KAIRO_DTYPE_F32 && c_dtype != a->dtype) return no("LINEAR output must be fp32 or the input dtype");
  }
  (void)ldc;
  (void)c;
  return true;
}

kairo_status tc_plan(const kairo_bsr* a, int32_t layout, int64_t n, const kairo_spmm_config* cfg, int device,
                     TcPlan* plan, int rg) {
  TcPlan p{};
  p.bm = a->bm;
  p.bk = a->bk;
  p.rg = rg;
  int nt = 1;
  if (cfg && cfg->n_tile) {
    if (cfg->n_tile != 128 && cfg->n_tile != 256) return fail(KAIRO_STATUS_INVALID_VALUE, "n_tile must be 128 or 256");
    nt = cfg->n_tile / 128;
  } else {
    // Two 128-column sub-tiles per work item: each block (the MMA B
    // operand) is loaded once for 256 columns of C, halving block re-reads
    // and pipeline handoffs per FLOP.  One sub-tile only when N <= 128.
    nt = n > 128 ? 2 : 1;
  }
  p.nt = nt;
  p.nchunks = static_cast<int>(ceil_div64(n, 128 * nt));
  // A block-row costs about as much as 8 blocks of work (its TMEM handoff,
  // epilogue and C stores); weighting rows this way keeps CTAs balanced on
  // masks with many short or empty rows (measured on a Zipf(1.1) mask: the
  // slowest CTA finished 80 % after the median with weight 2, 6 % with 8).
  p.row_cost = (cfg && cfg->row_cost > 0) ? cfg->row_cost : 8;
  if (cfg && (cfg->wait_kcycles < 0 || cfg->debug_hold_stage < 0 || cfg->debug_hold_stage > 1))
    return fail(KAIRO_STATUS_INVALID_VALUE, "wait_kcycles must be >= 0 and debug_hold_stage 0 or 1");
  p.wait_cycles = wait_bound_cycles(cfg);
  p.hold_stage = (cfg && cfg->debug_hold_stage) ? 1 : 0;
  p.w = a->nnzb + static_cast<int64_t>(p.row_cost) * a->nbr;
  const int sms = device_sm_count(device);
  // Two accumulator slots (double buffering between MMA and epilogue).
  const int need = 2 * nt * p.bm * rg;
  p.tmem_cols = 32;
  while (p.tmem_cols < static_cast<uint32_t>(need)) p.tmem_cols <<= 1;
  // Resident CTAs per SM: each has its own producer, MMA issuer and
  // epilogue, so one CTA's pipeline handoffs (stage commits, barrier waits,
  // row changes) overlap another's MMAs on the shared tensor pipe.  They
  // split the SM's shared memory and its 512 TMEM columns.
  if (cfg && (cfg->ctas_per_sm < 0 || cfg->ctas_per_sm > 4))
    return fail(KAIRO_STATUS_INVALID_VALUE, "ctas_per_sm must be between 0 and 4");
  // Packed stages (panels, then blocks side by side) for 16-row blocks: a
  // stage of consecutive stored blocks then arrives with one copy instead of
  // one per 512-byte block, whose copies bound the launch (65536^2 Zipf mask,
  // 16x16 blocks: 0.107 -> 0.098 ms).  Larger blocks keep one 1 KiB-aligned
  // slot per block, measured 0.5-1.5 % faster for 32x32 blocks.
  p.packed = (rg == 1 && p.bm == 16) ? 1 : 0;
  // Shared memory per block of a stage (packed: rounded up to 1 KiB per stage).
  const int sb = p.packed ? nt * 128 * p.bk * 2 + p.bm * p.bk * 2 : stage_bytes(p.bm, p.bk, nt, rg);
  const int reserve = 1024 /*alignment*/ + 1024 /*barriers and flags*/;
  int per_sm = (cfg && cfg->ctas_per_sm > 0) ? cfg->ctas_per_sm : default_ctas_per_sm(a, nt, sms);
  per_sm = std::max(1, std::min<int>(per_sm, static_cast<int>(512 / p.tmem_cols)));
  auto cta_budget = [&](int k) { return std::min(kMaxSmem, (kSmemPerSm - k * kSmemReservedPerCta) / k) - reserve; };
  while (per_sm > 1 && cta_budget(per_sm) < 2 * sb) --per_sm;
  const int budget = cta_budget(per_sm);
  p.ctas_per_sm = per_sm;
  int grid = (cfg && cfg->num_ctas > 0) ? cfg->num_ctas : sms * per_sm;
  if (grid > kCounterBankEntries) grid = kCounterBankEntries;
  // Smallest chunk group (a divisor of nchunks) whose counters fit one bank.
  p.chunk_group = p.nchunks;
  for (int cg = 1; cg <= p.nchunks; ++cg) {
    if (p.nchunks % cg) continue;
    if (static_cast<int64_t>(p.nchunks / cg) * grid <= kCounterBankEntries) {
      p.chunk_group = cg;
      break;
    }
  }
  p.ngroups = p.nchunks / p.chunk_group;
  const int64_t L = p.w * p.chunk_group;
  if (grid > L) grid = static_cast<int>(L);
  if (grid < 1) grid = 1;
  p.grid = grid;
  // Shared memory: `stages` groups of `group` block slots.  Prefer large
  // groups (fewer pipeline handoffs per block) while keeping enough groups
  // in flight to cover the load latency.
  int group = (cfg && cfg->group_blocks > 0) ? cfg->group_blocks : 0;
  if (group > 32) return fail(KAIRO_STATUS_INVALID_VALUE, "group_blocks must be at most 32");
  if (group == 0)
    group = default_group_blocks(budget / sb, b_slice_bytes(a, nt) > 0.5 * device_l2_bytes(device), per_sm);
  const int stage_total = tc_stage_bytes(p.bm, p.bk, nt, rg, group, p.packed != 0);
  int max_stages = budget / stage_total;
  if (max_stages > 32) max_stages = 32;
  int stages = (cfg && cfg->stages > 0) ? std::min(cfg->stages, max_stages) : max_stages;
  if (stages < 2) return fail(KAIRO_STATUS_NOT_SUPPORTED, "shared memory too small for two pipeline stages");
  p.group = group;
  p.stages = stages;
  p.smem_bytes = static_cast<size_t>(stages) * stage_total + reserve;
  p.counters_offset = kWorkspaceHeaderBytes;
  p.counters_bytes = kCounterRegionBytes;
  p.partials_offset = p.counters_offset + p.counters_bytes;
  p.partials_bytes = static_cast<size_t>(p.ngroups) * grid * 2 * nt * p.bm * rg * 128 * sizeof(float);
  p.workspace_bytes = p.partials_offset + p.partials_bytes;
  *plan = p;
  return KAIRO_STATUS_SUCCESS;
}

kairo_status tc_launch(const kairo_bsr* a, const void* b, int64_t ldb, int32_t layout, int64_t n, void* c,
                       int64_t ldc, kairo_dtype c_dtype, const TcPlan& plan, void* workspace, cudaStream_t stream) {
  const bool linear = layout == KAIRO_LAYOUT_LINEAR;
  KernelFn fn = pick_kernel(plan.bm, plan.nt, linear, a->dtype, c_dtype);
  if (!fn) return fail(KAIRO_STATUS_NOT_SUPPORTED, "no tcgen05 kernel for this block size / dtype combination");
  CUtensorMap map_a, map_b;
  int b_box3d = 0;
  kairo_status st = make_operand_maps(a, b, ldb, linear, n, plan.nt, &map_a, &map_b, &b_box3d);
  if (st) return st;
  // A stage of consecutive stored blocks as one copy of group * bm rows
  // (a TMA box is at most 256 rows).
  CUtensorMap map_run = map_a;
  int a_batch = 0;
  if (plan.packed && plan.group > 1 && plan.group * plan.bm <= 256) {
    // Optional: without this map every block is copied on its own.
    if (make_block_run_map(a, plan.group, &map_run) == KAIRO_STATUS_SUCCESS) {
      a_batch = 1;
    } else {
      map_run = map_a;
    }
  }

  TcArgs args{};
  args.row_ptr = a->row_ptr;
  args.col_idx = a->col_idx;
  args.blk_idx = a->blk_idx;
  args.c = c;
  args.ldc = ldc;
  args.w = plan.w;
  args.nblocks_stored = a->nblocks_stored;
  args.nnzb = a->nnzb;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  args.err = reinterpret_cast<unsigned*>(ws);
  const int bank = tc_next_counter_bank(workspace);
  unsigned* banks = reinterpret_cast<unsigned*>(ws + plan.counters_offset);
  args.counters = banks + bank * kCounterBankEntries;
  args.counters_other = banks + (1 - bank) * kCounterBankEntries;
  args.partials = reinterpret_cast<float*>(ws + plan.partials_offset);
  args.m = static_cast<int32_t>(a->rows);
  args.n = static_cast<int32_t>(n);
  args.nbr = a->nbr;
  args.nbc = static_cast<int32_t>(ceil_div64(a->cols, a->bk));
  args.chunk_group = plan.chunk_group;
  args.ngroups = plan.ngroups;
  args.row_cost = plan.row_cost;
  args.stages = plan.stages;
  args.group = plan.group;
  args.tmem_cols = plan.tmem_cols;
  const size_t osz = elem_size(c_dtype);
  args.b_box3d = b_box3d;
  args.hold_stage = plan.hold_stage;
  args.wait_cycles = plan.wait_cycles;
  args.vec_store = linear && ((reinterpret_cast<uintptr_t>(c) & 15u) == 0) && ((ldc * osz) % 16 == 0) ? 1 : 0;
  args.c_vec4 = !linear && ((reinterpret_cast<uintptr_t>(c) & 15u) == 0) && (ldc % 4 == 0) ? 1 : 0;
  args.packed = plan.packed;
  args.a_batch = a_batch;

  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(plan.smem_bytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  fn<<<plan.grid, kThreads, plan.smem_bytes, stream>>>(map_a, map_b, map_run, args);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the tcgen05 SpMM kernel");
  return KAIRO_STATUS_SUCCESS;
}

}  // namespace kairo
