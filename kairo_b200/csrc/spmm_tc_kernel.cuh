// Persistent TMA + tcgen05 BSR SpMM for sm_100a.
//
// Math (reference: kairo/ops/spmm.py:108-134, csrc/acc_spmm_kernel.cu:33-107):
//   C[i*bm + r, n] = sum over blocks p of block-row i, in BSR order, of
//                    sum_k blocks[p][r][k] * B[col_idx[p]*bk + k, n]
// accumulated in fp32.
//
// Formulation.  A tcgen05 MMA needs M = 128 rows, but a block has only 16-64
// rows.  So the kernel computes the transposed product per block:
//   C^T[n0:n0+128, rows of block] += B^T_panel[n0:n0+128, bk] * block^T
// MMA M = 128 columns of C, MMA N = bm, MMA K = bk (bk/16 instructions).
//   operand A = the gathered B row-panel, read MN-major straight from the
//               row-major B (or K-major from X in the LINEAR layout);
//   operand B = the nonzero block, K-major (row-major block storage);
//   D in TMEM = 128 lanes (columns of C) x bm fp32 columns (rows of C).
//
// Roles (192 threads; one or more persistent CTAs per SM, each with its own
// share of shared memory and TMEM):
//   warp 0      TMA producer: a stage holds `group` blocks and their B panels,
//               one lane per block; packed stages (16-row blocks) copy a run
//               of consecutive stored blocks with one TMA copy;
//   warp 1      TMEM allocator and single-thread MMA issuer;
//   warps 2..5  epilogue: TMEM -> registers -> C, or -> a partial slot; a
//               block-row without blocks is zeroed with 16-byte stores.
// Smem stages are released by tcgen05.commit; two TMEM accumulator slots let
// the epilogue of one block-row overlap the MMAs of the next.
//
// Scheduler.  Work is a merge path over (block-row heads, blocks): block-row
// i costs `row_cost` units and each of its blocks one unit, so a chunk of 128*NT
// columns of C is a path of W = nnzb + row_cost*nbr units.  `chunk_group`
// consecutive chunks are concatenated and cut into gridDim.x equal ranges; all
// CTAs therefore sweep the chunks in the same order, which keeps the B columns
// of the current chunk resident in L2.  A block-row cut by a range boundary is
// computed in pieces: each piece goes to a partial slot, and the CTA that
// completes the row (an atomic arrival counter) adds the pieces in CTA order
// and writes C.  The result is deterministic for a given grid size.
//
// Every mbarrier wait is bounded (ptx::wait_parity): on timeout the kernel
// records KAIRO_DEVERR_WAIT_TIMEOUT in the workspace, drains its own copies
// and MMAs, frees TMEM and returns.
//
// This header holds the kernel template and its device-side scheduler; the
// host code that plans and launches it is spmm_tc.cu (one block-row per
// item) and spmm_stack.cu (groups of block-rows stacked into one MMA).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "internal.h"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace kairo {
namespace {

enum RowKind : int { kSkip = 0, kZero = 1, kDirect = 2, kPartial = 3 };

struct TcArgs {
  const int32_t* row_ptr;
  const int32_t* col_idx;
  const int32_t* blk_idx;
  void* c;
  int64_t ldc;
  int64_t w;               // path units per chunk
  int64_t nblocks_stored;
  int64_t nnzb;
  unsigned* err;
  unsigned* counters;      // this launch's bank: [ngroups][grid]
  unsigned* counters_other;  // the other bank, zeroed by this launch
  float* partials;         // [ngroups][grid][2][NT*BM*128]
  int32_t m;
  int32_t n;
  int32_t nbr;
  int32_t nbc;
  int32_t chunk_group;
  int32_t ngroups;
  int32_t row_cost;
  int32_t stages;          // stage groups in the shared-memory ring
  int32_t group;           // blocks per stage group
  uint32_t tmem_cols;      // TMEM columns allocated (power of two, >= 2*NT*BM)
  int32_t vec_store;       // LINEAR: rows of Y may be written with 16-byte stores
  int32_t b_box3d;         // STANDARD: the whole B panel is one 3D box (N % 64 == 0)
  int32_t hold_stage;      // test hook: hold back the first stage's arrival until the kernel aborts
  long long wait_cycles;   // bound of every mbarrier wait
  // Row groups (RG > 1): row_ptr / col_idx / blk_idx are the group pointer,
  // the column-block and the row mask of every stacked block, nbr / nnzb
  // count groups / stacked blocks, and these two tables complete them.
  const int32_t* stack_blk;  // [nnzb][RG]: stored-block index of each present block
  const int32_t* row_map;    // [nbr][RG]: block-row of each group slot, -1 past the last
  int32_t packed;            // RG = 1: a stage holds its B panels, then its blocks packed
  int32_t a_batch;           // packed: tmap_a_run copies a whole stage of consecutive blocks
  int32_t c_vec4;            // STANDARD: C rows may be written with 16-byte stores
};

// Writes zeros to rows i*BM .. i*BM+BM-1 and columns n0 .. n0+NT*128-1 of
// the row-major fp32 C (clamped to M x N), for a block-row without blocks:
// the 128 epilogue threads (t = 0..127) store 16-byte vectors, a warp 512
// contiguous bytes of one row.
template <int BM, int NT>
__device__ __forceinline__ void zero_c_rows(const TcArgs& a, int i, int n0, int t) {
  float* c = static_cast<float*>(a.c);
  constexpr int V = NT * 32;  // 16-byte vectors per row of the item
#pragma unroll
  for (int q = t; q < BM * V; q += 128) {
    const int r = i * BM + q / V;
    const int col = n0 + (q % V) * 4;
    if (r >= a.m || col >= a.n) continue;
    float* dst = c + static_cast<int64_t>(r) * a.ldc + col;
    if (a.c_vec4 && col + 4 <= a.n) {
      __stcs(reinterpret_cast<float4*>(dst), make_float4(0.f, 0.f, 0.f, 0.f));
    } else {
      for (int u = 0; u < 4 && col + u < a.n; ++u) __stcs(dst + u, 0.f);
    }
  }
}

struct RowItem {
  int chunk;       // global chunk index
  int group;
  int row;
  int p0, p1;      // blocks of this piece
  int kind;        // RowKind
  int slot;        // partial slot this CTA writes (0 head, 1 tail)
  int b_lo, b_hi;  // contributing CTAs of a split row
  int lo_slot;     // slot used by b_lo
};

// Largest i in [0, nbr) with row_ptr[i] + R*i <= target, found by the whole
// CTA with a (blockDim)-ary search; every thread returns the same value.
__device__ int cta_find_row(const int32_t* __restrict__ row_ptr, int nbr, int R, int64_t target) {
  int lo = 0, hi = nbr;
  const int T = blockDim.x;
  while (hi - lo > 1) {
    const int span = hi - lo;
    const int np = min(T, span - 1);
    const int t = threadIdx.x;
    bool pred = false;
    if (t < np) {
      const int idx = lo + 1 + static_cast<int>(static_cast<int64_t>(t) * (span - 1) / np);
      pred = static_cast<int64_t>(__ldg(row_ptr + idx)) + static_cast<int64_t>(R) * idx <= target;
    }
    const int cnt = __syncthreads_count(pred);
    const int nlo = cnt > 0 ? lo + 1 + static_cast<int>(static_cast<int64_t>(cnt - 1) * (span - 1) / np) : lo;
    const int nhi = cnt < np ? lo + 1 + static_cast<int>(static_cast<int64_t>(cnt) * (span - 1) / np) : hi;
    lo = nlo;
    hi = nhi;
  }
  return lo;
}

// Walks this CTA's share of the work in launch order and calls f(item) for
// every (chunk, block-row) piece it touches.  Warp-uniform: all 32 lanes call
// f with the same item.  Returns false as soon as f returns false.
template <class F>
__device__ __forceinline__ bool walk_items(const TcArgs& a, int64_t s, int64_t e, int i_start,
                                           int lane, F&& f) {
  const int G = gridDim.x;
  const int b = blockIdx.x;
  const int64_t W = a.w;
  const int64_t R = a.row_cost;
  const int64_t L = W * a.chunk_group;
  const int32_t* __restrict__ row_ptr = a.row_ptr;
  const int64_t j_first = s / W;
  const int64_t j_last = (e - 1) / W;
  for (int g = 0; g < a.ngroups; ++g) {
    for (int64_t jl = j_first; jl <= j_last; ++jl) {
      const int64_t ls = max(s, jl * W) - jl * W;
      const int64_t le = min(e, (jl + 1) * W) - jl * W;
      int i = (jl == j_first) ? i_start : 0;
      int base = -64, v = 0, v32 = 0;
      while (i < a.nbr) {
        if (i - base >= 32) {
          base = i;
          v = __ldg(row_ptr + min(base + lane, a.nbr));
          v32 = __ldg(row_ptr + min(base + 32, a.nbr));
        }
        const int k = i - base;
        const int r0 = __shfl_sync(0xffffffffu, v, k);
        const int r1n = __shfl_sync(0xffffffffu, v, min(k + 1, 31));
        const int r1 = (k == 31) ? v32 : r1n;
        const int64_t P = static_cast<int64_t>(r0) + R * i;
        if (P >= le) break;
        RowItem it;
        it.chunk = g * a.chunk_group + static_cast<int>(jl);
        it.group = g;
        it.row = i;
        it.slot = 0;
        it.b_lo = it.b_hi = b;
        it.lo_slot = 0;
        const int64_t shift = R * (i + 1);  // block p sits at path position p + shift
        if (r1 == r0) {
          it.kind = (P >= ls) ? kZero : kSkip;
          it.p0 = it.p1 = r0;
        } else {
          const int64_t q0 = max(static_cast<int64_t>(r0), ls - shift);
          const int64_t q1 = min(static_cast<int64_t>(r1), le - shift);
          it.p0 = static_cast<int>(q0);
          it.p1 = static_cast<int>(q1);
          if (q0 >= q1) {
            it.kind = kSkip;
          } else if (q0 == r0 && q1 == r1) {
            it.kind = kDirect;
          } else {
            it.kind = kPartial;
            it.slot = (jl == j_first && i == i_start) ? 0 : 1;
            const int64_t off = jl * W;
            const int64_t d_first = off + r0 + shift;
            const int64_t d_last = off + r1 - 1 + shift;
            it.b_lo = static_cast<int>(((d_first + 1) * G - 1) / L);
            it.b_hi = static_cast<int>(((d_last + 1) * G - 1) / L);
            const int64_t s_lo = static_cast<int64_t>(it.b_lo) * L / G;
            it.lo_slot = (s_lo >= off + P) ? 0 : 1;
          }
        }
        if (it.kind != kSkip) {
          if (!f(it)) return false;
        }
        ++i;
      }
    }
  }
  return true;
}

// RG = 1: one block-row per item.  RG > 1: row groups.  An item is a group
// of RG block-rows (rows of similar length, chosen by kairo_bsr_stack_build)
// and its "blocks" are the group's distinct column-blocks: one stage slot
// holds that column's B panel once and the group's blocks there side by
// side (slot r at r * bm rows), so the blocks of consecutive group rows
// that share the column form one K-major operand of (run length) * bm rows
// and are multiplied by one MMA of N = run * bm into consecutive
// accumulator columns.  The accumulator is zeroed in TMEM (at start and by
// the epilogue after each read), so every MMA accumulates.
template <int BM, int BK, int NT, bool LINEAR, int IN_FMT, typename TOut, int RG = 1>
__global__ void __launch_bounds__(kThreads, 1)
    bsr_spmm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ CUtensorMap tmap_b,
                       const __grid_constant__ CUtensorMap tmap_a_run, const TcArgs args) {
  constexpr int PANEL_BYTES = NT * 128 * BK * 2;
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int A_BYTES_PAD = (RG * A_BYTES + 1023) / 1024 * 1024;
  constexpr int SLOT_BYTES = PANEL_BYTES + A_BYTES_PAD;  // a B panel and its block (RG blocks), unpacked stages
  constexpr uint32_t TX_BYTES = PANEL_BYTES + A_BYTES;
  constexpr int BME = BM * RG;        // accumulator columns of one 128-column sub-tile
  constexpr int ACC_COLS = NT * BME;  // one accumulator: NT sub-tiles of BME fp32 columns
  constexpr uint32_t IDESC = ptx::make_idesc_f16(IN_FMT, LINEAR ? 0u : 1u, 0u, 128u, BM);
  constexpr uint32_t SW_ROW = ptx::swizzle_code_for_row_bytes(BK * 2);
  constexpr int PART_ELEMS = NT * BME * 128;
  static_assert(BK % 16 == 0 && BM % 16 == 0 && BM <= 256, "block shape");
  static_assert(2 * ACC_COLS <= 512, "TMEM budget");
  static_assert(RG == 1 || (!LINEAR && RG <= 16 && BME <= 256), "row groups: STANDARD layout, N <= 256");
  const uint32_t TMEM_COLS = args.tmem_cols;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = args.stages;
  const int GB = args.group;
  // A stage holds GB blocks: GB slots of a B panel and its block (RG > 1:
  // RG blocks), each slot padded to 1 KiB, or, packed (RG = 1), the GB
  // panels and then the GB blocks side by side, so that consecutive stored
  // blocks arrive with one copy.
  const bool packed = RG == 1 && args.packed;
  const uint32_t STAGE_BYTES = static_cast<uint32_t>(tc_stage_bytes(BM, BK, NT, RG, GB, packed));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * STAGE_BYTES);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  int* misc = reinterpret_cast<int*>(mma_done + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 0);
  volatile int* abort_flag = misc + 1;
  int* red_flag = misc + 3;
  int* issued = misc + 4;  // [S]: parity+1 of the last group loaded into each stage

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
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
    misc[2] = 0;
    ptx::mbar_init_fence();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_a);
    if (packed && args.a_batch) ptx::prefetch_tmap(&tmap_a_run);
    ptx::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, TMEM_COLS);
    ptx::tmem_relinquish();
  }

  // Clear the counter bank the next launch on this workspace will use.
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < kCounterBankEntries; i += gridDim.x * kThreads)
    args.counters_other[i] = 0u;

  const int G = gridDim.x;
  const int64_t L = args.w * args.chunk_group;
  const int64_t s_range = static_cast<int64_t>(blockIdx.x) * L / G;
  const int64_t e_range = static_cast<int64_t>(blockIdx.x + 1) * L / G;
  const int64_t ls0 = s_range - (s_range / args.w) * args.w;
  const int i_start = cta_find_row(args.row_ptr, args.nbr, args.row_cost, ls0);

  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if constexpr (RG > 1) {
    // Row groups accumulate into zeroed TMEM (see above): clear both slots.
    if (warp >= 2) {
      const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) * 32) << 16;
      for (int c0 = 0; c0 < 2 * ACC_COLS; c0 += 16) ptx::tmem_st16_zero(tmem_base + lane_addr + c0);
      ptx::tmem_wait_st();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Blocks are loaded in groups of GB consecutive blocks per stage: one
    // lane per block issues that block's two TMA loads, so a whole group is
    // issued by a couple of warp instructions, and the group's full barrier
    // gets a single arrival once every block of it has its expect_tx.  The
    // warp stays converged: waits are polled by all lanes and single-lane
    // instructions are predicated, never branched around.
    const uint64_t pol_a = ptx::policy_evict_first();
    const uint64_t pol_b = ptx::policy_evict_last();
    const uint32_t leader = lane == 0 ? 1u : 0u;
    int gpos = 0;      // next slot in the current group
    int gidx = 0;      // stage of the current group
    uint32_t gph = 0;  // phase of that stage
    IndexWindow win;
    // Test hook (args.hold_stage): the first stage's arrival waits until a
    // consumer's bounded wait has run out and set the abort flag, or for
    // four wait bounds at most; then it arrives, so that the stage's phase
    // completes once its loads have landed and the drain below finds them.
    bool held = args.hold_stage == 0;
    auto hold_first_arrival = [&]() {
      if (held) return;
      held = true;
      const long long t0 = clock64();
      while (!*abort_flag && clock64() - t0 < 4 * args.wait_cycles) __nanosleep(256);
      __syncwarp();
    };
    walk_items(args, s_range, e_range, i_start, lane, [&](const RowItem& it) -> bool {
      if (it.kind != kDirect && it.kind != kPartial) return true;
      const int n0 = it.chunk * NT * 128;
      for (int pb = it.p0; pb < it.p1; pb += 32) {
        const int cnt = min(32, it.p1 - pb);
        int mc = 0, mb = 0;
        win.ensure(args.col_idx, args.blk_idx, args.nnzb, pb, lane);
        win.get(pb + lane, mc, mb);
        if (lane < cnt) {
          // RG > 1: mb is the group-row mask of the stacked block.
          const bool bad_b = RG > 1 ? (static_cast<uint32_t>(mb) >> RG) != 0u
                                    : (mb < 0 || static_cast<int64_t>(mb) >= args.nblocks_stored);
          if (static_cast<unsigned>(mc) >= static_cast<unsigned>(args.nbc) || bad_b) {
            atomicCAS(args.err, 0u, KAIRO_DEVERR_BAD_INDEX);
            mc = 0;
            mb = 0;
          }
        } else {
          mc = 0;
          mb = 0;
        }
        int j0 = 0;
        while (j0 < cnt) {
          const int take = min(GB - gpos, cnt - j0);
          if (gpos == 0) {
            int ok = ptx::wait_parity(&empty[gidx], gph ^ 1u, abort_flag, args.err, kTagEmpty, args.wait_cycles);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) return false;
            if (lane == 0) issued[gidx] = static_cast<int>(gph) + 1;
          }
          const uint32_t mine = (lane >= j0 && lane < j0 + take) ? 1u : 0u;
          uint8_t* stage = smem + gidx * STAGE_BYTES;
          const int js = gpos + (lane - j0);  // this lane's block slot in the stage
          uint8_t* st = packed ? stage + js * PANEL_BYTES : stage + js * SLOT_BYTES;  // its B panel
          if constexpr (RG == 1) {
            ptx::mbar_expect_tx_if(mine, &full[gidx], TX_BYTES);
            // A whole stage of consecutive stored blocks (a long block-row
            // with identity block order) arrives with one copy of GB * BM
            // rows; otherwise each lane copies its block.
            const int mb0 = __shfl_sync(0xffffffffu, mb, j0);
            const bool run = packed && args.a_batch && gpos == 0 && take == GB &&
                             __all_sync(0xffffffffu, !mine || mb == mb0 + (lane - j0));
            uint8_t* blocks = stage + GB * PANEL_BYTES;
            if (run) {
              ptx::tma_load_2d_if(lane == j0 ? 1u : 0u, blocks, &tmap_a_run, 0, mb0 * BM, &full[gidx], pol_a);
            } else {
              ptx::tma_load_2d_if(mine, packed ? blocks + js * A_BYTES : st + PANEL_BYTES, &tmap_a, 0, mb * BM,
                                  &full[gidx], pol_a);
            }
          } else {
            // The panel plus the group's present blocks, block of slot r at
            // r * A_BYTES.
            const uint32_t mask = mine ? static_cast<uint32_t>(mb) : 0u;
            ptx::mbar_expect_tx_if(mine, &full[gidx],
                                   static_cast<uint32_t>(PANEL_BYTES) + __popc(mask) * static_cast<uint32_t>(A_BYTES));
            const int32_t* sb = args.stack_blk + static_cast<int64_t>(pb + lane) * RG;
#pragma unroll
            for (int r = 0; r < RG; ++r) {
              const uint32_t has = (mask >> r) & 1u;
              int blk = has ? __ldg(sb + r) : 0;
              if (has && (blk < 0 || static_cast<int64_t>(blk) >= args.nblocks_stored)) {
                atomicCAS(args.err, 0u, KAIRO_DEVERR_BAD_INDEX);
                blk = 0;
              }
              ptx::tma_load_2d_if(has, st + PANEL_BYTES + r * A_BYTES, &tmap_a, 0, blk * BM, &full[gidx], pol_a);
            }
          }
          if (LINEAR) {
            // X rows n0 .. n0+128*NT as one box: sub-tile t lands at t*128*BK*2.
            ptx::tma_load_2d_if(mine, st, &tmap_b, mc * BK, n0, &full[gidx], pol_b);
          } else if (args.b_box3d) {
            // B viewed as [N/64][K][64]: the 2*NT column atoms of the
            // panel arrive as [atom][k][64] in one box.
            ptx::tma_load_3d_if(mine, st, &tmap_b, 0, mc * BK, n0 / 64, &full[gidx], pol_b);
          } else {
#pragma unroll
            for (int h = 0; h < 2 * NT; ++h)
              ptx::tma_load_2d_if(mine, st + h * BK * 128, &tmap_b, n0 + 64 * h, mc * BK, &full[gidx], pol_b);
          }
          __syncwarp();
          gpos += take;
          j0 += take;
          if (gpos == GB) {
            hold_first_arrival();
            ptx::mbar_arrive_if(leader, &full[gidx]);
            gpos = 0;
            if (++gidx == S) {
              gidx = 0;
              gph ^= 1u;
            }
          }
        }
      }
      return true;
    });
    // Close a partly filled last group (also after an abort, so that the
    // loads already issued can complete its phase before the drain below).
    if (gpos != 0) {
      hold_first_arrival();
      ptx::mbar_arrive_if(leader, &full[gidx]);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (uniform control flow); lane 0 is the
    // only one whose MMA / commit instructions are enabled.  Descriptors are
    // built once and advanced by adding (byte offset >> 4) to their
    // start-address field.
    const uint32_t leader = lane == 0 ? 1u : 0u;
    int mpos = 0, midx = 0;
    uint32_t mph = 0;
    int slot = 0;
    uint32_t aphase = 0;
    const uint32_t sbase = ptx::smem_u32(smem);
    const uint64_t adesc0 = LINEAR ? ptx::make_smem_desc(sbase, 16, 8 * BK * 2, SW_ROW)
                                   : ptx::make_smem_desc(sbase, BK * 128, 1024, 2u);
    const uint64_t bdesc0 = ptx::make_smem_desc(sbase, 16, 8 * BK * 2, SW_ROW);
    const uint32_t a_lo0 = static_cast<uint32_t>(adesc0), a_hi = static_cast<uint32_t>(adesc0 >> 32);
    const uint32_t b_lo0 = static_cast<uint32_t>(bdesc0), b_hi = static_cast<uint32_t>(bdesc0 >> 32);
    constexpr uint32_t SLOT16 = SLOT_BYTES >> 4;
    constexpr uint32_t PANEL16 = PANEL_BYTES >> 4;
    const uint32_t PAN_STEP16 = packed ? PANEL16 : SLOT16;
    const uint32_t BLK_STEP16 = packed ? static_cast<uint32_t>(A_BYTES >> 4) : SLOT16;
    uint32_t pan16 = 0;  // (byte offset of the current block's B panel) >> 4
    uint32_t blk16 = 0;  // (byte offset of the current block) >> 4
    walk_items(args, s_range, e_range, i_start, lane, [&](const RowItem& it) -> bool {
      if (it.kind != kDirect && it.kind != kPartial) return true;
      int ok = ptx::wait_parity(&tempty[slot], aphase ^ 1u, abort_flag, args.err, kTagTmemEmpty, args.wait_cycles);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) return false;
      ptx::tc_fence_after();
      const uint32_t d_base = tmem_base + static_cast<uint32_t>(slot * ACC_COLS);
      int p = it.p0;
      while (p < it.p1) {
        if (mpos == 0) {
          // No tcgen05 fence here: the MMAs read shared memory the TMA wrote,
          // and the mbarrier wait itself orders them after those writes.
          ok = ptx::wait_parity(&full[midx], mph, abort_flag, args.err, kTagFull, args.wait_cycles);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) return false;
          pan16 = (static_cast<uint32_t>(midx) * STAGE_BYTES) >> 4;
          blk16 = pan16 + (packed ? static_cast<uint32_t>(GB) * PANEL16 : PANEL16);
        }
        // Blocks [p, p + seg) all live in the current stage group.
        const int seg = min(it.p1 - p, GB - mpos);
        const int p_end = p + seg;
        if constexpr (RG == 1) {
#pragma unroll 2
          for (; p < p_end; ++p) {
            const uint32_t acc_any = (p != it.p0) ? 1u : 0u;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                const uint32_t a_off = LINEAR ? (t * 128 * BK * 2 + kk * 32) : (t * 2 * BK * 128 + kk * 2048);
                ptx::mma_f16_ss_if(leader, d_base + t * BM, a_lo0 + pan16 + (a_off >> 4), a_hi,
                                   b_lo0 + blk16 + ((kk * 32) >> 4), b_hi, IDESC, (acc_any | (kk > 0)) ? 1u : 0u);
              }
            }
            pan16 += PAN_STEP16;
            blk16 += BLK_STEP16;
          }
        } else {
          // One MMA per run of consecutive group rows present in this
          // column: N = run * BM, into the run's accumulator columns.  The
          // mask is read by every lane, so the loop stays warp-uniform.
          for (; p < p_end; ++p) {
            uint32_t mask = static_cast<uint32_t>(__ldg(args.blk_idx + p)) & ((1u << RG) - 1u);
            while (mask) {
              const int r0 = __ffs(mask) - 1;
              const int len = __ffs(~(mask >> r0)) - 1;
              mask &= ~(((1u << len) - 1u) << r0);
              const uint32_t idesc = ptx::make_idesc_f16(IN_FMT, 1u, 0u, 128u, static_cast<uint32_t>(len * BM));
#pragma unroll
              for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                  const uint32_t a_off = t * 2 * BK * 128 + kk * 2048;
                  ptx::mma_f16_ss_if(leader, d_base + t * BME + r0 * BM, a_lo0 + pan16 + (a_off >> 4), a_hi,
                                     b_lo0 + blk16 + ((r0 * A_BYTES + kk * 32) >> 4), b_hi, idesc, 1u);
                }
              }
            }
            pan16 += PAN_STEP16;
            blk16 += BLK_STEP16;
          }
        }
        mpos += seg;
        if (mpos == GB) {
          ptx::mma_commit_if(leader, &empty[midx]);
          mpos = 0;
          if (++midx == S) {
            midx = 0;
            mph ^= 1u;
          }
        }
      }
      ptx::mma_commit_if(leader, &tfull[slot]);
      slot ^= 1;
      if (slot == 0) aphase ^= 1u;
      return true;
    });
    // Every MMA issued above has completed once mma_done flips.
    if (mpos != 0) ptx::mma_commit_if(leader, &empty[midx]);
    ptx::mma_commit_if(leader, mma_done);
    int dummy = 0;
    ptx::wait_parity(mma_done, 0, reinterpret_cast<volatile int*>(&dummy), args.err, kTagDrain, args.wait_cycles);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int e = q * 32 + lane;     // TMEM lane == column within a 128-wide sub-tile
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    int slot = 0;
    uint32_t aphase = 0;
    walk_items(args, s_range, e_range, i_start, lane, [&](const RowItem& it) -> bool {
      const int n0 = it.chunk * NT * 128;
      if constexpr (RG > 1) {
        // Row groups: slot r of the group is block-row row_map[r] of C (or
        // padding when negative); each slot is read, zeroed in TMEM for the
        // next item, and stored (or written to the partial tile).
        const int32_t* rmap = args.row_map + static_cast<int64_t>(it.row) * RG;
        if (it.kind == kZero) {
          for (int r = 0; r < RG; ++r) {
            const int orow = __ldg(rmap + r);
            if (orow >= 0) zero_c_rows<BM, NT>(args, orow, n0, threadIdx.x - 64);
          }
          return true;
        }
        int ok = ptx::wait_parity(&tfull[slot], aphase, abort_flag, args.err, kTagTmemFull, args.wait_cycles, 200);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (epi_any(!ok)) return false;
        ptx::tc_fence_after();
        float* part = nullptr;
        if (it.kind == kPartial)
          part = args.partials + (static_cast<int64_t>(it.group * G + blockIdx.x) * 2 + it.slot) * PART_ELEMS;
        const uint32_t slot_cols = static_cast<uint32_t>(slot * ACC_COLS);
        for (int r = 0; r < RG; ++r) {
          const int orow = __ldg(rmap + r);
          if (orow < 0) continue;
#pragma unroll
          for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int j0 = 0; j0 < BM; j0 += 16) {
              const uint32_t col = slot_cols + static_cast<uint32_t>(t * BME + r * BM + j0);
              float v[16];
              ptx::tmem_ld16(tmem_base + lane_addr + col, v);
              ptx::tmem_wait_ld();
              ptx::tmem_st16_zero(tmem_base + lane_addr + col);
              if (it.kind == kDirect) {
                store16<false, TOut>(args, orow, BM, j0, n0 + t * 128 + e, v);
              } else {
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) part[(t * BME + r * BM + j0 + jj) * 128 + e] = v[jj];
              }
            }
          }
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&tempty[slot]);
        slot ^= 1;
        if (slot == 0) aphase ^= 1u;
        if (it.kind == kPartial) {
          __threadfence();
          epi_bar();
          if (threadIdx.x == 64) {
            const unsigned old = atomicAdd(args.counters + it.group * G + it.b_lo, 1u);
            *red_flag = (old == static_cast<unsigned>(it.b_hi - it.b_lo)) ? 1 : 0;
          }
          epi_bar();
          if (*red_flag) {
            __threadfence();
            // The pieces are summed in CTA order, 32 values of a thread at a
            // time (a group's rows can be cut into tens of pieces: the
            // loads of one piece are issued together).
            constexpr int FLAT = NT * BME;
            constexpr int CH = FLAT < 32 ? FLAT : 32;
            for (int f0 = 0; f0 < FLAT; f0 += CH) {
              float acc[CH];
#pragma unroll
              for (int i = 0; i < CH; ++i) acc[i] = 0.f;
              for (int bb = it.b_lo; bb <= it.b_hi; ++bb) {
                const int sl = (bb == it.b_lo) ? it.lo_slot : 0;
                const float* src = args.partials + (static_cast<int64_t>(it.group * G + bb) * 2 + sl) * PART_ELEMS;
#pragma unroll
                for (int i = 0; i < CH; ++i) acc[i] += __ldcg(src + (f0 + i) * 128 + e);
              }
#pragma unroll
              for (int i = 0; i < CH; i += 16) {
                const int f = f0 + i, t = f / BME, col = f % BME;
                const int orow = __ldg(rmap + col / BM);
                if (orow >= 0) store16<false, TOut>(args, orow, BM, col % BM, n0 + t * 128 + e, acc + i);
              }
            }
            if (threadIdx.x == 64) atomicExch(args.counters + it.group * G + it.b_lo, 0u);
          }
        }
        return true;
      }
      if (it.kind == kZero) {
        if constexpr (!LINEAR) {
          zero_c_rows<BM, NT>(args, it.row, n0, threadIdx.x - 64);
        } else {
          float z[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) z[jj] = 0.f;
#pragma unroll
          for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int j0 = 0; j0 < BM; j0 += 16) store16<LINEAR, TOut>(args, it.row, BM, j0, n0 + t * 128 + e, z);
        }
        return true;
      }
      int ok = ptx::wait_parity(&tfull[slot], aphase, abort_flag, args.err, kTagTmemFull, args.wait_cycles, 200);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (epi_any(!ok)) return false;
      ptx::tc_fence_after();
      float* part = nullptr;
      if (it.kind == kPartial)
        part = args.partials + (static_cast<int64_t>(it.group * G + blockIdx.x) * 2 + it.slot) * PART_ELEMS;
      const uint32_t slot_cols = static_cast<uint32_t>(slot * ACC_COLS);
      if constexpr (ACC_COLS <= 64) {
        // The whole accumulator (up to 64 values per thread) is loaded with
        // back-to-back TMEM loads and one wait, and its slot is released
        // before the stores to C, so the MMA warp can reuse it while they
        // drain.  With short block-rows the epilogue is otherwise what the
        // MMA warp waits for.
        float v[ACC_COLS];
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int j0 = 0; j0 < BM; j0 += 16)
            ptx::tmem_ld16(tmem_base + lane_addr + slot_cols + static_cast<uint32_t>(t * BM + j0), v + t * BM + j0);
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&tempty[slot]);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
          for (int j0 = 0; j0 < BM; j0 += 16) {
            if (it.kind == kDirect) {
              store16<LINEAR, TOut>(args, it.row, BM, j0, n0 + t * 128 + e, v + t * BM + j0);
            } else {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) part[(t * BM + j0 + jj) * 128 + e] = v[t * BM + j0 + jj];
            }
          }
        }
      } else {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
          for (int j0 = 0; j0 < BM; j0 += 16) {
            float v[16];
            ptx::tmem_ld16(tmem_base + lane_addr + slot_cols + static_cast<uint32_t>(t * BM + j0), v);
            ptx::tmem_wait_ld();
            if (it.kind == kDirect) {
              store16<LINEAR, TOut>(args, it.row, BM, j0, n0 + t * 128 + e, v);
            } else {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) part[(t * BM + j0 + jj) * 128 + e] = v[jj];
            }
          }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&tempty[slot]);
      }
      slot ^= 1;
      if (slot == 0) aphase ^= 1u;
      if (it.kind == kPartial) {
        __threadfence();
        epi_bar();
        if (threadIdx.x == 64) {
          const unsigned old = atomicAdd(args.counters + it.group * G + it.b_lo, 1u);
          *red_flag = (old == static_cast<unsigned>(it.b_hi - it.b_lo)) ? 1 : 0;
        }
        epi_bar();
        if (*red_flag) {
          __threadfence();
#pragma unroll
          for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int j0 = 0; j0 < BM; j0 += 16) {
              float acc[16];
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) acc[jj] = 0.f;
              for (int bb = it.b_lo; bb <= it.b_hi; ++bb) {
                const int sl = (bb == it.b_lo) ? it.lo_slot : 0;
                const float* src = args.partials + (static_cast<int64_t>(it.group * G + bb) * 2 + sl) * PART_ELEMS;
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) acc[jj] += __ldcg(src + (t * BM + j0 + jj) * 128 + e);
              }
              store16<LINEAR, TOut>(args, it.row, BM, j0, n0 + t * 128 + e, acc);
            }
          }
          if (threadIdx.x == 64) atomicExch(args.counters + it.group * G + it.b_lo, 0u);
        }
      }
      return true;
    });
  }

  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
    // A wait gave up: let the loads this CTA issued land before it exits.
    int dummy = 0;
    for (int s = 0; s < S; ++s)
      if (issued[s])
        ptx::wait_parity(&full[s], static_cast<uint32_t>(issued[s] - 1), reinterpret_cast<volatile int*>(&dummy),
                         args.err, kTagDrain, args.wait_cycles);
  }
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace
}  // namespace kairo
