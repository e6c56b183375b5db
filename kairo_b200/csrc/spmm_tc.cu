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
// Roles (192 threads, one CTA per SM, persistent):
//   warp 0      TMA producer: one A block + the matching B panel per stage;
//   warp 1      TMEM allocator and single-thread MMA issuer;
//   warps 2..5  epilogue: TMEM -> registers -> C, or -> a partial slot.
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
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <sstream>
#include <unordered_map>

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
};

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

template <int BM, int BK, int NT, bool LINEAR, int IN_FMT, typename TOut>
__global__ void __launch_bounds__(kThreads, 1)
    bsr_spmm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ CUtensorMap tmap_b, const TcArgs args) {
  constexpr int PANEL_BYTES = NT * 128 * BK * 2;
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int A_BYTES_PAD = (A_BYTES + 1023) / 1024 * 1024;
  constexpr int SLOT_BYTES = PANEL_BYTES + A_BYTES_PAD;  // one block + its B panel
  constexpr uint32_t TX_BYTES = PANEL_BYTES + A_BYTES;
  constexpr int ACC_COLS = NT * BM;  // one accumulator: NT sub-tiles of BM fp32 columns
  constexpr uint32_t IDESC = ptx::make_idesc_f16(IN_FMT, LINEAR ? 0u : 1u, 0u, 128u, BM);
  constexpr uint32_t SW_ROW = ptx::swizzle_code_for_row_bytes(BK * 2);
  constexpr int PART_ELEMS = NT * BM * 128;
  static_assert(BK % 16 == 0 && BM % 16 == 0 && BM <= 256, "block shape");
  static_assert(2 * ACC_COLS <= 512, "TMEM budget");
  const uint32_t TMEM_COLS = args.tmem_cols;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = args.stages;
  const int GB = args.group;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * GB * SLOT_BYTES);
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
          if (static_cast<unsigned>(mc) >= static_cast<unsigned>(args.nbc) ||
              mb < 0 || static_cast<int64_t>(mb) >= args.nblocks_stored) {
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
          uint8_t* st = smem + (gidx * GB + gpos + (lane - j0)) * SLOT_BYTES;
          ptx::mbar_expect_tx_if(mine, &full[gidx], TX_BYTES);
          ptx::tma_load_2d_if(mine, st + PANEL_BYTES, &tmap_a, 0, mb * BM, &full[gidx], pol_a);
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
    const uint64_t bdesc0 = ptx::make_smem_desc(sbase + PANEL_BYTES, 16, 8 * BK * 2, SW_ROW);
    const uint32_t a_lo0 = static_cast<uint32_t>(adesc0), a_hi = static_cast<uint32_t>(adesc0 >> 32);
    const uint32_t b_lo0 = static_cast<uint32_t>(bdesc0), b_hi = static_cast<uint32_t>(bdesc0 >> 32);
    constexpr uint32_t SLOT16 = SLOT_BYTES >> 4;
    uint32_t slot16 = 0;  // (byte offset of the current block slot) >> 4
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
          slot16 = static_cast<uint32_t>(midx * GB) * SLOT16;
        }
        // Blocks [p, p + seg) all live in the current stage group.
        const int seg = min(it.p1 - p, GB - mpos);
        const int p_end = p + seg;
#pragma unroll 2
        for (; p < p_end; ++p) {
          const uint32_t acc_any = (p != it.p0) ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              const uint32_t a_off = LINEAR ? (t * 128 * BK * 2 + kk * 32) : (t * 2 * BK * 128 + kk * 2048);
              ptx::mma_f16_ss_if(leader, d_base + t * BM, a_lo0 + slot16 + (a_off >> 4), a_hi,
                                 b_lo0 + slot16 + ((kk * 32) >> 4), b_hi, IDESC, (acc_any | (kk > 0)) ? 1u : 0u);
            }
          }
          slot16 += SLOT16;
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
      if (it.kind == kZero) {
        float z[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) z[jj] = 0.f;
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int j0 = 0; j0 < BM; j0 += 16) store16<LINEAR, TOut>(args, it.row, BM, j0, n0 + t * 128 + e, z);
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

// ---------------------------------------------------------------- host side

using KernelFn = void (*)(CUtensorMap, CUtensorMap, TcArgs);

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

// Counter bank of the next launch on `workspace` (alternates per workspace).
// The map is bounded: past kMaxTrackedWorkspaces entries it is cleared, and
// the next launch on a forgotten workspace uses bank 0.  That is safe after
// a launch that completed, which leaves both banks at zero (it zeroed the
// other bank and reset its own counters).  Only after an aborted launch
// (a recorded device error) can bank 0 still hold counters, which is why
// the banks alternate at all.
int next_counter_bank(void* workspace) {
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

}  // namespace

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
                     TcPlan* plan) {
  TcPlan p{};
  p.bm = a->bm;
  p.bk = a->bk;
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
  const int need = 2 * nt * p.bm;
  p.tmem_cols = 32;
  while (p.tmem_cols < static_cast<uint32_t>(need)) p.tmem_cols <<= 1;
  // Resident CTAs per SM: each has its own producer, MMA issuer and
  // epilogue, so one CTA's pipeline handoffs (stage commits, barrier waits,
  // row changes) overlap another's MMAs on the shared tensor pipe.  They
  // split the SM's shared memory and its 512 TMEM columns.
  if (cfg && (cfg->ctas_per_sm < 0 || cfg->ctas_per_sm > 4))
    return fail(KAIRO_STATUS_INVALID_VALUE, "ctas_per_sm must be between 0 and 4");
  const int sb = stage_bytes(p.bm, p.bk, nt);
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
  int max_stages = budget / (group * sb);
  if (max_stages > 32) max_stages = 32;
  int stages = (cfg && cfg->stages > 0) ? std::min(cfg->stages, max_stages) : max_stages;
  if (stages < 2) return fail(KAIRO_STATUS_NOT_SUPPORTED, "shared memory too small for two pipeline stages");
  p.group = group;
  p.stages = stages;
  p.smem_bytes = static_cast<size_t>(stages) * group * sb + reserve;
  p.counters_offset = kWorkspaceHeaderBytes;
  p.counters_bytes = kCounterRegionBytes;
  p.partials_offset = p.counters_offset + p.counters_bytes;
  p.partials_bytes = static_cast<size_t>(p.ngroups) * grid * 2 * nt * p.bm * 128 * sizeof(float);
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
  const int bank = next_counter_bank(workspace);
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

  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(plan.smem_bytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  fn<<<plan.grid, kThreads, plan.smem_bytes, stream>>>(map_a, map_b, args);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the tcgen05 SpMM kernel");
  return KAIRO_STATUS_SUCCESS;
}

}  // namespace kairo
