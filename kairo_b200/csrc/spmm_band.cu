// Band-schedule TMA + tcgen05 BSR SpMM for sm_100a.
//
// Math and MMA formulation are those of spmm_tc.cu (reference:
// kairo/ops/spmm.py:108-134): per nonzero block, C^T[n0:n0+128, rows of the
// block] += B^T_panel * block^T, with MMA M = 128 columns of C, N = bm and
// K = bk, fp32 accumulation in TMEM.
//
// Why a second schedule.  When the B slice of one chunk of C columns
// (K x 128*nt elements) is larger than L2, the row-split schedule reads most
// gathered B panels from HBM: the CTAs work on unrelated block-rows, so a
// panel is rarely still cached when the next block of its column comes by.
// Here every CTA keeps `rows` block-rows open at once (one TMEM accumulator
// each) and visits their blocks in column order.  All CTAs start their items
// together and sweep the columns at about the same pace, so a B panel fetched
// for one CTA is read from L2 by the others that need it in the same sweep.
// Odd waves of items sweep downwards (serpentine), starting where L2 still
// holds the end of the previous sweep.
//
// Work.  An item is (chunk of 128*nt columns of C, group of R consecutive
// block-rows); items are numbered chunk-major and dealt round-robin to the
// persistent CTAs, so wave k = items [k*grid, (k+1)*grid) covers R*grid
// consecutive block-rows of one chunk.  A block-row is never split: the
// schedule suits masks whose block-rows have similar lengths.  It runs when
// the caller asks for it (kairo_spmm_config.schedule); on the uniform
// 262144^2 mask it moves 13 % fewer DRAM bytes than the row-split schedule
// but is limited by the same per-SM TMA gather rate, so it is not the default.
//
// Column order.  A pre-pass (band_order_kernel) writes, for every BSR
// position of an item, the key (col << 40) | (row slot << 32) | stored block
// index, sorted by key within the item (items of more than kOrderSortCap
// blocks keep BSR order).  The summation order of a row is thus its column
// order: results match the oracle within fp32 rounding, not bit for bit.
//
// Roles (192 threads): warp 0 TMA producer (also writes each block's row slot
// into the stage's metadata), warp 1 TMEM allocator + MMA issuer, warps 2..5
// epilogue.  Every mbarrier wait is bounded as in spmm_tc.cu.
#include <cuda.h>

#include <algorithm>
#include <sstream>

#include "internal.h"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace kairo {
namespace {

constexpr int kOrderSortCap = 2048;  // blocks per item sorted by column; larger items keep BSR order
constexpr int kOrderThreads = 256;
constexpr int kMaxBandRows = 32;     // row slots fit a 32-bit "started" mask

struct BandArgs {
  const int32_t* row_ptr;
  const uint64_t* order;  // per BSR position: (col << 40) | (row slot << 32) | stored block index
  void* c;
  int64_t ldc;
  int64_t nitems;
  int64_t nblocks_stored;
  unsigned* err;
  int32_t m;
  int32_t n;
  int32_t nbr;
  int32_t nbc;
  int32_t nnzb;
  int32_t rows;        // R
  int32_t row_groups;  // ceil(nbr / R)
  int32_t stages;
  int32_t group;
  int32_t acc_slots;
  int32_t serpentine;
  uint32_t tmem_cols;
  int32_t vec_store;
  int32_t b_box3d;
  long long wait_cycles;  // bound of every mbarrier wait
};

// ------------------------------------------------------------ column order
// One CTA per row group (grid-stride).  Keys of the group's blocks are built
// in shared memory and bitonic-sorted; ids outside the block grid are
// recorded as KAIRO_DEVERR_BAD_INDEX and replaced by block 0 / column 0, and
// so are row offsets outside [0, nnzb] (those groups are clamped).
__global__ void __launch_bounds__(kOrderThreads)
    band_order_kernel(const int32_t* __restrict__ row_ptr, const int32_t* __restrict__ col_idx,
                      const int32_t* __restrict__ blk_idx, int32_t nbr, int32_t nbc, int32_t nnzb,
                      int64_t nblocks_stored, int32_t R, int32_t Q, uint64_t* __restrict__ order, unsigned* err) {
  __shared__ uint64_t keys[kOrderSortCap];
  __shared__ int32_t rp[kMaxBandRows + 1];
  for (int q = blockIdx.x; q < Q; q += gridDim.x) {
    const int r0 = q * R;
    const int nr = min(R, nbr - r0);
    for (int i = threadIdx.x; i <= nr; i += blockDim.x) {
      const int v = row_ptr[r0 + i];
      const int cv = min(max(v, 0), nnzb);
      if (cv != v) atomicCAS(err, 0u, KAIRO_DEVERR_BAD_INDEX);
      rp[i] = cv;
    }
    __syncthreads();
    if (threadIdx.x == 0)
      for (int i = 1; i <= nr; ++i)
        if (rp[i] < rp[i - 1]) {
          atomicCAS(err, 0u, KAIRO_DEVERR_BAD_INDEX);
          rp[i] = rp[i - 1];
        }
    __syncthreads();
    const int p0 = rp[0];
    const int cnt = rp[nr] - p0;
    const bool sorted = cnt <= kOrderSortCap;
    int npow = 1;
    while (npow < cnt) npow <<= 1;
    const int span = sorted ? npow : cnt;
    for (int i = threadIdx.x; i < span; i += blockDim.x) {
      uint64_t key = ~0ull;
      if (i < cnt) {
        const int p = p0 + i;
        int lo = 0, hi = nr;  // rp[lo] <= p < rp[hi]
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (rp[mid] <= p) lo = mid;
          else hi = mid;
        }
        int c = col_idx[p];
        int64_t b = blk_idx ? static_cast<int64_t>(blk_idx[p]) : static_cast<int64_t>(p);
        if (static_cast<unsigned>(c) >= static_cast<unsigned>(nbc) || b < 0 || b >= nblocks_stored) {
          atomicCAS(err, 0u, KAIRO_DEVERR_BAD_INDEX);
          c = 0;
          b = 0;
        }
        key = (static_cast<uint64_t>(static_cast<uint32_t>(c)) << 40) | (static_cast<uint64_t>(lo) << 32) |
              static_cast<uint64_t>(static_cast<uint32_t>(b));
      }
      if (sorted) keys[i] = key;
      else order[p0 + i] = key;
    }
    __syncthreads();
    if (sorted && cnt > 1) {
      for (int k = 2; k <= npow; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
          for (int i = threadIdx.x; i < npow; i += blockDim.x) {
            const int ixj = i ^ j;
            if (ixj > i) {
              const uint64_t x = keys[i], y = keys[ixj];
              if ((x > y) == ((i & k) == 0)) {
                keys[i] = y;
                keys[ixj] = x;
              }
            }
          }
          __syncthreads();
        }
      }
    }
    if (sorted)
      for (int i = threadIdx.x; i < cnt; i += blockDim.x) order[p0 + i] = keys[i];
    __syncthreads();
  }
}

// ------------------------------------------------------------ SpMM kernel
struct BandItem {
  int chunk;
  int r0;      // first block-row
  int nr;      // block-rows in the group (R, or fewer at the end)
  int p0, p1;  // BSR positions of the group's blocks
  bool reverse;
};

__device__ __forceinline__ BandItem band_item(const BandArgs& a, int64_t t, int64_t wave) {
  BandItem it;
  it.chunk = static_cast<int>(t / a.row_groups);
  const int q = static_cast<int>(t - static_cast<int64_t>(it.chunk) * a.row_groups);
  it.r0 = q * a.rows;
  it.nr = min(a.rows, a.nbr - it.r0);
  // Clamped like the column-order pass, which reports malformed offsets.
  it.p0 = min(max(__ldg(a.row_ptr + it.r0), 0), a.nnzb);
  it.p1 = min(max(__ldg(a.row_ptr + it.r0 + it.nr), it.p0), a.nnzb);
  it.reverse = a.serpentine && (wave & 1);
  return it;
}

// Item of index t without its block range (no memory access).
__device__ __forceinline__ BandItem band_item_shape(const BandArgs& a, int64_t t, int64_t wave) {
  BandItem it;
  it.chunk = static_cast<int>(t / a.row_groups);
  const int q = static_cast<int>(t - static_cast<int64_t>(it.chunk) * a.row_groups);
  it.r0 = q * a.rows;
  it.nr = min(a.rows, a.nbr - it.r0);
  it.p0 = it.p1 = 0;
  it.reverse = a.serpentine && (wave & 1);
  return it;
}

// Key of stream position s of an item (its s-th block in visiting order), or
// all ones past the item's end.
__device__ __forceinline__ uint64_t band_key(const BandArgs& a, const BandItem& it, int s) {
  if (s >= it.p1 - it.p0) return ~0ull;
  const int64_t idx = it.reverse ? static_cast<int64_t>(it.p1) - 1 - s : static_cast<int64_t>(it.p0) + s;
  return __ldg(reinterpret_cast<const unsigned long long*>(a.order) + idx);
}

template <int BM, int BK, int NT, bool LINEAR, int IN_FMT, typename TOut>
__global__ void __launch_bounds__(kThreads, 1)
    bsr_spmm_band_kernel(const __grid_constant__ CUtensorMap tmap_a,
                         const __grid_constant__ CUtensorMap tmap_b, const BandArgs args) {
  constexpr int PANEL_BYTES = NT * 128 * BK * 2;
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int A_BYTES_PAD = (A_BYTES + 1023) / 1024 * 1024;
  constexpr int SLOT_BYTES = PANEL_BYTES + A_BYTES_PAD;
  constexpr uint32_t TX_BYTES = PANEL_BYTES + A_BYTES;
  constexpr int ROW_COLS = NT * BM;  // TMEM columns of one block-row's accumulator
  constexpr uint32_t IDESC = ptx::make_idesc_f16(IN_FMT, LINEAR ? 0u : 1u, 0u, 128u, BM);
  constexpr uint32_t SW_ROW = ptx::swizzle_code_for_row_bytes(BK * 2);
  static_assert(BK % 16 == 0 && BM % 16 == 0 && BM <= 256, "block shape");
  const uint32_t TMEM_COLS = args.tmem_cols;
  const uint32_t ACC_COLS = static_cast<uint32_t>(args.rows * ROW_COLS);
  const int NSLOT = args.acc_slots;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = args.stages;
  const int GB = args.group;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * GB * SLOT_BYTES);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint8_t* meta = reinterpret_cast<uint8_t*>(mma_done + 1);  // [S*GB]: row slot of each block slot
  int* misc = reinterpret_cast<int*>(meta + ((S * GB + 15) & ~15));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 0);
  volatile int* abort_flag = misc + 1;
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
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int64_t G = gridDim.x;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Same grouped, lane-parallel issue as the row-split kernel; each lane
    // also records its block's row slot in the stage metadata before the
    // group's full barrier is arrived on.  Memory reads of the producer are
    // software-pipelined so that it never waits on them: the keys of the
    // current item are held one 32-block window ahead of use (k0, k1), the
    // first two windows of the next item are loaded when the current one
    // starts (nk0, nk1), and the block range of the item after that is
    // loaded one item ahead (raw0, raw1).
    const uint64_t pol_a = ptx::policy_evict_first();
    const uint64_t pol_b = ptx::policy_evict_last();
    const uint32_t leader = lane == 0 ? 1u : 0u;
    int gpos = 0, gidx = 0;
    uint32_t gph = 0;
    bool alive = true;
    int64_t t = blockIdx.x, wave = 0;
    BandItem cur = band_item(args, t, wave);
    BandItem nxt = cur;
    int base = 0;
    uint64_t k0 = 0, k1 = 0, nk0 = 0, nk1 = 0;
    int raw0 = 0, raw1 = 0;
    bool has_nxt = false, has_after = false;
    if (t < args.nitems) {
      k0 = band_key(args, cur, lane);
      k1 = band_key(args, cur, 32 + lane);
      if (t + G < args.nitems) {
        has_nxt = true;
        nxt = band_item(args, t + G, wave + 1);
        nk0 = band_key(args, nxt, lane);
        nk1 = band_key(args, nxt, 32 + lane);
      }
      if (t + 2 * G < args.nitems) {
        has_after = true;
        const BandItem sh = band_item_shape(args, t + 2 * G, wave + 2);
        raw0 = __ldg(args.row_ptr + sh.r0);
        raw1 = __ldg(args.row_ptr + sh.r0 + sh.nr);
      }
    }
    while (t < args.nitems && alive) {
      const int n0 = cur.chunk * NT * 128;
      const int total = cur.p1 - cur.p0;
      for (int pb = 0; pb < total && alive; pb += 32) {
        const int cnt = min(32, total - pb);
        // Batches start at multiples of 32: once past window k0, shift so
        // that the batch is window k0 (loaded a batch ago) and load the next.
        if (pb >= base + 32) {
          k0 = k1;
          base += 32;
          k1 = band_key(args, cur, base + 32 + lane);
        }
        const uint64_t key = k0;
        int mc = static_cast<int>(key >> 40);
        int ms = static_cast<int>((key >> 32) & 0xffu);
        int mb = static_cast<int>(static_cast<uint32_t>(key));
        if (lane < cnt) {
          if (mc >= args.nbc || ms >= cur.nr || mb < 0 || static_cast<int64_t>(mb) >= args.nblocks_stored) {
            atomicCAS(args.err, 0u, KAIRO_DEVERR_BAD_INDEX);
            mc = 0;
            mb = 0;
            ms = 0;
          }
        } else {
          mc = 0;
          mb = 0;
          ms = 0;
        }
        int j0 = 0;
        while (j0 < cnt) {
          const int take = min(GB - gpos, cnt - j0);
          if (gpos == 0) {
            int ok = ptx::wait_parity(&empty[gidx], gph ^ 1u, abort_flag, args.err, kTagEmpty, args.wait_cycles);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
              alive = false;
              break;
            }
            if (lane == 0) issued[gidx] = static_cast<int>(gph) + 1;
          }
          const uint32_t mine = (lane >= j0 && lane < j0 + take) ? 1u : 0u;
          const int sidx = gidx * GB + gpos + (lane - j0);
          uint8_t* st = smem + sidx * SLOT_BYTES;
          if (mine) meta[sidx] = static_cast<uint8_t>(ms);
          ptx::mbar_expect_tx_if(mine, &full[gidx], TX_BYTES);
          ptx::tma_load_2d_if(mine, st + PANEL_BYTES, &tmap_a, 0, mb * BM, &full[gidx], pol_a);
          if (LINEAR) {
            ptx::tma_load_2d_if(mine, st, &tmap_b, mc * BK, n0, &full[gidx], pol_b);
          } else if (args.b_box3d) {
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
            ptx::mbar_arrive_if(leader, &full[gidx]);
            gpos = 0;
            if (++gidx == S) {
              gidx = 0;
              gph ^= 1u;
            }
          }
        }
      }
      if (!alive || !has_nxt) break;
      // Advance: the next item becomes current; the one after it gets its
      // range from the values loaded an item ago and its first keys loaded
      // now; the range of the item after that is loaded for later.
      t += G;
      ++wave;
      cur = nxt;
      base = 0;
      k0 = nk0;
      k1 = nk1;
      has_nxt = has_after;
      if (has_nxt) {
        nxt = band_item_shape(args, t + G, wave + 1);
        nxt.p0 = min(max(raw0, 0), args.nnzb);
        nxt.p1 = min(max(raw1, nxt.p0), args.nnzb);
        nk0 = band_key(args, nxt, lane);
        nk1 = band_key(args, nxt, 32 + lane);
      }
      has_after = t + 2 * G < args.nitems;
      if (has_after) {
        const BandItem sh = band_item_shape(args, t + 2 * G, wave + 2);
        raw0 = __ldg(args.row_ptr + sh.r0);
        raw1 = __ldg(args.row_ptr + sh.r0 + sh.nr);
      }
    }
    if (gpos != 0) ptx::mbar_arrive_if(leader, &full[gidx]);
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t leader = lane == 0 ? 1u : 0u;
    int mpos = 0, midx = 0;
    uint32_t mph = 0;
    const uint32_t sbase = ptx::smem_u32(smem);
    const uint64_t adesc0 = LINEAR ? ptx::make_smem_desc(sbase, 16, 8 * BK * 2, SW_ROW)
                                   : ptx::make_smem_desc(sbase, BK * 128, 1024, 2u);
    const uint64_t bdesc0 = ptx::make_smem_desc(sbase + PANEL_BYTES, 16, 8 * BK * 2, SW_ROW);
    const uint32_t a_lo0 = static_cast<uint32_t>(adesc0), a_hi = static_cast<uint32_t>(adesc0 >> 32);
    const uint32_t b_lo0 = static_cast<uint32_t>(bdesc0), b_hi = static_cast<uint32_t>(bdesc0 >> 32);
    constexpr uint32_t SLOT16 = SLOT_BYTES >> 4;
    uint32_t slot16 = 0;
    bool alive = true;
    int64_t nonempty = 0;
    int64_t wave = 0;
    for (int64_t t = blockIdx.x; t < args.nitems && alive; t += G, ++wave) {
      const BandItem it = band_item(args, t, wave);
      const int total = it.p1 - it.p0;
      if (total == 0) continue;
      const int buf = static_cast<int>(nonempty % NSLOT);
      const uint32_t ph = static_cast<uint32_t>((nonempty / NSLOT) & 1);
      ++nonempty;
      int ok = ptx::wait_parity(&tempty[buf], ph ^ 1u, abort_flag, args.err, kTagTmemEmpty, args.wait_cycles);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      ptx::tc_fence_after();
      const uint32_t d_base = tmem_base + static_cast<uint32_t>(buf) * ACC_COLS;
      uint32_t started = 0;  // bit s: row slot s already holds a partial sum
      int i = 0;
      while (i < total) {
        if (mpos == 0) {
          ok = ptx::wait_parity(&full[midx], mph, abort_flag, args.err, kTagFull, args.wait_cycles);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) {
            alive = false;
            break;
          }
          slot16 = static_cast<uint32_t>(midx * GB) * SLOT16;
        }
        const int seg = min(total - i, GB - mpos);
        const uint8_t* mrow = meta + midx * GB + mpos;
        for (int j = 0; j < seg; ++j) {
          const uint32_t s = mrow[j];
          const uint32_t acc0 = (started >> s) & 1u;
          started |= 1u << s;
          const uint32_t d = d_base + s * ROW_COLS;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
            for (int t2 = 0; t2 < NT; ++t2) {
              const uint32_t a_off = LINEAR ? (t2 * 128 * BK * 2 + kk * 32) : (t2 * 2 * BK * 128 + kk * 2048);
              ptx::mma_f16_ss_if(leader, d + t2 * BM, a_lo0 + slot16 + (a_off >> 4), a_hi,
                                 b_lo0 + slot16 + ((kk * 32) >> 4), b_hi, IDESC, (acc0 | (kk > 0)) ? 1u : 0u);
            }
          }
          slot16 += SLOT16;
        }
        i += seg;
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
      if (!alive) break;
      ptx::mma_commit_if(leader, &tfull[buf]);
    }
    if (mpos != 0) ptx::mma_commit_if(leader, &empty[midx]);
    ptx::mma_commit_if(leader, mma_done);
    int dummy = 0;
    ptx::wait_parity(mma_done, 0, reinterpret_cast<volatile int*>(&dummy), args.err, kTagDrain, args.wait_cycles);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int e = q * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    int64_t nonempty = 0;
    int64_t wave = 0;
    for (int64_t t = blockIdx.x; t < args.nitems; t += G, ++wave) {
      const BandItem it = band_item(args, t, wave);
      const int n0 = it.chunk * NT * 128;
      if (it.p1 == it.p0) {
        float z[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) z[jj] = 0.f;
        for (int s = 0; s < it.nr; ++s)
#pragma unroll
          for (int t2 = 0; t2 < NT; ++t2)
#pragma unroll
            for (int j0 = 0; j0 < BM; j0 += 16) store16<LINEAR, TOut>(args, it.r0 + s, BM, j0, n0 + t2 * 128 + e, z);
        continue;
      }
      const int buf = static_cast<int>(nonempty % NSLOT);
      const uint32_t ph = static_cast<uint32_t>((nonempty / NSLOT) & 1);
      ++nonempty;
      int ok = ptx::wait_parity(&tfull[buf], ph, abort_flag, args.err, kTagTmemFull, args.wait_cycles, 200);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (epi_any(!ok)) break;
      ptx::tc_fence_after();
      const uint32_t cols0 = static_cast<uint32_t>(buf) * ACC_COLS;
      int rp_prev = it.p0;
      for (int s = 0; s < it.nr; ++s) {
        const int rp_next = __ldg(args.row_ptr + it.r0 + s + 1);
        const bool has = rp_next > rp_prev;
        rp_prev = rp_next;
#pragma unroll
        for (int t2 = 0; t2 < NT; ++t2) {
#pragma unroll
          for (int j0 = 0; j0 < BM; j0 += 16) {
            float v[16];
            if (has) {
              ptx::tmem_ld16(tmem_base + lane_addr + cols0 + static_cast<uint32_t>(s * ROW_COLS + t2 * BM + j0), v);
              ptx::tmem_wait_ld();
            } else {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) v[jj] = 0.f;
            }
            store16<LINEAR, TOut>(args, it.r0 + s, BM, j0, n0 + t2 * 128 + e, v);
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&tempty[buf]);
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0 && *abort_flag) {
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

using BandFn = void (*)(CUtensorMap, CUtensorMap, BandArgs);

template <int BM, int NT, bool LINEAR, int IN_FMT, typename TOut>
BandFn band4() {
  return reinterpret_cast<BandFn>(&bsr_spmm_band_kernel<BM, BM, NT, LINEAR, IN_FMT, TOut>);
}

template <bool LINEAR, int IN_FMT, typename TOut>
BandFn band3(int bm, int nt) {
#define KAIRO_BAND_CASE(B, T) \
  if (bm == B && nt == T) return band4<B, T, LINEAR, IN_FMT, TOut>();
  KAIRO_BAND_CASE(16, 1)
  KAIRO_BAND_CASE(16, 2)
  KAIRO_BAND_CASE(32, 1)
  KAIRO_BAND_CASE(32, 2)
  KAIRO_BAND_CASE(64, 1)
  KAIRO_BAND_CASE(64, 2)
#undef KAIRO_BAND_CASE
  return nullptr;
}

BandFn pick_band(int bm, int nt, bool linear, kairo_dtype in, kairo_dtype out) {
  if (!linear) {
    if (out != KAIRO_DTYPE_F32) return nullptr;
    return in == KAIRO_DTYPE_F16 ? band3<false, 0, float>(bm, nt) : band3<false, 1, float>(bm, nt);
  }
  if (in == KAIRO_DTYPE_F16) {
    if (out == KAIRO_DTYPE_F32) return band3<true, 0, float>(bm, nt);
    if (out == KAIRO_DTYPE_F16) return band3<true, 0, __half>(bm, nt);
  } else {
    if (out == KAIRO_DTYPE_F32) return band3<true, 1, float>(bm, nt);
    if (out == KAIRO_DTYPE_BF16) return band3<true, 1, __nv_bfloat16>(bm, nt);
  }
  return nullptr;
}

// Shared memory besides the stage slots: barriers, per-slot metadata, flags.
size_t band_aux_bytes(int stages, int group) {
  return 8 * (2 * stages + 5) + ((stages * group + 15) & ~15) + 16 + 4 * stages;
}

}  // namespace

bool band_supported(const kairo_bsr* a, std::string* why) {
  auto no = [&](const char* w) {
    if (why) *why = w;
    return false;
  };
  if (ceil_div64(a->cols, a->bk) >= (int64_t(1) << 24)) return no("band schedule needs fewer than 2^24 block-columns");
  if (a->nnzb > INT32_MAX) return no("band schedule needs fewer than 2^31 blocks");
  return true;
}

bool band_preferred(const kairo_bsr* a, int64_t n, int device) {
  // The row-split schedule cuts a block-row wherever a CTA's share of the
  // merge path ends and sums the pieces through partial tiles.  When a chunk
  // has fewer block-rows than twice the CTAs, most rows are cut (the linear
  // layer: 128 rows, 148 CTAs, 1.54 ms) and the band schedule, which keeps
  // rows whole, is faster (1.40 ms).  It needs enough items to balance the
  // CTAs and rows of similar length, which only the caller's max_row_blocks
  // can vouch for.
  // With many rows it still wins on a dense block grid, where the CTAs'
  // common column sweep keeps the gathered panels in L2 (the transposed
  // linear-layer weight: 512 rows at 20 % density, 1.46 ms against 1.61 ms);
  // on a sparse grid the row split balances better (262144^2 at 0.5 %:
  // 2.38 ms against 2.72 ms).
  if (a->max_row_blocks <= 0 || a->nbr <= 0 || a->nnzb <= 0) return false;
  const int sms = device_sm_count(device);
  const int64_t nbc = ceil_div64(a->cols, a->bk);
  const double density = nbc > 0 ? static_cast<double>(a->nnzb) / (static_cast<double>(a->nbr) * nbc) : 0.0;
  if (a->nbr >= 2 * sms && density < 0.1) return false;
  const double mean = static_cast<double>(a->nnzb) / a->nbr;
  if (a->max_row_blocks > 2.0 * mean + 8.0) return false;
  const int nt = n > 128 ? 2 : 1;
  const int R = std::max(1, std::min(kMaxBandRows, 256 / (nt * a->bm)));
  const int64_t nitems = ceil_div64(n, 128 * nt) * ceil_div64(a->nbr, R);
  return nitems >= 4 * static_cast<int64_t>(sms);
}

kairo_status band_plan(const kairo_bsr* a, int32_t layout, int64_t n, const kairo_spmm_config* cfg, int device,
                       BandPlan* plan) {
  (void)layout;
  BandPlan p{};
  p.bm = a->bm;
  p.bk = a->bk;
  int nt = n > 128 ? 2 : 1;
  if (cfg && cfg->n_tile) {
    if (cfg->n_tile != 128 && cfg->n_tile != 256) return fail(KAIRO_STATUS_INVALID_VALUE, "n_tile must be 128 or 256");
    nt = cfg->n_tile / 128;
  }
  p.nt = nt;
  p.nchunks = static_cast<int>(ceil_div64(n, 128 * nt));
  const int row_cols = nt * p.bm;
  // Resident CTAs per SM (kairo_spmm_config.ctas_per_sm, default 2): they
  // split the SM's 512 TMEM columns and its shared memory, so one CTA's
  // pipeline handoffs overlap the other's MMAs.  Measured on B200 with the
  // 8192 x 32768 linear layer (64x64 blocks, 20 %, batch 8192): the
  // forward 1.41 -> 1.22 ms (2 CTAs of one block-row per item, against one
  // CTA of two), dX of its backward 1.52 -> 1.29 ms.
  if (cfg && (cfg->ctas_per_sm < 0 || cfg->ctas_per_sm > 4))
    return fail(KAIRO_STATUS_INVALID_VALUE, "ctas_per_sm must be between 0 and 4");
  int per_sm = (cfg && cfg->ctas_per_sm > 0) ? cfg->ctas_per_sm : 2;
  // Clamped to what the TMEM holds: at least one block-row per item, or the
  // caller's band_rows.
  const int min_rows = (cfg && cfg->band_rows > 0) ? std::min(cfg->band_rows, kMaxBandRows) : 1;
  while (per_sm > 1 && 512 / per_sm < min_rows * row_cols) --per_sm;
  const int tmem_budget = 512 / per_sm;
  // Default: the most rows that still leave room for two accumulator sets,
  // so the epilogue of one item overlaps the MMAs of the next.
  int R = (cfg && cfg->band_rows > 0) ? cfg->band_rows : std::max(1, (tmem_budget / 2) / row_cols);
  if (R > kMaxBandRows) R = kMaxBandRows;
  if (R * row_cols > tmem_budget)
    return fail(KAIRO_STATUS_INVALID_VALUE, "band_rows * n_tile/128 * block size exceeds the CTA's TMEM");
  if (R > a->nbr && a->nbr > 0) R = a->nbr;
  if (R < 1) R = 1;
  p.rows = R;
  p.acc_slots = (2 * R * row_cols <= tmem_budget) ? 2 : 1;
  p.tmem_cols = 32;
  while (p.tmem_cols < static_cast<uint32_t>(p.acc_slots * R * row_cols)) p.tmem_cols <<= 1;
  while (per_sm > 1 && static_cast<uint32_t>(per_sm) * p.tmem_cols > 512) --per_sm;
  p.row_groups = static_cast<int>(ceil_div64(a->nbr, R));
  p.nitems = static_cast<int64_t>(p.nchunks) * p.row_groups;
  const int sms = device_sm_count(device);
  int64_t grid = (cfg && cfg->num_ctas > 0) ? cfg->num_ctas : static_cast<int64_t>(sms) * per_sm;
  if (grid > p.nitems) grid = p.nitems;
  if (grid < 1) grid = 1;
  p.grid = static_cast<int>(grid);
  p.serpentine = 1;
  if (cfg && cfg->wait_kcycles < 0) return fail(KAIRO_STATUS_INVALID_VALUE, "wait_kcycles must be >= 0");
  p.wait_cycles = wait_bound_cycles(cfg);
  const int sb = stage_bytes(p.bm, p.bk, nt);
  int group = (cfg && cfg->group_blocks > 0) ? cfg->group_blocks : 0;
  if (group > 32) return fail(KAIRO_STATUS_INVALID_VALUE, "group_blocks must be at most 32");
  const int budget = std::min(kMaxSmem, (kSmemPerSm - per_sm * kSmemReservedPerCta) / per_sm) - 1024 /*alignment*/ -
                     static_cast<int>(band_aux_bytes(32, 32));
  if (group == 0) group = default_group_blocks(budget / sb, b_slice_bytes(a, nt) > 0.5 * device_l2_bytes(device));
  int max_stages = budget / (group * sb);
  if (max_stages > 32) max_stages = 32;
  const int stages = (cfg && cfg->stages > 0) ? std::min(cfg->stages, max_stages) : max_stages;
  if (stages < 2) return fail(KAIRO_STATUS_NOT_SUPPORTED, "shared memory too small for two pipeline stages");
  p.group = group;
  p.stages = stages;
  p.smem_bytes = static_cast<size_t>(stages) * group * sb + 1024 + band_aux_bytes(stages, group);
  p.order_offset = kWorkspaceHeaderBytes + kCounterRegionBytes;
  p.order_bytes = static_cast<size_t>(a->nnzb) * sizeof(uint64_t);
  p.workspace_bytes = p.order_offset + p.order_bytes;
  *plan = p;
  return KAIRO_STATUS_SUCCESS;
}

kairo_status band_launch(const kairo_bsr* a, const void* b, int64_t ldb, int32_t layout, int64_t n, void* c,
                         int64_t ldc, kairo_dtype c_dtype, const BandPlan& plan, void* workspace,
                         cudaStream_t stream) {
  const bool linear = layout == KAIRO_LAYOUT_LINEAR;
  BandFn fn = pick_band(plan.bm, plan.nt, linear, a->dtype, c_dtype);
  if (!fn) return fail(KAIRO_STATUS_NOT_SUPPORTED, "no band-schedule kernel for this block size / dtype combination");
  CUtensorMap map_a, map_b;
  int b_box3d = 0;
  kairo_status st = make_operand_maps(a, b, ldb, linear, n, plan.nt, &map_a, &map_b, &b_box3d);
  if (st) return st;

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  unsigned* err = reinterpret_cast<unsigned*>(ws);
  uint64_t* order = reinterpret_cast<uint64_t*>(ws + plan.order_offset);
  const int nbc = static_cast<int>(ceil_div64(a->cols, a->bk));
  const int order_grid = std::max(1, std::min(plan.row_groups, device_sm_count(current_device()) * 8));
  band_order_kernel<<<order_grid, kOrderThreads, 0, stream>>>(a->row_ptr, a->col_idx, a->blk_idx, a->nbr, nbc,
                                                              static_cast<int32_t>(a->nnzb), a->nblocks_stored,
                                                              plan.rows, plan.row_groups, order, err);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the band column-order kernel");

  BandArgs args{};
  args.row_ptr = a->row_ptr;
  args.order = order;
  args.c = c;
  args.ldc = ldc;
  args.nitems = plan.nitems;
  args.nblocks_stored = a->nblocks_stored;
  args.err = err;
  args.m = static_cast<int32_t>(a->rows);
  args.n = static_cast<int32_t>(n);
  args.nbr = a->nbr;
  args.nbc = nbc;
  args.nnzb = static_cast<int32_t>(a->nnzb);
  args.rows = plan.rows;
  args.row_groups = plan.row_groups;
  args.stages = plan.stages;
  args.group = plan.group;
  args.acc_slots = plan.acc_slots;
  args.serpentine = plan.serpentine;
  args.tmem_cols = plan.tmem_cols;
  args.b_box3d = b_box3d;
  args.wait_cycles = plan.wait_cycles;
  const size_t osz = c_dtype == KAIRO_DTYPE_F32 ? 4 : 2;
  args.vec_store = linear && ((reinterpret_cast<uintptr_t>(c) & 15u) == 0) && ((ldc * osz) % 16 == 0) ? 1 : 0;

  e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn), cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(plan.smem_bytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  fn<<<plan.grid, kThreads, plan.smem_bytes, stream>>>(map_a, map_b, args);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "launch of the band-schedule SpMM kernel");
  return KAIRO_STATUS_SUCCESS;
}

}  // namespace kairo
