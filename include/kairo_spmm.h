/*
 * kairo_spmm.h -- C ABI of the B200 (sm_100a) block-sparse SpMM library.
 *
 * This is the drop-in boundary for Kairo's block-sparse matmul path.  It
 * replaces the pybind11 module of the reference (csrc/bindings.cpp:84-103,
 * 119-124) and its host wrapper acc_spmm_forward_cuda
 * (csrc/acc_spmm_kernel.cu:158-207) with plain C entry points: raw device
 * pointers, integer sizes, a caller-owned workspace and the caller's CUDA
 * stream.  No C++ exception and no framework type crosses this boundary;
 * every entry point returns a kairo_status and keeps a per-thread message
 * that kairo_last_error_message() returns.
 *
 * Conventions
 *  - All matrices are row-major.  Block (tile) storage is (nblocks, bm, bk)
 *    row-major, the layout of the reference's A_tiles (kairo/ops/spmm.py:42-53).
 *  - "BSR" means: row_ptr (nbr+1, int32, exclusive prefix of blocks per
 *    block-row), col_idx (nnzb, int32, block-column of each block in row
 *    order), and optionally blk_idx (nnzb, int32, which stored block holds
 *    block p; NULL means block p is stored at position p).  Row order within a
 *    block-row is the stable order of the input COO list, as produced by the
 *    reference's _sort_coo_by_row + _coo_to_row_offsets
 *    (kairo/ops/sparse_embedding.py:49-56, 23-46).
 *  - Launches are asynchronous on `stream` (a cudaStream_t; NULL = legacy
 *    default stream).  Device-side failures (an index out of range, a
 *    pipeline wait that timed out) are recorded in the workspace error word
 *    and read back with kairo_workspace_error().
 *  - Workspaces are caller-allocated device memory.  They must be zero-filled
 *    before their first use; the library leaves every counter it uses at zero
 *    when a launch completes normally, so one workspace can be reused by
 *    consecutive launches on one stream.  Launches that overlap in time (two
 *    streams) must use different workspaces.
 */
#ifndef KAIRO_SPMM_H_
#define KAIRO_SPMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KAIRO_ABI_VERSION 2

#if defined(__GNUC__)
#define KAIRO_API __attribute__((visibility("default")))
#else
#define KAIRO_API
#endif

typedef enum kairo_status {
  KAIRO_STATUS_SUCCESS = 0,
  KAIRO_STATUS_INVALID_VALUE = 1,     /* bad argument (the reference raises via TORCH_CHECK) */
  KAIRO_STATUS_NOT_SUPPORTED = 2,     /* valid input outside what the kernels implement */
  KAIRO_STATUS_CUDA_ERROR = 3,        /* a CUDA runtime/driver call failed */
  KAIRO_STATUS_WORKSPACE_TOO_SMALL = 4,
  KAIRO_STATUS_DEVICE_ERROR = 5       /* the device recorded an error (see kairo_workspace_error) */
} kairo_status;

typedef enum kairo_dtype {
  KAIRO_DTYPE_F32 = 0,
  KAIRO_DTYPE_F16 = 1,
  KAIRO_DTYPE_BF16 = 2
} kairo_dtype;

/* Kernel family chosen by kairo_spmm_config.kernel. */
typedef enum kairo_kernel {
  KAIRO_KERNEL_AUTO = 0,     /* tcgen05 for f16/bf16 when the shape allows it, else SIMT */
  KAIRO_KERNEL_SIMT = 1,     /* CUDA-core FMA kernel (fp32 path, any shape) */
  KAIRO_KERNEL_TCGEN05 = 2,  /* TMA + tcgen05/TMEM persistent kernel (f16/bf16) */
  KAIRO_KERNEL_SPLIT_BF16 = 3  /* opt-in, fp32 A and B: the tcgen05 kernel on a bf16 hi/lo split,
                                  A_hi B_hi + A_hi B_lo + A_lo B_hi (about 2^-15 relative error per
                                  product); square 16/32/64 blocks, STANDARD layout.  Needs extra
                                  workspace for the derived operands.  No reference counterpart. */
} kairo_kernel;

/* Device error codes written to the workspace error word (low 8 bits). */
#define KAIRO_DEVERR_NONE 0u
#define KAIRO_DEVERR_WAIT_TIMEOUT 1u      /* a pipeline wait ran out; the kernel stopped */
#define KAIRO_DEVERR_BAD_INDEX 2u         /* a tile row/column id outside the block grid */
#define KAIRO_DEVERR_ROW_TOO_LONG 3u      /* unsorted COO with a block-row longer than the sort limit */
/* Site tags of KAIRO_DEVERR_WAIT_TIMEOUT (bits 8..15): which wait ran out. */
#define KAIRO_WAIT_SITE_EMPTY 1u          /* producer waiting for a free shared-memory stage */
#define KAIRO_WAIT_SITE_FULL 2u           /* MMA issuer waiting for a loaded stage */
#define KAIRO_WAIT_SITE_TMEM_EMPTY 3u     /* MMA issuer waiting for a drained TMEM accumulator */
#define KAIRO_WAIT_SITE_TMEM_FULL 4u      /* epilogue waiting for a finished accumulator */
#define KAIRO_WAIT_SITE_DRAIN 5u          /* a CTA draining its copies or MMAs before it exits */

/* Block-sparse matrix in BSR form (all pointers are device pointers). */
typedef struct kairo_bsr {
  int64_t rows;              /* M: logical rows of A */
  int64_t cols;              /* K: logical columns of A */
  int32_t bm;                /* block rows (tile_m) */
  int32_t bk;                /* block columns (tile_k) */
  int32_t nbr;               /* number of block-rows = ceil(M / bm) */
  int32_t reserved0;
  int64_t nnzb;              /* number of nonzero blocks */
  int64_t nblocks_stored;    /* blocks in `blocks` storage (>= nnzb when blk_idx != NULL) */
  const int32_t* row_ptr;    /* nbr + 1 */
  const int32_t* col_idx;    /* nnzb */
  const int32_t* blk_idx;    /* nnzb, or NULL for identity */
  const void* blocks;        /* (nblocks_stored, bm, bk) row-major, dtype below */
  kairo_dtype dtype;
  int32_t max_row_blocks;    /* longest block-row in blocks, if known (0 = unknown); a scheduling hint */
} kairo_bsr;

/* Tuning knobs of one launch; zero-initialised means "library default". */
typedef struct kairo_spmm_config {
  int32_t kernel;            /* kairo_kernel */
  int32_t n_tile;            /* C columns per work item on tcgen05: 128 or 256 (0 = auto) */
  int32_t stages;            /* pipeline stages in shared memory (0 = auto) */
  int32_t row_cost;          /* scheduler weight of one block-row in units of one block (0 = auto) */
  int32_t num_ctas;          /* persistent grid size (0 = one CTA per SM) */
  int32_t group_blocks;      /* nonzero blocks per pipeline stage, 1..32 (0 = auto) */
  int32_t schedule;          /* kairo_schedule (tcgen05 kernel only) */
  int32_t band_rows;         /* block-rows per item of the band schedule (0 = auto) */
  int32_t wait_kcycles;      /* bound of every pipeline wait of the tcgen05 kernels, in thousands of SM
                                cycles (0 = the default, 8e9 cycles, about 4 s); a debugging knob */
  int32_t debug_hold_stage;  /* test hook, 0 in normal use.  1: the row-split kernel's producer holds
                                back the arrival of its first pipeline stage until the kernel aborts
                                (bounded by 4 wait bounds), so that a consumer's bounded wait runs out:
                                the launch records KAIRO_DEVERR_WAIT_TIMEOUT with the wait's site tag,
                                drains its copies and MMAs, frees TMEM and returns.  Ignored by the other
                                kernels. */
  int32_t ctas_per_sm;       /* resident CTAs per SM of the tcgen05 kernels, 1..4 (0 = auto: 2, or 1 for
                                the row-split schedule with 64-row blocks): the SM's shared memory and
                                TMEM are split between them, so that one CTA's pipeline handoffs
                                overlap another's MMAs; clamped to what the SM can hold */
  int32_t reserved[1];
} kairo_spmm_config;

/* Work schedules of the tcgen05 kernel.
 * ROWS:  block-rows split over CTAs by a merge path over (rows, blocks); long
 *        rows are cut and their pieces summed in a fixed order.  Robust to
 *        skewed masks.
 * BANDS: each CTA holds `band_rows` block-rows in TMEM and visits their
 *        blocks in column order, all CTAs sweeping B together so gathered B
 *        panels are shared through L2.  Rows are never cut.
 * AUTO picks BANDS when a chunk has fewer block-rows than twice the SM
 * count (the row-split schedule would cut most rows), there are at least
 * four band items per SM, and kairo_bsr.max_row_blocks shows rows of
 * similar length; otherwise ROWS. */
typedef enum kairo_schedule {
  KAIRO_SCHEDULE_AUTO = 0,
  KAIRO_SCHEDULE_ROWS = 1,
  KAIRO_SCHEDULE_BANDS = 2,
  KAIRO_SCHEDULE_GROUPS = 3  /* row groups (kairo_bsr_spmm_stacked); reported by describe, not a selector here */
} kairo_schedule;

/* Operand layouts of kairo_bsr_spmm. */
#define KAIRO_LAYOUT_STANDARD 0  /* B is (K x N), C is (M x N):  C = A * B            */
#define KAIRO_LAYOUT_LINEAR 1    /* X is (N x K), Y is (N x M):  Y = X * A^T (a linear layer) */

/* ------------------------------------------------------------------------
 * BSR SpMM.  STANDARD: C[M x N] = A_bsr[M x K] * B[K x N].
 *            LINEAR:   Y[N x M] = X[N x K] * A_bsr^T, i.e. C^T with B = X^T.
 * `b` has leading dimension ldb (elements), `c` has ldc.  B's dtype equals
 * A->dtype; c_dtype is F32 (fp32 accumulate, fp32 out) or, in LINEAR layout,
 * may equal A->dtype (fp32 accumulate, rounded once on store).
 * Every element of C (all M x N) is written, including all-zero block-rows.
 * Replaces the numerical part of acc_spmm_forward_cuda
 * (csrc/acc_spmm_kernel.cu:158-207) for BSR input.
 * ---------------------------------------------------------------------- */
KAIRO_API kairo_status kairo_bsr_spmm(const kairo_bsr* a, const void* b, int64_t ldb,
                            int32_t layout, int64_t n, void* c, int64_t ldc,
                            kairo_dtype c_dtype, const kairo_spmm_config* cfg,
                            void* workspace, size_t workspace_bytes, void* stream);

/* kairo_bsr_spmm without a workspace argument, for callers that cannot
 * allocate device memory (a framework that forbids plugins to cudaMalloc, a
 * path that must not stall the device, a stateless callback).  This entry
 * point has no counterpart in the reference.  Its scratch is a 32 MiB array
 * built into the library, one per device: every GPU that loads the library
 * holds it until the process exits.  Problems needing more scratch than that
 * return KAIRO_STATUS_NOT_SUPPORTED.  The first call on a device looks up the
 * array's device address (make it before any stream capture); the address is
 * cached per device and CUDA context, and looked up again under a new
 * context.  Each call clears the array's error word and counters on
 * `stream`.  Calls share the array, so calls whose launches overlap on the
 * GPU race: order them. */
KAIRO_API kairo_status kairo_bsr_spmm_noalloc(const kairo_bsr* a, const void* b, int64_t ldb,
                                              int32_t layout, int64_t n, void* c, int64_t ldc,
                                              kairo_dtype c_dtype, const kairo_spmm_config* cfg,
                                              void* stream);

/* The device error word of the last kairo_bsr_spmm_noalloc call on the
 * current device (KAIRO_DEVERR_* in the low 8 bits, a site tag above), read
 * like kairo_workspace_error: synchronises `stream`, optionally clears the
 * word.  Read it after a call and before the next one, which clears it.  No
 * counterpart in the reference.  Allocates nothing. */
KAIRO_API kairo_status kairo_noalloc_error(int32_t clear, uint32_t* code, void* stream);

/* What kairo_bsr_spmm would run for this problem (no device work).  Fills
 * `out` from the same decision as kairo_bsr_spmm_workspace_size, assuming
 * 16-byte aligned operands.  No counterpart in the reference; used by the
 * autotuner and benchmarks to report the kernel and its launch count. */
typedef struct kairo_spmm_plan {
  int32_t kernel;            /* kairo_kernel actually used (0 = nothing to compute) */
  int32_t schedule;          /* kairo_schedule used by the tcgen05 kernel (0 otherwise) */
  int32_t launches;          /* kernel launches per call */
  int32_t grid;              /* CTAs of the main kernel */
  int32_t n_tile;            /* C columns per work item */
  int32_t stages;            /* pipeline stages */
  int32_t group_blocks;      /* blocks per stage */
  int32_t rows;              /* band_rows (BANDS) or row_cost (ROWS) */
  uint64_t workspace_bytes;
} kairo_spmm_plan;
KAIRO_API kairo_status kairo_bsr_spmm_describe(const kairo_bsr* a, int32_t layout, int64_t n,
                                               const kairo_spmm_config* cfg, kairo_spmm_plan* out);

/* Bytes of zero-initialised workspace kairo_bsr_spmm needs for this problem. */
KAIRO_API kairo_status kairo_bsr_spmm_workspace_size(const kairo_bsr* a, int32_t layout, int64_t n,
                                           const kairo_spmm_config* cfg, size_t* bytes);

/* ------------------------------------------------------------------------
 * Row groups: the same SpMM for masks whose block-rows are long and share
 * columns (a skewed mask such as Zipf row counts, where a few rows hold most
 * blocks).  The block-rows, ordered by block count (longest first, ties by
 * index), are taken R at a time; a group's "stacked blocks" are its distinct
 * column-blocks, each with a mask of the group rows that have a block there.
 * The tcgen05 kernel then loads one B panel per stacked block and multiplies
 * each run of consecutive present rows with one MMA of N = run * bm.  Same
 * result as kairo_bsr_spmm (fp32 accumulate; the sums run in another order,
 * so the two agree to fp32 rounding, not bit for bit).  No counterpart in
 * the reference: the reference has one kernel for every mask
 * (csrc/acc_spmm_kernel.cu:158-207); this is an added schedule for the
 * operator that kairo/ops/spmm.py:58-105 defines.
 *
 * kairo_bsr_stack_build builds the groups on the device into `mem`
 * (kairo_bsr_stack_size bytes), fills `out` and synchronises `stream` once
 * (it reads the stacked-block count back).  R is 2, 4 or 8; nbr and the
 * number of block-columns must be at most 16384.  A block-row holding two
 * blocks in one column returns NOT_SUPPORTED; a column index out of range
 * returns INVALID_VALUE.  The structure depends only on row_ptr / col_idx /
 * blk_idx: it stays valid while those are unchanged (block values may
 * change).
 * kairo_bsr_spmm_stacked: STANDARD layout, f16/bf16 square blocks of 16 or
 * 32, fp32 C; R * bm * (n_tile / 128) must be at most 128 (n_tile 256 is
 * used when N > 128 and that product allows it).
 * ---------------------------------------------------------------------- */
typedef struct kairo_bsr_stack {
  int32_t rows_per_group;    /* R */
  int32_t ngroups;           /* ceil(nbr / R) */
  int64_t nsuper;            /* stacked blocks */
  const int32_t* group_ptr;  /* ngroups + 1: stacked blocks of each group */
  const int32_t* super_col;  /* nsuper: column-block of each stacked block, ascending within a group */
  const int32_t* super_mask; /* nsuper: bit r set when group row r has a block in that column */
  const int32_t* super_blk;  /* nsuper * R: stored-block index (blk_idx) of each present block */
  const int32_t* row_map;    /* ngroups * R: block-row of each group row, -1 past the last */
} kairo_bsr_stack;

KAIRO_API kairo_status kairo_bsr_stack_size(const kairo_bsr* a, int32_t rows_per_group, size_t* bytes);
KAIRO_API kairo_status kairo_bsr_stack_build(const kairo_bsr* a, int32_t rows_per_group, void* mem,
                                             size_t mem_bytes, kairo_bsr_stack* out, void* stream);
KAIRO_API kairo_status kairo_bsr_spmm_stacked_workspace_size(const kairo_bsr* a, const kairo_bsr_stack* s,
                                                             int64_t n, const kairo_spmm_config* cfg,
                                                             size_t* bytes);
KAIRO_API kairo_status kairo_bsr_spmm_stacked_describe(const kairo_bsr* a, const kairo_bsr_stack* s, int64_t n,
                                                       const kairo_spmm_config* cfg, kairo_spmm_plan* out);
KAIRO_API kairo_status kairo_bsr_spmm_stacked(const kairo_bsr* a, const kairo_bsr_stack* s, const void* b,
                                              int64_t ldb, int64_t n, void* c, int64_t ldc,
                                              const kairo_spmm_config* cfg, void* workspace,
                                              size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * COO tile list -> BSR, on the device, bit-identical to the reference's
 * convention: perm = argsort(tile_row_ids, stable) (sparse_embedding.py:55),
 * col_idx = tile_col_ids[perm], row_ptr = row offsets of the sorted rows
 * (sparse_embedding.py:23-46, here int32).  `perm` receives the stored-block
 * index of every BSR position (use it as kairo_bsr.blk_idx).  *is_identity
 * (host) tells whether the input was already row-sorted (perm[p] == p); when
 * it is, callers may pass blk_idx = NULL.  *max_row_blocks (host, may be
 * NULL) receives the longest block-row, for kairo_bsr.max_row_blocks.
 * Ids outside [0, nbr) x [0, nbc)
 * raise INVALID_VALUE.  Unsorted input is supported when no block-row holds
 * more than 16384 tiles (NOT_SUPPORTED otherwise).
 * This call synchronises `stream` once (it reads two flags back).
 * ---------------------------------------------------------------------- */
KAIRO_API kairo_status kairo_bsr_build(const int32_t* tile_row_ids, const int32_t* tile_col_ids,
                             int64_t num_tiles, int32_t nbr, int32_t nbc,
                             int32_t* row_ptr, int32_t* col_idx, int32_t* perm,
                             int32_t* is_identity, int32_t* max_row_blocks, void* workspace,
                             size_t workspace_bytes, void* stream);
KAIRO_API kairo_status kairo_bsr_build_workspace_size(int64_t num_tiles, int32_t nbr, size_t* bytes);

/* ------------------------------------------------------------------------
 * BSR transpose on the device, for the backward pass of the linear layer
 * (dX = dY * W is the LINEAR-layout product with W^T).  No counterpart in
 * the reference, which has no SpMM backward.
 *
 * W^T has cols/bk block-rows and the same blocks, each transposed (bk x bm).
 * Its order is the stable sort of W's positions by block-column, i.e.
 * (column, row) order, the BSR convention applied to W^T's COO list.
 *   row_ptr_t  (cols/bk + 1)   block-row offsets of W^T;
 *   col_idx_t  (nnzb)          block-columns of W^T (block-rows of W);
 *   perm_t     (nnzb)          W's BSR position of every W^T position;
 *   blocks_t   (nnzb, bk, bm)  transposed blocks in W^T order, W's dtype
 *                              (NULL: structure only).
 * Asynchronous on `stream` (no host synchronisation).  Invalid ids, or a
 * block-column of more than 16384 blocks, are reported in the workspace
 * error word (kairo_workspace_error), not by the return value.
 * kairo_bsr_transpose_values refreshes blocks_t alone from a cached perm_t
 * when only the values of W changed (a workspace of >= 256 bytes holds the
 * error word).
 * ---------------------------------------------------------------------- */
KAIRO_API kairo_status kairo_bsr_transpose(const kairo_bsr* a, int32_t* row_ptr_t, int32_t* col_idx_t,
                                           int32_t* perm_t, void* blocks_t, void* workspace,
                                           size_t workspace_bytes, void* stream);
KAIRO_API kairo_status kairo_bsr_transpose_workspace_size(const kairo_bsr* a, size_t* bytes);
KAIRO_API kairo_status kairo_bsr_transpose_values(const kairo_bsr* a, const int32_t* perm_t, void* blocks_t,
                                                  void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Weight gradient of the linear layer Y = X * W^T restricted to W's nonzero
 * blocks (block-sampled dense x dense product).  No counterpart in the
 * reference.  For every BSR position p = (block-row i, block-column j):
 *   dblocks[p] = dY[:, i*bm : (i+1)*bm]^T * X[:, j*bk : (j+1)*bk]   (bm x bk)
 * summed over the n batch rows; dY is (n x rows), X is (n x cols), both
 * row-major with leading dimensions lddy / ldx, W's dtype.  `a` is W (its
 * col_idx is read; values are not); row_ptr_t / col_idx_t / perm_t are W's
 * transposed structure from kairo_bsr_transpose.  dblocks is (nnzb, bm, bk)
 * in W's BSR order, fp32 or W's dtype.  64 x 64 f16/bf16 blocks run on the
 * tensor cores, other shapes and fp32 on CUDA cores.  Asynchronous; device
 * errors go to the workspace error word.
 * ---------------------------------------------------------------------- */
KAIRO_API kairo_status kairo_bsr_sddmm(const kairo_bsr* a, const int32_t* row_ptr_t, const int32_t* col_idx_t,
                                       const int32_t* perm_t, const void* dy, int64_t lddy, const void* x,
                                       int64_t ldx, int64_t n, void* dblocks, kairo_dtype out_dtype,
                                       void* workspace, size_t workspace_bytes, void* stream);
KAIRO_API kairo_status kairo_bsr_sddmm_workspace_size(const kairo_bsr* a, size_t* bytes);

/* ------------------------------------------------------------------------
 * Block-granular pruning (no counterpart in the reference, which prunes
 * element by element: kairo/training/sparse_rec/topology.py:50-118).
 *   kairo_block_norms      L2 norm of every bm x bk block of a dense matrix
 *                          (m x k, lda), fp32, row-major over the block grid.
 *   kairo_bsr_block_norms  L2 norm of every BSR block, in BSR order.
 *   kairo_topk_indices     indices of the `count` largest scores, ascending;
 *                          ties at the threshold go to the lower index, NaN
 *                          ranks lowest ("topk, then sort" of the reference's
 *                          prune_mask for distinct scores).
 * All asynchronous on `stream`.
 * ---------------------------------------------------------------------- */
KAIRO_API kairo_status kairo_block_norms(const void* a, int64_t m, int64_t k, int64_t lda, int32_t bm, int32_t bk,
                                         kairo_dtype dtype, float* norms, void* stream);
KAIRO_API kairo_status kairo_bsr_block_norms(const kairo_bsr* a, float* norms, void* stream);
KAIRO_API kairo_status kairo_topk_indices(const float* scores, int64_t n, int64_t count, int64_t* out,
                                          void* workspace, size_t workspace_bytes, void* stream);
KAIRO_API kairo_status kairo_topk_workspace_size(int64_t n, size_t* bytes);

/* ------------------------------------------------------------------------
 * Masked embedding lookup and its gradient (the reference's other extension
 * functions, csrc/bindings.cpp:39-82 -> csrc/sparse_embedding_kernel.cu:
 * 135-219, called from kairo/ops/sparse_embedding.py:59-161).
 *   kairo_coo_sort_rows   stable sort of a COO element mask by row on the
 *                         device (_sort_coo_by_row, sparse_embedding.py:49-56)
 *                         and its int64 row offsets (_coo_to_row_offsets,
 *                         :23-46).  rows_sorted and perm may be NULL.  Rows of
 *                         more than 16384 entries keep an unspecified order.
 *                         Ids outside [0, n_rows) x [0, n_cols) set the
 *                         workspace error word (KAIRO_DEVERR_BAD_INDEX).
 *   kairo_sparse_gather   out[b, :] = weight[ids[b], :] on the row's active
 *                         columns, 0 elsewhere; an id outside [0, n_rows)
 *                         gives a zero row (sparse_gather_forward).  weight
 *                         is (n_rows, dim) row-major, out (nids, dim); mask
 *                         values are not read (an entry means "active").
 *   kairo_sparse_scatter_grad
 *                         grad_weight (n_rows, dim, written whole) = the sum
 *                         of grad_output's rows b with batch_ids[b] == r for
 *                         every r in active_ids (sorted, unique), 0 on all
 *                         other rows (sparse_scatter_backward).  Sums run in
 *                         fp32 in ascending b order: deterministic, no
 *                         atomics.  An active id outside [0, n_rows) sets
 *                         the workspace error word.
 * dtype f32, f16 or bf16; all asynchronous on `stream`.
 * ---------------------------------------------------------------------- */
KAIRO_API kairo_status kairo_coo_sort_rows(const int64_t* rows, const int64_t* cols, int64_t nnz, int64_t n_rows,
                                           int64_t n_cols, int64_t* row_offsets, int64_t* rows_sorted,
                                           int64_t* cols_sorted, int64_t* perm, void* workspace,
                                           size_t workspace_bytes, void* stream);
KAIRO_API kairo_status kairo_coo_sort_rows_workspace_size(int64_t n_rows, int64_t nnz, size_t* bytes);
KAIRO_API kairo_status kairo_sparse_gather(const void* weight, int64_t n_rows, int64_t dim, kairo_dtype dtype,
                                           const int64_t* row_offsets, const int64_t* mask_cols, int64_t nnz,
                                           const int64_t* ids, int64_t nids, void* out, void* stream);
/* Row bitmask of a COO element mask: bits is (n_rows, ceil(n_cols / 32))
 * uint32 words, bit c % 32 of word c / 32 of row r set for entry (r, c);
 * entries outside the grid are skipped.  kairo_sparse_gather_bits is
 * kairo_sparse_gather reading that bitmask instead of the row offsets and
 * columns (same result; whole rows are read with 16-byte vectors). */
KAIRO_API kairo_status kairo_mask_bits(const int64_t* rows, const int64_t* cols, int64_t nnz, int64_t n_rows,
                                       int64_t n_cols, uint32_t* bits, void* stream);
KAIRO_API kairo_status kairo_sparse_gather_bits(const void* weight, int64_t n_rows, int64_t dim, kairo_dtype dtype,
                                                const uint32_t* bits, const int64_t* ids, int64_t nids, void* out,
                                                void* stream);
KAIRO_API kairo_status kairo_sparse_scatter_grad(const void* grad_output, kairo_dtype dtype,
                                                 const int64_t* active_ids, int64_t nactive,
                                                 const int64_t* batch_ids, int64_t nbatch, int64_t n_rows,
                                                 int64_t dim, void* grad_weight, void* workspace,
                                                 size_t workspace_bytes, void* stream);
KAIRO_API kairo_status kairo_sparse_scatter_grad_workspace_size(int64_t nactive, int64_t nbatch, size_t* bytes);

/* ------------------------------------------------------------------------
 * Diagnostics (no counterpart in the reference): the rate at which the SMs
 * pull bulk copies of `load_bytes` (a multiple of 16 dividing 32768) from
 * pseudo-random offsets of `buffer` into shared memory, in GB/s summed over
 * all SMs.  With a buffer smaller than the L2 this is the L2 -> SM gather
 * ceiling that bounds the tcgen05 kernels (one gathered panel per block).
 * Runs one CTA per SM on `stream` and synchronises it.
 * ---------------------------------------------------------------------- */
KAIRO_API kairo_status kairo_gather_probe(const void* buffer, size_t buffer_bytes, uint32_t load_bytes,
                                          int32_t iterations, double* gb_per_s, void* stream);

/* ------------------------------------------------------------------------
 * Dense A (M x K, leading dimension lda) -> tiles (num_tiles, tile, tile) in
 * COO order, zero-padding tiles that cross the right/bottom edge.  Replaces
 * the per-tile host loop of _dense_to_block_sparse (kairo/ops/spmm.py:16-55).
 * ---------------------------------------------------------------------- */
KAIRO_API kairo_status kairo_dense_to_tiles(const void* a, int64_t m, int64_t k, int64_t lda,
                                  const int32_t* tile_row_ids, const int32_t* tile_col_ids,
                                  int64_t num_tiles, int32_t tile, kairo_dtype dtype,
                                  void* tiles, void* stream);

/* ------------------------------------------------------------------------
 * The reference extension function acc_spmm_forward
 * (csrc/bindings.cpp:84-103 -> csrc/acc_spmm_kernel.cu:158-207):
 * C[M x N] (fp32, caller-allocated) = sum over tiles t of
 * A_tiles[t] * B[col_t*tile_k : +tile_k, :] placed at rows row_t*tile_m.
 * Tiles may come in any order (mask order); they are converted to BSR with
 * the stable row sort above.  dtype is the dtype of A_tiles and B (the
 * reference accepts f32 for any tile and f16 for tile 16; this library
 * accepts f32, f16 and bf16 for tiles 16/32/64).  num_tiles == 0 writes
 * zeros, like the reference's zero-initialised output.
 * Synchronises `stream` once (through kairo_bsr_build).
 * ---------------------------------------------------------------------- */
KAIRO_API kairo_status kairo_acc_spmm_forward(const void* a_tiles, const int32_t* tile_row_ids,
                                    const int32_t* tile_col_ids, const void* b, float* c,
                                    int32_t m, int32_t k, int32_t n, int32_t num_tiles,
                                    int32_t tile_m, int32_t tile_k, kairo_dtype dtype,
                                    void* workspace, size_t workspace_bytes, void* stream);
KAIRO_API kairo_status kairo_acc_spmm_forward_workspace_size(int32_t m, int32_t k, int32_t n,
                                                   int32_t num_tiles, int32_t tile_m,
                                                   int32_t tile_k, kairo_dtype dtype,
                                                   size_t* bytes);

/* ------------------------------------------------------------------------
 * Host helper: nnz-balanced contiguous block-row partition for multi-GPU
 * sharding.  row_ptr is a HOST array (nbr+1, int64).  bounds (parts+1) gets
 * bounds[p] = lower_bound(row_ptr, p * nnzb / parts) (clamped, monotone),
 * bounds[0] = 0, bounds[parts] = nbr.  The reference has no multi-GPU path;
 * this is the partition rule of the sharded SpMM.
 * ---------------------------------------------------------------------- */
KAIRO_API kairo_status kairo_partition_rows(const int64_t* row_ptr, int32_t nbr, int32_t parts,
                                  int32_t* bounds);

/* Reads (and optionally clears) the device error word of a workspace.
 * Synchronises `stream`.  *code receives KAIRO_DEVERR_* in the low 8 bits and
 * a location tag in the upper bits (0 when no error was recorded). */
KAIRO_API kairo_status kairo_workspace_error(void* workspace, int32_t clear, uint32_t* code,
                                   void* stream);

KAIRO_API const char* kairo_status_string(kairo_status s);
KAIRO_API const char* kairo_last_error_message(void);
KAIRO_API int32_t kairo_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KAIRO_SPMM_H_ */
