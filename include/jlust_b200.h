/*
 * jlust_b200.h -- C ABI of libjlust_b200.so, the B200 (sm_100a) sparse-kernel
 * backend for JLUST.
 *
 * The library is what a `B200Backend <: AbstractUSTBackend` Julia extension
 * reaches with `ccall`: plain pointers, sizes and enums, no C++ or torch types.
 * Every entry point returns an int status (JLB_OK == 0); a failing call also
 * stores a message retrievable with jlb_last_error() on the calling thread.
 * Nothing throws across the ABI.
 *
 * Ownership: all matrix / vector buffers are device memory owned by the caller
 * (CuArray in Julia).  The library never frees or retains them beyond a call,
 * except that a plan remembers the index buffers it was created from; the
 * caller keeps those alive until jlb_*_plan_destroy.
 *
 * Streams: `stream` is a cudaStream_t passed as void* (NULL = legacy default
 * stream).  Execute calls are asynchronous, never synchronise the host and
 * never allocate device memory, so they can be captured into CUDA graphs.
 * Plan creation and conversion count phases synchronise `stream`.
 *
 * Index origin: idx_base is 0 (ZeroBased) or 1 (OneBased), applied to every
 * position and coordinate buffer, as JLUST's `_origin_off`
 * (ext/KernelAbstractionsExt/ops/spmv.jl:380).
 *
 * Dense operands carry (order, leading dimension): order JLB_ROW_MAJOR puts
 * element (i, j) at i*ld + j, JLB_COL_MAJOR at i + j*ld (Julia's native
 * layout, ext/CUDAExt/ops/spmm.jl:1-4).
 */
#ifndef JLUST_B200_H
#define JLUST_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define JLB_API __attribute__((visibility("default")))

/* Status codes.  Codes 1-7 map one to one onto JLUST's exception types
 * (src/errors.jl:1-9); the Julia glue rethrows them as those exceptions. */
enum jlb_status_code {
    JLB_OK = 0,
    JLB_ERR_UNSUPPORTED_FORMAT = 1,     /* UnsupportedFormat      errors.jl:3 */
    JLB_ERR_UNSUPPORTED_INDEX_TYPE = 2, /* UnsupportedIndexType   errors.jl:4 */
    JLB_ERR_UNSUPPORTED_VALUE_TYPE = 3, /* UnsupportedValueType   errors.jl:5 */
    JLB_ERR_INDEX_ORIGIN_MISMATCH = 4,  /* IndexOriginMismatch    errors.jl:6 */
    JLB_ERR_DEVICE_MISMATCH = 5,        /* DeviceMismatch         errors.jl:7 */
    JLB_ERR_INCOMPATIBLE_EXTENTS = 6,   /* IncompatibleExtents    errors.jl:8 */
    JLB_ERR_NONCANONICAL_STORAGE = 7,   /* NonCanonicalStorage    errors.jl:9 */
    JLB_ERR_INVALID_ARGUMENT = 8,       /* null pointer, bad enum, bad alignment */
    JLB_ERR_CUDA = 9,                   /* a CUDA runtime / driver call failed */
    JLB_ERR_DEVICE_TIMEOUT = 10,        /* a bounded device-side wait gave up */
    JLB_ERR_WORKSPACE = 11              /* workspace smaller than the size query */
};

/* Value types (JLUST eltype): Float32, Float64, BFloat16. */
enum jlb_dtype { JLB_F32 = 0, JLB_F64 = 1, JLB_BF16 = 2 };

/* Dense layouts. */
enum jlb_order { JLB_ROW_MAJOR = 0, JLB_COL_MAJOR = 1 };

/* SDDMM modes. */
enum jlb_sddmm_mode {
    JLB_SDDMM_ADD = 0, /* out[p] = alpha*dot + beta*out[p]        (reference) */
    JLB_SDDMM_MUL = 1  /* out[p] = (alpha*dot)*S[p] + beta*out[p] (sampled)   */
};

typedef struct jlb_spmv_plan_s *jlb_spmv_plan;
typedef struct jlb_spmm_plan_s *jlb_spmm_plan;
typedef struct jlb_spgemm_plan_s *jlb_spgemm_plan;

/* ---------------------------------------------------------------- runtime */

/* Library version, major*10000 + minor*100 + patch. */
JLB_API int jlb_version(void);

/* Static description of a status code. */
JLB_API const char *jlb_status_string(int status);

/* Copies the calling thread's last error message into buf (always
 * NUL-terminated when len > 0) and returns the last status. */
JLB_API int jlb_last_error(char *buf, size_t len);

/* Binds the calling thread to `device` and checks that it is an sm_100 part.
 * Replaces nothing in the reference (CUDA.jl does this implicitly). */
JLB_API int jlb_init(int device);

/* Synchronises `stream`, then reads and clears the device error word that
 * kernels set when a bounded wait gave up or a bounds check failed.  Returns
 * JLB_OK, JLB_ERR_DEVICE_TIMEOUT or JLB_ERR_NONCANONICAL_STORAGE. */
JLB_API int jlb_device_status(void *stream);

/* ------------------------------------------------------- validation (CSR) */

/* Checks the invariants JLUST's validate_storage (src/backends.jl:309-316)
 * and the kernels rely on: rowptr[0] == idx_base, rowptr non-decreasing,
 * rowptr[m] == nnz + idx_base, idx_base <= colind < n + idx_base and, when
 * `require_sorted` is set, strictly increasing columns inside each row.
 * Synchronises `stream`.  Returns JLB_ERR_NONCANONICAL_STORAGE on violation. */
JLB_API int jlb_csr_validate(void *stream, int idx_base, int64_t m, int64_t n, int64_t nnz,
                             const int32_t *rowptr, const int32_t *colind, int require_sorted);

/* ------------------------------------------------------------------- SpMV */

/* y = alpha * A * x + beta * y for an m x n CSR matrix A (dtype F32 or F64).
 * beta == 0 never reads y.  Rows of up to 32 entries are summed in storage
 * order with separately rounded products and sums, which reproduces JLUST's
 * CPU walker bit for bit; longer rows use a fixed-order warp reduction.
 * Replaces execute(::EmitterBackend, ::Op{:SpMV}) in
 * ext/KernelAbstractionsExt/ops/spmv.jl:371-504 (walker kernels K1/K2) and
 * the merge-based hook _csr_spmv_merge! in ext/CUDAExt/ops/spmv.jl:195-208. */
JLB_API int jlb_csr_spmv(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                         int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                         const void *val, const void *x, void *y, double alpha, double beta);

/* y = alpha * A * x + beta * y for an m x n DCSR matrix: nfib stored rows,
 * row_ids[f] (nfib, the outer level's coordinates) the row of stored row f,
 * fibptr (nfib + 1, the inner level's positions) and colind / val its
 * entries.  Stored rows are summed exactly as jlb_csr_spmv sums a CSR row;
 * rows that are not stored are not written (JLUST's DCSR walk,
 * ext/KernelAbstractionsExt/ops/_walker.jl:323-342, dispatched from
 * ops/spmv.jl:371-504; KAT test/test_emitter.jl:127-157). */
JLB_API int jlb_dcsr_spmv(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                          int64_t nfib, int64_t nnz, const int32_t *fibptr,
                          const int32_t *row_ids, const int32_t *colind, const void *val,
                          const void *x, void *y, double alpha, double beta);

/* y = alpha * (A * x + P * x) + beta * y: a CSR A (m x n) plus npatch
 * selector patches P, patch p adding patch_vals[p] * x[r - patch_rows[2p] +
 * patch_cols[p]] to each row r in patch_rows[2p] .. patch_rows[2p+1]
 * (0-based, inclusive; the patch arrays are device memory).  Each row's CSR
 * entries are summed in storage order by one thread, the patches into a
 * second sum in patch order, and the two added: JLUST's BlockSparseMatrix
 * kernel with selector patches (ext/KernelAbstractionsExt/ops/
 * block_periodic.jl:40-79, launched from ext/CUDAExt/ops/block_mul.jl:275-288,
 * which has alpha = 1).  rowptr may be NULL when nnz = 0: no CSR entries, as
 * for a standalone ShiftedDiag tensor (one patch over all rows; JLUST's
 * walker with a ShiftedDiag leaf, src/backends.jl:223-227). */
JLB_API int jlb_csr_patched_spmv(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                 int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                                 const void *val, int npatch, const int64_t *patch_rows,
                                 const int64_t *patch_cols, const double *patch_vals,
                                 const void *x, void *y, double alpha, double beta);

/* y = alpha * A * x + beta * y for COO (row and column coordinates per entry,
 * any order, duplicates add) and for CSC (column pointer n + 1, row
 * coordinates).  As in JLUST's COO and scatter paths
 * (ext/KernelAbstractionsExt/ops/spmv.jl:386-420, ops/_walker.jl:343-375),
 * y is scaled by beta first (set to 0 when beta == 0) and every entry adds
 * alpha * v * x[col] to its row with an atomic add, so the order of a row's
 * terms is not fixed: results agree within floating-point tolerance, not
 * bit for bit.  KAT test/test_emitter.jl:161-192 (COO). */
JLB_API int jlb_coo_spmv(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                         int64_t nnz, const int32_t *rows, const int32_t *cols, const void *val,
                         const void *x, void *y, double alpha, double beta);
JLB_API int jlb_csc_spmv(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                         int64_t nnz, const int32_t *colptr, const int32_t *rowind,
                         const void *val, const void *x, void *y, double alpha, double beta);

/* y = alpha * M * x + beta * y for a periodic block-banded matrix M with T
 * periods of n_cols columns: one n_diag x n_cols diagonal block shared by
 * every period (a CSR plus npatch selector patches, encoded as for
 * jlb_csr_patched_spmv with rows and columns relative to the block) and one
 * coupling pair (neg, pos; n_off x n_cols) shared by every transition, each
 * a CSR or, when its rowptr is NULL, a ShiftedDiag selector whose row r holds
 * *_sel at column r + *_shift.  Rows run period by period -- period t's
 * diagonal rows (D x_t), then for t < T-1 its coupling rows
 * (neg x_t + pos x_{t+1}) -- T*n_diag + (T-1)*n_off rows in all, without
 * storing the T-fold matrix.  A diagonal row sums its CSR entries in storage
 * order, then adds its patches' sum; a coupling row sums neg's entries, then
 * pos's, into one sum: JLUST's fused periodic kernel
 * (ext/KernelAbstractionsExt/ops/block_periodic.jl:114-163, launched from
 * ext/CUDAExt/ops/block_mul.jl:660-680). */
JLB_API int jlb_bbm_periodic_spmv(void *stream, int dtype, int idx_base, int64_t T, int64_t n_diag,
                                  int64_t n_off, int64_t n_cols, const int32_t *diag_rowptr,
                                  const int32_t *diag_colind, const void *diag_val, int npatch,
                                  const int64_t *patch_rows, const int64_t *patch_cols,
                                  const double *patch_vals, const int32_t *neg_rowptr,
                                  const int32_t *neg_colind, const void *neg_val,
                                  int64_t neg_shift, double neg_sel, const int32_t *pos_rowptr,
                                  const int32_t *pos_colind, const void *pos_val,
                                  int64_t pos_shift, double pos_sel, const void *x, void *y,
                                  double alpha, double beta);

/* Prepared SpMV: validates the structure once, records the row-length
 * profile and picks the kernel variant.  Replaces prepare(backend, SpMVOp,
 * u_A) (src/ops.jl:187-202; EmitterSpMVHandle, KA spmv.jl:518-531). */
JLB_API int jlb_spmv_plan_create(jlb_spmv_plan *plan, void *stream, int dtype, int idx_base,
                                 int64_t m, int64_t n, int64_t nnz, const int32_t *rowptr,
                                 const int32_t *colind);
/* execute(h, u_A, u_x, u_y; alpha, beta) (KA spmv.jl:533-544); `val` may be a
 * new value buffer of the same structure (update_values!, src/ops.jl:204-211). */
JLB_API int jlb_spmv_plan_execute(jlb_spmv_plan plan, void *stream, const void *val,
                                  const void *x, void *y, double alpha, double beta);
/* Row-length profile recorded by the plan: max and mean entries per row and
 * the kernel variant the plan picked from them (the reference's warp-vector
 * choice, KA spmv.jl:296-323, re-tuned on B200).  Variant 0: a thread per
 * row, summing in storage order (bit-exact with the CPU walker) for rows of
 * up to 32 entries, a warp for longer rows.  Variant W (2, 4, 8, 16, 32):
 * groups of W lanes per row, 16-byte loads of four columns and values per
 * lane, a fixed-order butterfly across the group (within tolerance).  The
 * plan takes 4 when the mean row length is 12 to 96 and no row exceeds 128
 * entries, else 0. */
JLB_API int jlb_spmv_plan_info(jlb_spmv_plan plan, int64_t *max_row, double *mean_row,
                               int *variant);
/* Overrides the plan's variant, e.g. to tune it for a matrix: 0 (a thread
 * per row, the warp for rows over 32 entries), 1 (the same sums with each
 * block of 1024 rows' window of x -- columns [row - lower bandwidth, row +
 * upper bandwidth], from the plan's scan -- staged in shared memory by one
 * bulk copy: banded structure; variant 0 runs when the window does not fit),
 * or W = 2, 4, 8, 16, 32 (groups of W lanes per row).  No counterpart in the
 * reference. */
JLB_API int jlb_spmv_plan_set_variant(jlb_spmv_plan plan, int variant);
JLB_API int jlb_spmv_plan_destroy(jlb_spmv_plan plan);

/* ------------------------------------------------------------------- SpMM */

/* C = alpha * A * B + beta * C; A m x n CSR (F32 or F64), B n x k, C m x k,
 * each with its own order and leading dimension.  beta == 0 never reads C.
 * Per (row, column) the sum runs over the row's entries in storage order
 * (bit-exact with JLUST's Tiled strategy, KA spmm.jl:272-292) for rows of up
 * to 256 entries; longer rows are split into 16 segments combined in order.
 * Replaces execute(::EmitterBackend, ::Op{:SpMM}) (KA spmm.jl:397-423) and
 * the CUSPARSEBackend SpMM default (ext/CUDAExt/ops/spmm.jl:50-58). */
JLB_API int jlb_csr_spmm(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                         int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                         const void *val, int64_t k, const void *B, int64_t ldb, int b_order,
                         void *C, int64_t ldc, int c_order, double alpha, double beta);

/* jlb_csr_spmm with a caller workspace, for JLUST's native column-major B
 * and C (KA spmm.jl:31-38, ext/CUDAExt/ops/spmm.jl:1-4): on the stream, a
 * column-major B is transposed into the workspace (n*k values) and its rows
 * are gathered from there, and a column-major C is computed row-major in the
 * workspace (m*k values; transposed in first when beta != 0) and transposed
 * out.  The streaming kernels' order of operations -- hence the results --
 * is the row-major case's.  Without a large enough workspace the call
 * behaves as jlb_csr_spmm.  jlb_csr_spmm_workspace_size returns 0 when no
 * workspace is used.  Same contract as execute(::EmitterBackend,
 * ::Op{:SpMM}) (KA spmm.jl:397-423). */
JLB_API size_t jlb_csr_spmm_workspace_size(int dtype, int64_t m, int64_t n, int64_t k,
                                           int b_order, int c_order);
JLB_API int jlb_csr_spmm_ws(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                            int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                            const void *val, int64_t k, const void *B, int64_t ldb, int b_order,
                            void *C, int64_t ldc, int c_order, double alpha, double beta,
                            void *workspace, size_t workspace_bytes);

/* ------------------------------------------------------------------ SDDMM */

/* Sampled dense-dense product over the sparsity pattern of the m x n CSR
 * matrix (rowptr, colind): for every stored position p = (i, j)
 *   dot = sum_{kk < K} A(i, kk) * B(kk, j)
 * with A m x K (order a_order, leading dim lda) and B the K x n operand
 * (order b_order, leading dim ldb; a row-major n x K array is the K x n
 * operand in JLB_COL_MAJOR with ldb = K).  mode JLB_SDDMM_ADD writes
 * out[p] = alpha*dot + beta*out[p] (KA sddmm.jl:23-36); JLB_SDDMM_MUL writes
 * out[p] = (alpha*dot)*S[p] + beta*out[p].  beta == 0 never reads out.
 * Replaces execute(::EmitterBackend, ::Op{:SDDMM}) (KA sddmm.jl:49-65) and
 * the CUSPARSEBackend SDDMM default (ext/CUDAExt/ops/sddmm.jl:53-62). */
JLB_API int jlb_sddmm(void *stream, int dtype, int idx_base, int64_t m, int64_t n, int64_t nnz,
                      const int32_t *rowptr, const int32_t *colind, int64_t K, const void *A,
                      int64_t lda, int a_order, const void *B, int64_t ldb, int b_order,
                      const void *S, void *out, int mode, double alpha, double beta);

/* --------------------------------------------------------------- BSR SpMM */

/* C = alpha * A * B + beta * C for a BSRRight((bs, bs)) matrix A with mb
 * block rows, nb block columns and nnzb stored row-major bs x bs blocks of
 * bf16 values; B is (nb*bs) x N bf16 row-major (leading dim ldb), C is
 * (mb*bs) x N fp32 row-major (leading dim ldc); fp32 accumulation.
 * bs == 64 with N a multiple of 128 (N <= 512), ldb a multiple of 8 and
 * 16-byte aligned B and values runs on tcgen05 tensor cores (TMA-fed shared
 * memory tiles, accumulators in TMEM); other shapes run a SIMT kernel.
 * Replaces execute(BlockSpMMOp, ...) (src/block_sparse.jl:284-302; fused CPU
 * loop :177-188) for BSR-structured block matrices, which the reference
 * cannot run on the GPU (no BSR path in ext/CUDAExt/CUDAExt.jl:253-290). */
JLB_API int jlb_bsr_spmm(void *stream, int idx_base, int64_t mb, int64_t nb, int64_t nnzb,
                         int bs, const int32_t *browptr, const int32_t *bcolind,
                         const void *bval, int64_t N, const void *B, int64_t ldb, float *C,
                         int64_t ldc, double alpha, double beta);

/* ------------------------------------------------ conversion and scans */

/* Exclusive scan of n int32 counts into n+1 positions, out[0] = idx_base
 * (the composer's position buffer, src/convert.jl:154-168).  `workspace`
 * holds at least jlb_scan_workspace_size(n) bytes of device memory.  `out`
 * may alias `counts` shifted by one (in-place scan of a row pointer whose
 * entries 1..n hold counts).  Overflow of int32 sets the device error word. */
JLB_API size_t jlb_scan_workspace_size(int64_t n);
JLB_API int jlb_exclusive_scan_i32(void *stream, int64_t n, const int32_t *counts, int32_t *out,
                                   int idx_base, void *workspace, size_t workspace_bytes);

/* Allocation-free variant of jlb_exclusive_scan_i32, with no counterpart in
 * the reference.  It is for callers that cannot call cudaMalloc -- for
 * example code that must not re-enter a memory pool (Julia finalizers and
 * callbacks run while CUDA.jl's allocator may be busy) or that runs on a
 * device whose memory is entirely handed to another allocator.  Its scratch
 * is a static 64 KB device array inside the library (present on every GPU
 * that loads it, until the process exits), so n is limited to 33,554,432
 * counts; larger n fails with JLB_ERR_INVALID_ARGUMENT.  The first call on a
 * device looks up that array's device address (cudaGetSymbolAddress), so
 * make the first call on each device before any stream capture.  All calls
 * share the one array: calls that may run concurrently on the GPU (other
 * streams, other host threads) race and must be serialised by the caller.
 * Same result and semantics as jlb_exclusive_scan_i32; allocates nothing.
 * n = 0 only writes out[0] = idx_base, by a kernel on the stream. */
#define JLB_SCAN_NOALLOC_MAX_N 33554432 /* 8192 tiles of 4096 counts */
JLB_API int jlb_exclusive_scan_i32_noalloc(void *stream, int64_t n, const int32_t *counts,
                                           int32_t *out, int idx_base);

/* CSR -> BSRRight((b1, b2)) on the GPU, bit-exact with JLUST's convert_format
 * (src/convert.jl:302-388) using the block-row level extent ceil(m/b1):
 * explicit zeros dropped, block columns ascending, b1 x b2 row-major tiles
 * zero-filled where no entry lands, output origin = input origin.
 * Phase 1 (count) fills browptr (ceil(m/b1)+1 entries) and returns nnzb in
 * *nnzb (synchronises `stream`); the caller allocates bcolind (nnzb) and bval
 * (nnzb*b1*b2 values of dtype); phase 2 (fill) writes them.  `workspace`
 * holds jlb_csr_to_bsr_workspace_size(...) bytes for both phases; passing the
 * same workspace to fill lets it reuse the block-column bitmaps that count
 * left there (matrices of up to 163,840 block columns), so fill reads the CSR
 * once.  Any other workspace, or a smaller one, is also correct: fill then
 * rebuilds the bitmaps.
 * Replaces convert_format(u, Formats.BSRRight((b1,b2))) for CSR sources and
 * cuSPARSE csr2bsr (supports_convert, ext/CUDAExt/CUDAExt.jl:330-339). */
JLB_API size_t jlb_csr_to_bsr_workspace_size(int64_t m, int64_t n, int64_t nnz, int b1, int b2);
JLB_API int jlb_csr_to_bsr_count(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                 int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                                 const void *val, int b1, int b2, int32_t *browptr,
                                 int64_t *nnzb, void *workspace, size_t workspace_bytes);
JLB_API int jlb_csr_to_bsr_fill(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                                const void *val, int b1, int b2, const int32_t *browptr,
                                int64_t nnzb, int32_t *bcolind, void *bval, void *workspace,
                                size_t workspace_bytes);

/* COO -> BSRRight((b1, b2)); entries in any order, duplicates allowed: the
 * nonzero entry with the lowest storage index wins a cell, as the composer's
 * stable sort keeps the first value of a run (src/convert.jl:222,231-238). */
JLB_API size_t jlb_coo_to_bsr_workspace_size(int64_t m, int64_t n, int64_t nnz, int b1, int b2,
                                             int64_t nnzb);
JLB_API int jlb_coo_to_bsr_count(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                 int64_t nnz, const int32_t *rows, const int32_t *cols,
                                 const void *val, int b1, int b2, int32_t *browptr,
                                 int64_t *nnzb, void *workspace, size_t workspace_bytes);
JLB_API int jlb_coo_to_bsr_fill(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                int64_t nnz, const int32_t *rows, const int32_t *cols,
                                const void *val, int b1, int b2, const int32_t *browptr,
                                int64_t nnzb, int32_t *bcolind, void *bval, void *workspace,
                                size_t workspace_bytes);

/* ----------------------------------------------------------------- SpGEMM */

/* Prepared sparse x sparse product C = alpha * A * B, A m x k and B k x n CSR
 * (Int32 indices, one origin), C m x n CSR with that origin: the reference's
 * prepare(EmitterBackend, SpGEMMOp, u_A, u_B) / EmitterSpGEMMHandle
 * (ext/KernelAbstractionsExt/ops/spgemm.jl:313-438; one-shot execute at
 * :493-506 is create + execute).  Create runs the symbolic pass on the index
 * buffers (synchronises `stream`, allocates the plan's device memory): C's
 * row i holds one entry per distinct column among the products of row i's A
 * entries with their B rows (explicit zeros included, as in the reference);
 * it returns nnz(C) and the product count (more than 2^31 - 2 products, or a
 * row of C with more than 2^24 products, is refused with
 * JLB_ERR_UNSUPPORTED_INDEX_TYPE).  Structure copies C's row pointer (m + 1)
 * and columns (ascending per row) into caller buffers.  Execute computes C's
 * values for value buffers a_val, b_val of the planned structures (the
 * handle's execute(h, u_A, u_B; alpha), :453-491): each entry is the sum from
 * zero of its products (A value * B value, times alpha unless alpha = 1) in
 * the order of A's entries then B's entries -- deterministic, where the
 * reference adds them by atomics.  F32 and F64; beta = 0 only, as in the
 * reference. */
JLB_API int jlb_spgemm_plan_create(jlb_spgemm_plan *plan, void *stream, int dtype, int idx_base,
                                   int64_t m, int64_t k, int64_t n, int64_t nnz_a,
                                   const int32_t *a_rowptr, const int32_t *a_colind, int64_t nnz_b,
                                   const int32_t *b_rowptr, const int32_t *b_colind,
                                   int64_t *nnz_c, int64_t *products);
JLB_API int jlb_spgemm_plan_structure(jlb_spgemm_plan plan, void *stream, int32_t *c_rowptr,
                                      int32_t *c_colind);
JLB_API int jlb_spgemm_plan_execute(jlb_spgemm_plan plan, void *stream, const void *a_val,
                                    const void *b_val, void *c_val, double alpha);
JLB_API int jlb_spgemm_plan_destroy(jlb_spgemm_plan plan);

/* COO -> CSR (convert_format(u, Formats.CSR) for a COO u, src/convert.jl:
 * 302-388).  JLUST's COO declares its rows ordered, so the reference composes
 * the entries in storage order without sorting: rows must not decrease
 * (NonCanonicalStorage otherwise, where the composer's assertion fails,
 * src/convert.jl:246), explicit zeros are dropped, columns keep their storage
 * order within a row, and an entry whose (row, column) equals that of the
 * nonzero entry before it is merged into it, keeping the first value.  Count
 * fills rowptr (m + 1, origin idx_base) and *nnz_out (synchronises `stream`);
 * the caller allocates colind and csr_val (nnz_out each); fill writes them
 * (columns keep the origin), reusing the flags count left in the workspace
 * when it gets the same workspace for the same buffers (any other workspace
 * of the queried size is also correct: fill then recomputes them; fill
 * synchronises `stream` to tell).  A CSR source converts the same way after
 * jlb_positions_to_coordinates expands its rows. */
JLB_API size_t jlb_coo_to_csr_workspace_size(int64_t m, int64_t n, int64_t nnz);
JLB_API int jlb_coo_to_csr_count(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                 int64_t nnz, const int32_t *rows, const int32_t *cols,
                                 const void *val, int32_t *rowptr, int64_t *nnz_out,
                                 void *workspace, size_t workspace_bytes);
JLB_API int jlb_coo_to_csr_fill(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                int64_t nnz, const int32_t *rows, const int32_t *cols,
                                const void *val, int64_t nnz_out, int32_t *colind, void *csr_val,
                                void *workspace, size_t workspace_bytes);

/* COO -> COO and, after jlb_positions_to_coordinates, CSR -> COO: a COO
 * target's levels are not unique and an ordered source is not sorted
 * (src/convert.jl:346-355), so only the explicit zeros go; the other entries
 * keep their storage order.  Count returns the number kept (synchronises
 * `stream`); fill writes rows_out, cols_out and val_out (nnz_out each). */
JLB_API size_t jlb_coo_drop_zeros_workspace_size(int64_t nnz);
JLB_API int jlb_coo_drop_zeros_count(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                     int64_t nnz, const int32_t *rows, const int32_t *cols,
                                     const void *val, int64_t *nnz_out, void *workspace,
                                     size_t workspace_bytes);
JLB_API int jlb_coo_drop_zeros_fill(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                    int64_t nnz, const int32_t *rows, const int32_t *cols,
                                    const void *val, int64_t nnz_out, int32_t *rows_out,
                                    int32_t *cols_out, void *val_out, void *workspace,
                                    size_t workspace_bytes);

/* Sorted compression: nnz (outer, inner) coordinate pairs compressed along the
 * outer coordinate with the entries lexsorted by (outer, inner, storage
 * index), explicit zeros dropped and the first of each run of equal
 * coordinates kept -- the composer's path when the target's level order
 * differs from the source's (src/convert.jl:334-345, 419-424): COO -> CSC
 * (outer = columns, inner = rows), CSR -> CSC (outer = colind, inner = the
 * expanded rows), CSC -> CSR (outer = rowind, inner = the expanded columns).
 * Count fills ptr (n_outer + 1, origin idx_base) and *nnz_out (synchronises
 * `stream`) and leaves the sorted entries in the workspace; fill needs that
 * same workspace, unchanged (JLB_ERR_WORKSPACE otherwise), and writes
 * inner_out and val_out (nnz_out each).  Outer indices holding more than
 * 16,777,216 entries are refused (UnsupportedIndexType). */
JLB_API size_t jlb_sorted_compress_workspace_size(int64_t n_outer, int64_t nnz);
JLB_API int jlb_sorted_compress_count(void *stream, int dtype, int idx_base, int64_t n_outer,
                                      int64_t n_inner, int64_t nnz, const int32_t *outer,
                                      const int32_t *inner, const void *val, int32_t *ptr,
                                      int64_t *nnz_out, void *workspace, size_t workspace_bytes);
JLB_API int jlb_sorted_compress_fill(void *stream, int dtype, int idx_base, int64_t n_outer,
                                     int64_t n_inner, int64_t nnz, const int32_t *outer,
                                     const int32_t *inner, const void *val, const int32_t *ptr,
                                     int64_t nnz_out, int32_t *inner_out, void *val_out,
                                     void *workspace, size_t workspace_bytes);

/* coords[k] = i + idx_base for every k in [ptr[i], ptr[i+1]) - idx_base: the
 * outer coordinate of each entry of a compressed level (the decomposer's walk
 * of a dense-over-compressed level, src/convert.jl:5-111). */
JLB_API int jlb_positions_to_coordinates(void *stream, int idx_base, int64_t n_outer, int64_t nnz,
                                         const int32_t *ptr, int32_t *coords);

/* ------------------------------------- row-partitioned SpMV (multi-GPU) */

/* Steps first_step .. first_step+nsteps-1 of x <- A x for a row-partitioned
 * iteration, each fused with its halo exchange over NVLink peer memory (one
 * process per GPU, one kernel launch per step).  No counterpart in the
 * reference, which has no multi-GPU layer; it serves the row-partitioned 2-D
 * Laplacian configuration.
 * This rank owns R rows of A (CSR, columns shifted into the halo buffer) and
 * keeps x in two buffers x_bufs[0..1] of R + 2h values laid out [lower halo |
 * own | upper halo]; step t reads x_bufs[t%2] and writes the own part of
 * x_bufs[(t+1)%2].  Steps count from 0 across calls.  Rows [interior_lo,
 * interior_hi) must read no halo entry.  lower_bufs / upper_bufs are the
 * neighbours' two buffers (peer pointers from jlb_ipc_open), or NULL at the
 * ends: the first h own results of step t are also stored into the lower
 * neighbour's buffer (t+1)%2 (its upper halo), the last h into the upper
 * neighbour's (its lower halo).  my_flags is this rank's int[4], zeroed once
 * before step 0: [published by lower, published by upper, internal,
 * internal]; lower_flag = &lower neighbour's my_flags[1], upper_flag =
 * &upper neighbour's my_flags[0].  Boundary rows wait (at most timeout_ns of
 * GPU time) for the neighbour's publication of step t; on expiry the device
 * error word reports JLB_ERR_DEVICE_TIMEOUT through jlb_device_status(). */
JLB_API int jlb_halo_spmv_steps(void *stream, int dtype, int idx_base, int64_t R, int64_t h,
                                int64_t interior_lo, int64_t interior_hi, const int32_t *rowptr,
                                const int32_t *colind, const void *val, void *const *x_bufs,
                                void *const *lower_bufs, void *const *upper_bufs, int *my_flags,
                                int *lower_flag, int *upper_flag, int first_step, int nsteps,
                                uint64_t timeout_ns);

/* CUDA IPC for the buffers above (no counterpart in the reference).
 * jlb_ipc_handle writes the 64-byte handle of the allocation containing ptr
 * and ptr's offset inside it; jlb_ipc_open maps a peer's handle and returns
 * the allocation's base (add the offset); jlb_ipc_close unmaps it. */
JLB_API int jlb_ipc_handle(void *ptr, void *handle_out, uint64_t *offset_out);
JLB_API int jlb_ipc_open(const void *handle, void **base_out);
JLB_API int jlb_ipc_close(void *base);

/* L2 residency for iterative solves (no counterpart in the reference).
 * Marks [base, base + bytes) as a persisting access-policy window on
 * `stream`: kernels launched on the stream afterwards keep up to the device's
 * persisting L2 set-aside of that range in L2 across launches (the window is
 * clipped to the device's maximum window size and the hit ratio set to
 * set-aside / window).  The set-aside is reserved for the calling process's
 * context and released with it.  bytes == 0 clears the window on the stream,
 * resets persisting lines to normal and returns the set-aside.  *persisted_out
 * (may be NULL) receives the bytes the set-aside covers. */
JLB_API int jlb_l2_persist(void *stream, const void *base, size_t bytes, size_t *persisted_out);

#ifdef __cplusplus
}
#endif

#endif /* JLUST_B200_H */
