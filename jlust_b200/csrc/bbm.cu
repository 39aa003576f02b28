// bbm.cu -- SpMV of a periodic block-banded matrix on sm_100a without
// building its T-fold copy.
//
// The matrix has T periods of n_cols columns.  One diagonal block D
// (n_diag x n_cols CSR, plus optional selector patches) is shared by every
// period and one coupling pair (neg, pos; n_off x n_cols each, CSR or a
// ShiftedDiag selector) by every transition t -> t+1.  Rows run period by
// period: period t's n_diag diagonal rows compute D x_t, then (for t < T-1)
// its n_off coupling rows compute neg x_t + pos x_{t+1}.  One thread per
// output row finds its period and kind from its index and walks the shared
// block with the period's column offset.  A diagonal row sums its CSR
// entries, then adds the sum of its patches; a coupling row adds its neg
// entries, then its pos entries, into one sum (a ShiftedDiag block adds its
// one term val * x[row + shift]); all in storage order with separately
// rounded products and sums: the order of JLUST's fused periodic kernel
// (ext/KernelAbstractionsExt/ops/block_periodic.jl:114-163), so the result is
// bit-identical to the oracle's restatement of it.  The shared blocks are
// read once per period from L2, not stored T times.
#include "common.cuh"

namespace jlb {

JLB_DEFINE_DEV_ERROR(bbm)

namespace bbm {

constexpr int kThreads = 256;

// One shared block: CSR when rowptr is set, else a ShiftedDiag selector
// (row r holds sel at column r + shift).
struct Block {
    const int32_t *rowptr, *colind;
    const void *val;
    int64_t shift;
    double sel;
};

// Adds row `row` of a shared CSR block into acc in storage order, columns
// shifted by col_off; four entries' loads are issued before their sums.  A
// column outside the block is reported and skipped.
template <typename T>
__device__ __forceinline__ T walk(int64_t row, const int32_t *__restrict__ rowptr,
                                  const int32_t *__restrict__ colind, const T *__restrict__ val,
                                  const T *__restrict__ x, int64_t col_off, int64_t n_cols,
                                  int base, T acc) {
    const int lo = ldg(rowptr + row) - base, hi = ldg(rowptr + row + 1) - base;
    int k = lo;
    for (; k + 4 <= hi; k += 4) {
        int c[4];
        T v[4], xv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            c[u] = ldg(colind + k + u) - base;
            v[u] = ldg(val + k + u);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const bool in = c[u] >= 0 && c[u] < n_cols;
            if (!in) dev_error(DEV_ERR_BOUNDS);
            xv[u] = in ? ldg(x + col_off + c[u]) : T(0);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (c[u] >= 0 && c[u] < n_cols) acc = add_rn(acc, mul_rn(v[u], xv[u]));
    }
    for (; k < hi; ++k) {
        const int64_t c = (int64_t)(ldg(colind + k) - base);
        if (c < 0 || c >= n_cols) {
            dev_error(DEV_ERR_BOUNDS);
            continue;
        }
        acc = add_rn(acc, mul_rn(ldg(val + k), ldg(x + col_off + c)));
    }
    return acc;
}

// Row `row` of a coupling block added into acc: the CSR walk, or the
// selector's one term.
template <typename T>
__device__ __forceinline__ T leaf(int64_t row, const Block &b, const T *__restrict__ x,
                                  int64_t col_off, int64_t n_cols, int base, T acc) {
    if (b.rowptr)
        return walk<T>(row, b.rowptr, b.colind, (const T *)b.val, x, col_off, n_cols, base, acc);
    const int64_t c = row + b.shift;
    if (c < 0 || c >= n_cols) {
        dev_error(DEV_ERR_BOUNDS);
        return acc;
    }
    return add_rn(acc, mul_rn((T)b.sel, ldg(x + col_off + c)));
}

template <typename T, bool kBeta>
__global__ void __launch_bounds__(kThreads)
periodic_rows(int64_t T_periods, int64_t n_diag, int64_t n_off, int64_t n_cols, Block diag,
              int npatch, const int64_t *__restrict__ prows, const int64_t *__restrict__ pcols,
              const double *__restrict__ pvals, Block neg, Block pos, const T *__restrict__ x,
              T *__restrict__ y, T alpha, T beta, int base) {
    const int64_t rows = T_periods * n_diag + (T_periods - 1) * n_off;
    const int64_t r = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (r >= rows) return;
    const int64_t period = n_diag + n_off;
    const int64_t t = r / period, rem = r - t * period;
    T acc = T(0);
    if (rem < n_diag) {
        acc = walk<T>(rem, diag.rowptr, diag.colind, (const T *)diag.val, x, t * n_cols, n_cols,
                      base, acc);
        if (npatch > 0) {
            bool bad = false;
            acc = add_rn(acc, patch_sum<T>(rem, npatch, prows, pcols, pvals, x, t * n_cols, n_cols,
                                           bad));
            if (bad) dev_error(DEV_ERR_BOUNDS);
        }
    } else {
        acc = leaf<T>(rem - n_diag, neg, x, t * n_cols, n_cols, base, acc);
        acc = leaf<T>(rem - n_diag, pos, x, (t + 1) * n_cols, n_cols, base, acc);
    }
    T out = mul_rn(alpha, acc);
    if (kBeta) out = add_rn(out, mul_rn(beta, y[r]));
    y[r] = out;
}

template <typename T>
int launch(cudaStream_t st, int base, int64_t Tp, int64_t n_diag, int64_t n_off, int64_t n_cols,
           const Block &diag, int npatch, const int64_t *prows, const int64_t *pcols,
           const double *pvals, const Block &neg, const Block &pos, const void *x, void *y,
           double alpha, double beta) {
    const int64_t rows = Tp * n_diag + (Tp - 1) * n_off;
    if (rows == 0) return ok();
    const unsigned grid = (unsigned)ceil_div(rows, kThreads);
    const T a = (T)alpha, b = (T)beta;
    if (b == T(0))
        periodic_rows<T, false><<<grid, kThreads, 0, st>>>(Tp, n_diag, n_off, n_cols, diag, npatch,
                                                           prows, pcols, pvals, neg, pos,
                                                           (const T *)x, (T *)y, a, b, base);
    else
        periodic_rows<T, true><<<grid, kThreads, 0, st>>>(Tp, n_diag, n_off, n_cols, diag, npatch,
                                                          prows, pcols, pvals, neg, pos,
                                                          (const T *)x, (T *)y, a, b, base);
    JLB_LAUNCH_CHECK("periodic_rows");
    return ok();
}

}  // namespace bbm
}  // namespace jlb

using namespace jlb;

extern "C" JLB_API int jlb_bbm_periodic_spmv(
    void *stream, int dtype, int idx_base, int64_t T, int64_t n_diag, int64_t n_off,
    int64_t n_cols, const int32_t *diag_rowptr, const int32_t *diag_colind, const void *diag_val,
    int npatch, const int64_t *patch_rows, const int64_t *patch_cols, const double *patch_vals,
    const int32_t *neg_rowptr, const int32_t *neg_colind, const void *neg_val, int64_t neg_shift,
    double neg_sel, const int32_t *pos_rowptr, const int32_t *pos_colind, const void *pos_val,
    int64_t pos_shift, double pos_sel, const void *x, void *y, double alpha, double beta) {
    if (dtype != JLB_F32 && dtype != JLB_F64)
        return fail(JLB_ERR_UNSUPPORTED_VALUE_TYPE, "periodic SpMV supports Float32 and Float64");
    if (idx_base != 0 && idx_base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (T < 1 || n_diag < 0 || n_off < 0 || n_cols < 0)
        return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "need T >= 1 and non-negative block sizes");
    if (!x || !y || !diag_rowptr) return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    if (npatch < 0 || (npatch > 0 && (!patch_rows || !patch_cols || !patch_vals)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "bad patch arrays");
    if (n_off > 0 && T > 1) {
        const int64_t shifts[2] = {neg_shift, pos_shift};
        const int32_t *rps[2] = {neg_rowptr, pos_rowptr};
        for (int s = 0; s < 2; ++s)
            if (!rps[s] && (shifts[s] < 0 || n_off - 1 + shifts[s] >= n_cols))
                return fail(JLB_ERR_INCOMPATIBLE_EXTENTS,
                            "ShiftedDiag coupling block reaches outside its columns");
    }
    const bbm::Block diag{diag_rowptr, diag_colind, diag_val, 0, 0.0};
    const bbm::Block neg{neg_rowptr, neg_colind, neg_val, neg_shift, neg_sel};
    const bbm::Block pos{pos_rowptr, pos_colind, pos_val, pos_shift, pos_sel};
    if (dtype == JLB_F64)
        return bbm::launch<double>(as_stream(stream), idx_base, T, n_diag, n_off, n_cols, diag,
                                   npatch, patch_rows, patch_cols, patch_vals, neg, pos, x, y,
                                   alpha, beta);
    return bbm::launch<float>(as_stream(stream), idx_base, T, n_diag, n_off, n_cols, diag, npatch,
                              patch_rows, patch_cols, patch_vals, neg, pos, x, y, alpha, beta);
}
