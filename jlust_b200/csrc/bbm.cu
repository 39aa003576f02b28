// bbm.cu -- SpMV of a periodic block-banded matrix on sm_100a without
// building its T-fold copy.
//
// The matrix has T periods of n_cols columns.  One diagonal block D
// (n_diag x n_cols CSR) is shared by every period and one coupling pair
// (neg, pos; n_off x n_cols CSR each) by every transition t -> t+1.  Rows run
// period by period: period t's n_diag diagonal rows compute D x_t, then (for
// t < T-1) its n_off coupling rows compute neg x_t + pos x_{t+1}.  One thread
// per output row finds its period and kind from its index and walks the
// shared block with the period's column offset; a coupling row adds its neg
// entries, then its pos entries, into one sum, in storage order with
// separately rounded products and sums: the order of JLUST's fused periodic
// kernel (ext/KernelAbstractionsExt/ops/block_periodic.jl:126-163), so the
// result is bit-identical to the oracle's restatement of it.  The shared
// blocks are read once per period from L2, not stored T times.
#include "common.cuh"

namespace jlb {

JLB_DEFINE_DEV_ERROR(bbm)

namespace bbm {

constexpr int kThreads = 256;

// Adds row `row` of a shared block into acc in storage order, columns
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

template <typename T, bool kBeta>
__global__ void __launch_bounds__(kThreads)
periodic_rows(int64_t T_periods, int64_t n_diag, int64_t n_off, int64_t n_cols,
              const int32_t *__restrict__ d_rp, const int32_t *__restrict__ d_ci,
              const T *__restrict__ d_v, const int32_t *__restrict__ n_rp,
              const int32_t *__restrict__ n_ci, const T *__restrict__ n_v,
              const int32_t *__restrict__ p_rp, const int32_t *__restrict__ p_ci,
              const T *__restrict__ p_v, const T *__restrict__ x, T *__restrict__ y, T alpha,
              T beta, int base) {
    const int64_t rows = T_periods * n_diag + (T_periods - 1) * n_off;
    const int64_t r = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (r >= rows) return;
    const int64_t period = n_diag + n_off;
    const int64_t t = r / period, rem = r - t * period;
    T acc = T(0);
    if (rem < n_diag) {
        acc = walk<T>(rem, d_rp, d_ci, d_v, x, t * n_cols, n_cols, base, acc);
    } else {
        acc = walk<T>(rem - n_diag, n_rp, n_ci, n_v, x, t * n_cols, n_cols, base, acc);
        acc = walk<T>(rem - n_diag, p_rp, p_ci, p_v, x, (t + 1) * n_cols, n_cols, base, acc);
    }
    T out = mul_rn(alpha, acc);
    if (kBeta) out = add_rn(out, mul_rn(beta, y[r]));
    y[r] = out;
}

template <typename T>
int launch(cudaStream_t st, int base, int64_t Tp, int64_t n_diag, int64_t n_off, int64_t n_cols,
           const int32_t *d_rp, const int32_t *d_ci, const void *d_v, const int32_t *n_rp,
           const int32_t *n_ci, const void *n_v, const int32_t *p_rp, const int32_t *p_ci,
           const void *p_v, const void *x, void *y, double alpha, double beta) {
    const int64_t rows = Tp * n_diag + (Tp - 1) * n_off;
    if (rows == 0) return ok();
    const unsigned grid = (unsigned)ceil_div(rows, kThreads);
    const T a = (T)alpha, b = (T)beta;
    if (b == T(0))
        periodic_rows<T, false><<<grid, kThreads, 0, st>>>(
            Tp, n_diag, n_off, n_cols, d_rp, d_ci, (const T *)d_v, n_rp, n_ci, (const T *)n_v,
            p_rp, p_ci, (const T *)p_v, (const T *)x, (T *)y, a, b, base);
    else
        periodic_rows<T, true><<<grid, kThreads, 0, st>>>(
            Tp, n_diag, n_off, n_cols, d_rp, d_ci, (const T *)d_v, n_rp, n_ci, (const T *)n_v,
            p_rp, p_ci, (const T *)p_v, (const T *)x, (T *)y, a, b, base);
    JLB_LAUNCH_CHECK("periodic_rows");
    return ok();
}

}  // namespace bbm
}  // namespace jlb

using namespace jlb;

extern "C" JLB_API int jlb_bbm_periodic_spmv(void *stream, int dtype, int idx_base, int64_t T,
                                             int64_t n_diag, int64_t n_off, int64_t n_cols,
                                             const int32_t *diag_rowptr,
                                             const int32_t *diag_colind, const void *diag_val,
                                             const int32_t *neg_rowptr, const int32_t *neg_colind,
                                             const void *neg_val, const int32_t *pos_rowptr,
                                             const int32_t *pos_colind, const void *pos_val,
                                             const void *x, void *y, double alpha, double beta) {
    if (dtype != JLB_F32 && dtype != JLB_F64)
        return fail(JLB_ERR_UNSUPPORTED_VALUE_TYPE, "periodic SpMV supports Float32 and Float64");
    if (idx_base != 0 && idx_base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (T < 1 || n_diag < 0 || n_off < 0 || n_cols < 0)
        return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "need T >= 1 and non-negative block sizes");
    if (!x || !y || !diag_rowptr || (n_off > 0 && T > 1 && (!neg_rowptr || !pos_rowptr)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    if (dtype == JLB_F64)
        return bbm::launch<double>(as_stream(stream), idx_base, T, n_diag, n_off, n_cols,
                                   diag_rowptr, diag_colind, diag_val, neg_rowptr, neg_colind,
                                   neg_val, pos_rowptr, pos_colind, pos_val, x, y, alpha, beta);
    return bbm::launch<float>(as_stream(stream), idx_base, T, n_diag, n_off, n_cols, diag_rowptr,
                              diag_colind, diag_val, neg_rowptr, neg_colind, neg_val, pos_rowptr,
                              pos_colind, pos_val, x, y, alpha, beta);
}
