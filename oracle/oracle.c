/*
 * oracle.c -- CPU restatement of JLUST's CPU semantics for the sparse hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links or calls this
 * file; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * it (through oracle/oracle.py) as the checker or as the timed CPU baseline.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).  -ffp-contract=off
 * matters: Julia never contracts `acc += a*b` into an FMA unless asked to, so the
 * restatement must round the product and the sum separately to reproduce the
 * reference's values bit for bit.
 *
 * Reference semantics followed (paths inside the JLUST project):
 *   SpMV   ext/KernelAbstractionsExt/ops/_walker.jl:111-146 (inner compressed
 *          walk, k ascending) + ops/spmv.jl:154 (leaf `_acc += nz*x`) and
 *          ops/spmv.jl:161-178 (row write `alpha*acc (+ beta*y)`, zero-beta
 *          specialisation skips the y read).
 *   SpMM   ext/KernelAbstractionsExt/ops/spmm.jl:272-292 (Tiled strategy chosen
 *          for k=64 at :347): per (row, col) the sum runs over k in storage
 *          order; C = alpha*acc + beta*C.
 *   SDDMM  ext/KernelAbstractionsExt/ops/sddmm.jl:23-36: dot over k = 1..K in
 *          order, nz = alpha*dot + beta*nz.
 *   Block SpMM  src/block_sparse.jl:177-188 + :231-246: Y zero-filled, then for
 *          every block (block columns ascending), row, stored entry (columns
 *          ascending) and output column t, Y[row,t] += v * X[col,t].
 *   CSR/COO -> BSR  src/convert.jl:302-388 (decompose in storage order, drop
 *          explicit zeros at :316, dim2lvl, stable lexsort at :343/:419-424,
 *          two-pass compose at :271-292) with the level extents of
 *          dim2lvl(...; as_size=true) (src/formats.jl:204-220,429-431): the
 *          block-row level has ceil(m/b1) entries, the in-block levels b1, b2.
 *   Scans  src/convert.jl:154-168 (position buffer = running count, first
 *          entry = origin).
 *
 * Semantics chosen where the reference is silent or inconsistent:
 *   - beta == 0 never reads the output (BLAS / cuSPARSE convention; the
 *     reference's Tiled SpMM and SDDMM bodies multiply the old value by 0).
 *   - duplicate COO coordinates: the composer keeps the first value of a run of
 *     equal level coordinates after a stable sort (src/convert.jl:231-238 +
 *     :222), i.e. the nonzero entry with the lowest storage index wins.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <omp.h>

#define OR_EXPORT __attribute__((visibility("default")))

/* dtype codes shared with include/jlust_b200.h */
enum { OR_F32 = 0, OR_F64 = 1, OR_BF16 = 2 };

OR_EXPORT int or_max_threads(void) { return omp_get_max_threads(); }
OR_EXPORT void or_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* ------------------------------------------------------------------------- */
/* CSR SpMV, value type T, reference order.                                   */
/* ------------------------------------------------------------------------- */

#define DEFINE_SPMV(NAME, T)                                                    \
OR_EXPORT void NAME(int64_t m, const int32_t *rowptr, const int32_t *colind,    \
                    const T *val, const T *x, T *y, double alpha_d,             \
                    double beta_d, int base) {                                  \
    const T alpha = (T)alpha_d, beta = (T)beta_d;                               \
    const int zero_beta = (beta == (T)0);                                       \
    _Pragma("omp parallel for schedule(static, 4096)")                          \
    for (int64_t r = 0; r < m; ++r) {                                           \
        T acc = (T)0;                                                           \
        const int64_t lo = (int64_t)rowptr[r] - base;                           \
        const int64_t hi = (int64_t)rowptr[r + 1] - base;                       \
        for (int64_t k = lo; k < hi; ++k) {                                     \
            T prod = val[k] * x[(int64_t)colind[k] - base];                     \
            acc = acc + prod;                                                   \
        }                                                                       \
        T out = alpha * acc;                                                    \
        if (!zero_beta) { T by = beta * y[r]; out = out + by; }                 \
        y[r] = out;                                                             \
    }                                                                           \
}

DEFINE_SPMV(or_csr_spmv_f64, double)
DEFINE_SPMV(or_csr_spmv_f32, float)

/* DCSR SpMV: JLUST's DCSR walk (ext/KernelAbstractionsExt/ops/_walker.jl:
 * 323-342, dispatched from ops/spmv.jl:371-504).  Stored row f is row
 * row_ids[f]; its entries fibptr[f] .. fibptr[f+1]-1 are summed in storage
 * order as a CSR row is; rows that are not stored are not written. */
#define DEFINE_DCSR_SPMV(NAME, T)                                               \
OR_EXPORT void NAME(int64_t nfib, const int32_t *fibptr, const int32_t *row_ids, \
                    const int32_t *colind, const T *val, const T *x, T *y,      \
                    double alpha_d, double beta_d, int base) {                  \
    const T alpha = (T)alpha_d, beta = (T)beta_d;                               \
    const int zero_beta = (beta == (T)0);                                       \
    for (int64_t f = 0; f < nfib; ++f) {                                        \
        const int64_t r = (int64_t)row_ids[f] - base;                           \
        T acc = (T)0;                                                           \
        for (int64_t k = (int64_t)fibptr[f] - base; k < (int64_t)fibptr[f + 1] - base; ++k) { \
            T prod = val[k] * x[(int64_t)colind[k] - base];                     \
            acc = acc + prod;                                                   \
        }                                                                       \
        T out = alpha * acc;                                                    \
        if (!zero_beta) { T by = beta * y[r]; out = out + by; }                 \
        y[r] = out;                                                             \
    }                                                                           \
}

DEFINE_DCSR_SPMV(or_dcsr_spmv_f64, double)
DEFINE_DCSR_SPMV(or_dcsr_spmv_f32, float)

/* COO and CSC SpMV: JLUST's COO and scatter paths (ops/spmv.jl:386-420):
 * y scaled by beta (set to 0 when beta is 0), then every entry, in storage
 * order here, adds (alpha * v) * x[col] to its row.  The reference and the
 * GPU add the same terms in an order that is not fixed (atomics). */
#define DEFINE_ENTRY_SPMV(NAME, T)                                              \
OR_EXPORT void NAME(int64_t m, int64_t n, int64_t nnz, const int32_t *rows,     \
                    const int32_t *cols, const int32_t *colptr, const T *val,   \
                    const T *x, T *y, double alpha_d, double beta_d, int base) { \
    const T alpha = (T)alpha_d, beta = (T)beta_d;                               \
    for (int64_t r = 0; r < m; ++r) y[r] = (beta == (T)0) ? (T)0 : beta * y[r]; \
    if (colptr) {                                                               \
        for (int64_t j = 0; j < n; ++j)                                         \
            for (int64_t p = (int64_t)colptr[j] - base; p < (int64_t)colptr[j + 1] - base; ++p) { \
                T t = alpha * val[p];                                           \
                y[(int64_t)rows[p] - base] += t * x[j];                         \
            }                                                                   \
    } else {                                                                    \
        for (int64_t p = 0; p < nnz; ++p) {                                     \
            T t = alpha * val[p];                                               \
            y[(int64_t)rows[p] - base] += t * x[(int64_t)cols[p] - base];       \
        }                                                                       \
    }                                                                           \
}

DEFINE_ENTRY_SPMV(or_entry_spmv_f64, double)
DEFINE_ENTRY_SPMV(or_entry_spmv_f32, float)

/* Periodic block-banded SpMV: JLUST's fused periodic kernel
 * (ext/KernelAbstractionsExt/ops/block_periodic.jl:114-163).  Row r of
 * T*n_diag + (T-1)*n_off: period t = r / (n_diag + n_off); a diagonal row sums
 * D's row with columns shifted by t*n_cols, then adds the sum of its selector
 * patches (npatch of them: rows prows[2p]..prows[2p+1] inclusive, value
 * pvals[p] times x[t*n_cols + r - prows[2p] + pcols[p]], summed from zero in
 * patch order, _apply_patches at :39-49); a coupling row sums neg's row (shift
 * t*n_cols) then pos's row (shift (t+1)*n_cols) into the same sum.  A coupling
 * block whose rowptr is NULL is a ShiftedDiag selector: its row adds
 * sel * x[off + row + shift]. */
#define DEFINE_BBM_PERIODIC(NAME, T)                                            \
OR_EXPORT void NAME(int64_t Tp, int64_t n_diag, int64_t n_off, int64_t n_cols,  \
                    const int32_t *drp, const int32_t *dci, const T *dv,        \
                    int64_t npatch, const int64_t *prows, const int64_t *pcols, \
                    const double *pvals,                                        \
                    const int32_t *nrp, const int32_t *nci, const T *nv,        \
                    int64_t nshift, double nsel,                                \
                    const int32_t *prp, const int32_t *pci, const T *pv,        \
                    int64_t pshift, double psel,                                \
                    const T *x, T *y, double alpha_d, double beta_d, int base) { \
    const T alpha = (T)alpha_d, beta = (T)beta_d;                               \
    const int64_t rows = Tp * n_diag + (Tp - 1) * n_off;                        \
    for (int64_t r = 0; r < rows; ++r) {                                        \
        const int64_t t = r / (n_diag + n_off);                                 \
        int64_t rem = r - t * (n_diag + n_off);                                 \
        T acc = (T)0;                                                           \
        const int32_t *rp[2], *ci[2]; const T *v[2]; int64_t off[2], sh[2];     \
        double sel[2]; int nb;                                                  \
        if (rem < n_diag) { rp[0] = drp; ci[0] = dci; v[0] = dv; off[0] = t * n_cols; nb = 1; } \
        else { rem -= n_diag; rp[0] = nrp; ci[0] = nci; v[0] = nv; off[0] = t * n_cols;        \
               sh[0] = nshift; sel[0] = nsel;                                   \
               rp[1] = prp; ci[1] = pci; v[1] = pv; off[1] = (t + 1) * n_cols; nb = 2;          \
               sh[1] = pshift; sel[1] = psel; }                                 \
        for (int b = 0; b < nb; ++b) {                                          \
            if (!rp[b]) {                                                       \
                T prod = (T)sel[b] * x[off[b] + rem + sh[b]];                   \
                acc = acc + prod;                                               \
                continue;                                                       \
            }                                                                   \
            for (int64_t k = (int64_t)rp[b][rem] - base; k < (int64_t)rp[b][rem + 1] - base; ++k) { \
                T prod = v[b][k] * x[off[b] + (int64_t)ci[b][k] - base];        \
                acc = acc + prod;                                               \
            }                                                                   \
        }                                                                       \
        if (nb == 1) {                                                          \
            T pacc = (T)0;                                                      \
            for (int64_t p = 0; p < npatch; ++p)                                \
                if (rem >= prows[2 * p] && rem <= prows[2 * p + 1]) {           \
                    T prod = (T)pvals[p] * x[off[0] + rem - prows[2 * p] + pcols[p]]; \
                    pacc = pacc + prod;                                         \
                }                                                               \
            acc = acc + pacc;                                                   \
        }                                                                       \
        T out = alpha * acc;                                                    \
        if (beta != (T)0) { T by = beta * y[r]; out = out + by; }               \
        y[r] = out;                                                             \
    }                                                                           \
}

DEFINE_BBM_PERIODIC(or_bbm_periodic_spmv_f64, double)
DEFINE_BBM_PERIODIC(or_bbm_periodic_spmv_f32, float)

/* SpGEMM C = alpha*A*B (A m x k, B k x n CSR, one origin): JLUST's
 * scatter-sort-reduce order (ext/KernelAbstractionsExt/ops/spgemm.jl:40-80,
 * 330-400).  Row i's products A[i,j]*B[j,c] in the order of its A entries,
 * then of B row j's entries, each times alpha unless alpha == 1; sorted by
 * (column, product order) -- the reference's stable sort of (row, column)
 * keys; every run of equal columns is one entry of C, its products summed
 * from zero left to right (the reference adds them by atomics, in an order
 * this fixes).  With crp == NULL only nnz(C) is returned. */
typedef struct { int32_t col; int64_t ord; } or_prod_key;
static int or_prod_cmp(const void *a, const void *b) {
    const or_prod_key *x = (const or_prod_key *)a, *y = (const or_prod_key *)b;
    if (x->col != y->col) return x->col < y->col ? -1 : 1;
    return x->ord < y->ord ? -1 : (x->ord > y->ord);
}

#define DEFINE_SPGEMM(NAME, T)                                                  \
OR_EXPORT int64_t NAME(int64_t m, const int32_t *arp, const int32_t *aci,       \
                       const T *av, const int32_t *brp, const int32_t *bci,     \
                       const T *bv, double alpha_d, int base, int32_t *crp,     \
                       int32_t *cci, T *cv) {                                   \
    const T alpha = (T)alpha_d;                                                 \
    int64_t maxp = 0;                                                           \
    for (int64_t i = 0; i < m; ++i) {                                           \
        int64_t c = 0;                                                          \
        for (int64_t p = arp[i] - base; p < arp[i + 1] - base; ++p) {           \
            const int64_t j = aci[p] - base;                                    \
            c += brp[j + 1] - brp[j];                                           \
        }                                                                       \
        if (c > maxp) maxp = c;                                                 \
    }                                                                           \
    or_prod_key *key = (or_prod_key *)malloc(sizeof(or_prod_key) * (maxp ? maxp : 1)); \
    T *pv = (T *)malloc(sizeof(T) * (maxp ? maxp : 1));                         \
    int64_t nnz = 0;                                                            \
    if (crp) crp[0] = base;                                                     \
    for (int64_t i = 0; i < m; ++i) {                                           \
        int64_t np = 0;                                                         \
        for (int64_t p = arp[i] - base; p < arp[i + 1] - base; ++p) {           \
            const int64_t j = aci[p] - base;                                    \
            for (int64_t q = brp[j] - base; q < brp[j + 1] - base; ++q) {       \
                T t = av[p] * bv[q];                                            \
                if (alpha != (T)1) t = t * alpha;                               \
                key[np].col = bci[q] - base; key[np].ord = np; pv[np] = t; ++np; \
            }                                                                   \
        }                                                                       \
        qsort(key, (size_t)np, sizeof(or_prod_key), or_prod_cmp);               \
        for (int64_t s = 0; s < np;) {                                          \
            int64_t e = s;                                                      \
            T acc = (T)0;                                                       \
            while (e < np && key[e].col == key[s].col) { acc = acc + pv[key[e].ord]; ++e; } \
            if (crp) { cci[nnz] = key[s].col + base; cv[nnz] = acc; }           \
            ++nnz;                                                              \
            s = e;                                                              \
        }                                                                       \
        if (crp) crp[i + 1] = (int32_t)(nnz + base);                            \
    }                                                                           \
    free(key);                                                                  \
    free(pv);                                                                   \
    return nnz;                                                                 \
}

DEFINE_SPGEMM(or_spgemm_f64, double)
DEFINE_SPGEMM(or_spgemm_f32, float)

/* fp64 reference of the same product plus the per-row magnitude bound
 * sum_k |v_k * x_k|, used for tolerance checks of any value type. */
OR_EXPORT void or_csr_spmv_ref64(int dtype, int64_t m, const int32_t *rowptr,
                                 const int32_t *colind, const void *val,
                                 const void *x, const void *y_in, double *y_out,
                                 double *bound, double alpha, double beta,
                                 int base) {
    #pragma omp parallel for schedule(static, 4096)
    for (int64_t r = 0; r < m; ++r) {
        double acc = 0.0, mag = 0.0;
        const int64_t lo = (int64_t)rowptr[r] - base;
        const int64_t hi = (int64_t)rowptr[r + 1] - base;
        for (int64_t k = lo; k < hi; ++k) {
            const int64_t c = (int64_t)colind[k] - base;
            double v, xv;
            if (dtype == OR_F64) { v = ((const double *)val)[k]; xv = ((const double *)x)[c]; }
            else if (dtype == OR_F32) { v = ((const float *)val)[k]; xv = ((const float *)x)[c]; }
            else { v = bf16_to_f32(((const uint16_t *)val)[k]); xv = bf16_to_f32(((const uint16_t *)x)[c]); }
            acc += v * xv;
            mag += fabs(v * xv);
        }
        double yo = 0.0;
        if (beta != 0.0 && y_in) {
            if (dtype == OR_F64) yo = ((const double *)y_in)[r];
            else if (dtype == OR_F32) yo = ((const float *)y_in)[r];
            else yo = bf16_to_f32(((const uint16_t *)y_in)[r]);
        }
        y_out[r] = alpha * acc + beta * yo;
        if (bound) bound[r] = fabs(alpha) * mag + fabs(beta * yo);
    }
}

/* ------------------------------------------------------------------------- */
/* Dense operand addressing: order 0 = row-major (element (i,j) at i*ld + j),  */
/* order 1 = column-major (element (i,j) at i + j*ld).                         */
/* ------------------------------------------------------------------------- */
static inline int64_t didx(int order, int64_t ld, int64_t i, int64_t j) {
    return order == 0 ? i * ld + j : i + j * ld;
}

/* CSR SpMM  C = alpha*A*B + beta*C  (A m x n CSR, B n x k, C m x k), Tiled order:
 * per (row, col) the k-loop runs over the row's entries in storage order. */
#define DEFINE_SPMM(NAME, T)                                                    \
OR_EXPORT void NAME(int64_t m, int64_t k, const int32_t *rowptr,                \
                    const int32_t *colind, const T *val, const T *B,            \
                    int64_t ldb, int b_order, T *C, int64_t ldc, int c_order,   \
                    double alpha_d, double beta_d, int base) {                  \
    const T alpha = (T)alpha_d, beta = (T)beta_d;                               \
    const int zero_beta = (beta == (T)0);                                       \
    _Pragma("omp parallel for schedule(dynamic, 256)")                          \
    for (int64_t r = 0; r < m; ++r) {                                           \
        const int64_t lo = (int64_t)rowptr[r] - base;                           \
        const int64_t hi = (int64_t)rowptr[r + 1] - base;                       \
        for (int64_t t = 0; t < k; ++t) {                                       \
            T acc = (T)0;                                                       \
            for (int64_t p = lo; p < hi; ++p) {                                 \
                const int64_t c = (int64_t)colind[p] - base;                    \
                T prod = val[p] * B[didx(b_order, ldb, c, t)];                  \
                acc = acc + prod;                                               \
            }                                                                   \
            const int64_t ci = didx(c_order, ldc, r, t);                        \
            T out = alpha * acc;                                                \
            if (!zero_beta) { T bc = beta * C[ci]; out = out + bc; }            \
            C[ci] = out;                                                        \
        }                                                                       \
    }                                                                           \
}

DEFINE_SPMM(or_csr_spmm_f32, float)
DEFINE_SPMM(or_csr_spmm_f64, double)

/* fp64 SpMM reference + magnitude bound (fp32 inputs). */
OR_EXPORT void or_csr_spmm_ref64_f32(int64_t m, int64_t k, const int32_t *rowptr,
                                     const int32_t *colind, const float *val,
                                     const float *B, int64_t ldb, int b_order,
                                     const float *C_in, int64_t ldc_in, int c_order_in,
                                     double *C_out, double *bound,
                                     double alpha, double beta, int base) {
    #pragma omp parallel for schedule(dynamic, 256)
    for (int64_t r = 0; r < m; ++r) {
        const int64_t lo = (int64_t)rowptr[r] - base;
        const int64_t hi = (int64_t)rowptr[r + 1] - base;
        for (int64_t t = 0; t < k; ++t) {
            double acc = 0.0, mag = 0.0;
            for (int64_t p = lo; p < hi; ++p) {
                const int64_t c = (int64_t)colind[p] - base;
                double pr = (double)val[p] * (double)B[didx(b_order, ldb, c, t)];
                acc += pr; mag += fabs(pr);
            }
            double co = 0.0;
            if (beta != 0.0 && C_in) co = C_in[didx(c_order_in, ldc_in, r, t)];
            C_out[r * k + t] = alpha * acc + beta * co;
            if (bound) bound[r * k + t] = fabs(alpha) * mag + fabs(beta * co);
        }
    }
}

/* ------------------------------------------------------------------------- */
/* SDDMM over a CSR pattern (m x n).  A is m x K, B is K x n (element (kk, j)).*/
/*   mode 0 (reference, sddmm.jl:23-36): out[p] = alpha*dot + beta*out[p]      */
/*   mode 1 (sampled product):           out[p] = (alpha*dot)*S[p] + beta*out[p]*/
/* dot = sum_{kk=0}^{K-1} A[i,kk]*B[kk,j] in order.  beta == 0 skips the read. */
/* ------------------------------------------------------------------------- */
#define DEFINE_SDDMM(NAME, T)                                                   \
OR_EXPORT void NAME(int64_t m, int64_t K, const int32_t *rowptr,                \
                    const int32_t *colind, const T *A, int64_t lda,             \
                    int a_order, const T *B, int64_t ldb, int b_order,          \
                    const T *S, T *out, int mode, double alpha_d,               \
                    double beta_d, int base) {                                  \
    const T alpha = (T)alpha_d, beta = (T)beta_d;                               \
    const int zero_beta = (beta == (T)0);                                       \
    _Pragma("omp parallel for schedule(dynamic, 256)")                          \
    for (int64_t i = 0; i < m; ++i) {                                           \
        const int64_t lo = (int64_t)rowptr[i] - base;                           \
        const int64_t hi = (int64_t)rowptr[i + 1] - base;                       \
        for (int64_t p = lo; p < hi; ++p) {                                     \
            const int64_t j = (int64_t)colind[p] - base;                        \
            T dot = (T)0;                                                       \
            for (int64_t kk = 0; kk < K; ++kk) {                                \
                T prod = A[didx(a_order, lda, i, kk)] * B[didx(b_order, ldb, kk, j)]; \
                dot = dot + prod;                                               \
            }                                                                   \
            T o = alpha * dot;                                                  \
            if (mode == 1) o = o * S[p];                                        \
            if (!zero_beta) { T bo = beta * out[p]; o = o + bo; }               \
            out[p] = o;                                                         \
        }                                                                       \
    }                                                                           \
}

DEFINE_SDDMM(or_sddmm_f32, float)
DEFINE_SDDMM(or_sddmm_f64, double)

/* fp64 SDDMM reference + bound (fp32 inputs). */
OR_EXPORT void or_sddmm_ref64_f32(int64_t m, int64_t K, const int32_t *rowptr,
                                  const int32_t *colind, const float *A, int64_t lda,
                                  int a_order, const float *B, int64_t ldb, int b_order,
                                  const float *S, const float *out_in, double *out,
                                  double *bound, int mode, double alpha, double beta,
                                  int base) {
    #pragma omp parallel for schedule(dynamic, 256)
    for (int64_t i = 0; i < m; ++i) {
        const int64_t lo = (int64_t)rowptr[i] - base;
        const int64_t hi = (int64_t)rowptr[i + 1] - base;
        for (int64_t p = lo; p < hi; ++p) {
            const int64_t j = (int64_t)colind[p] - base;
            double dot = 0.0, mag = 0.0;
            for (int64_t kk = 0; kk < K; ++kk) {
                double pr = (double)A[didx(a_order, lda, i, kk)] *
                            (double)B[didx(b_order, ldb, kk, j)];
                dot += pr; mag += fabs(pr);
            }
            double s = (mode == 1) ? (double)S[p] : 1.0;
            double oin = (beta != 0.0 && out_in) ? (double)out_in[p] : 0.0;
            out[p] = alpha * dot * s + beta * oin;
            if (bound) bound[p] = fabs(alpha * s) * mag + fabs(beta * oin);
        }
    }
}

/* ------------------------------------------------------------------------- */
/* Block SpMM on a BSR matrix (row-major b1 x b2 blocks, BSRRight), bf16 values */
/* and bf16 X, fp32 accumulation in the reference's fused-loop order:          */
/* per output element, block columns ascending, then in-block columns.         */
/*   Y[I*b1 + r, t] = alpha * sum + beta * Y   (beta == 0 skips the read)      */
/* X is (nb*b2) x N row-major with leading dimension ldx; Y is (mb*b1) x N.    */
/* ------------------------------------------------------------------------- */
OR_EXPORT void or_bsr_spmm_bf16(int64_t mb, int64_t N, int b1, int b2,
                                const int32_t *browptr, const int32_t *bcolind,
                                const uint16_t *bval, const uint16_t *X, int64_t ldx,
                                float *Y, int64_t ldy, double alpha_d, double beta_d,
                                int base) {
    const float alpha = (float)alpha_d, beta = (float)beta_d;
    #pragma omp parallel
    {
        float *acc = (float *)malloc(sizeof(float) * (size_t)b1 * (size_t)N);
        float *xrow = (float *)malloc(sizeof(float) * (size_t)N);
        #pragma omp for schedule(dynamic, 1)
        for (int64_t I = 0; I < mb; ++I) {
            memset(acc, 0, sizeof(float) * (size_t)b1 * (size_t)N);
            const int64_t qlo = (int64_t)browptr[I] - base, qhi = (int64_t)browptr[I + 1] - base;
            for (int64_t q = qlo; q < qhi; ++q) {
                const int64_t J = (int64_t)bcolind[q] - base;
                const uint16_t *blk = bval + q * (int64_t)b1 * b2;
                for (int r = 0; r < b1; ++r) {
                    float *a = acc + (size_t)r * N;
                    for (int c = 0; c < b2; ++c) {
                        const float v = bf16_to_f32(blk[r * b2 + c]);
                        const uint16_t *xr = X + (J * b2 + c) * ldx;
                        for (int64_t t = 0; t < N; ++t) xrow[t] = bf16_to_f32(xr[t]);
                        for (int64_t t = 0; t < N; ++t) { float pr = v * xrow[t]; a[t] = a[t] + pr; }
                    }
                }
            }
            for (int r = 0; r < b1; ++r) {
                float *yr = Y + (I * b1 + r) * ldy;
                for (int64_t t = 0; t < N; ++t) {
                    float o = alpha * acc[(size_t)r * N + t];
                    if (beta != 0.0f) { float by = beta * yr[t]; o = o + by; }
                    yr[t] = o;
                }
            }
        }
        free(acc); free(xrow);
    }
}

/* fp64 reference + magnitude bound of the same block product (Y_in read only if beta != 0). */
OR_EXPORT void or_bsr_spmm_ref64_bf16(int64_t mb, int64_t N, int b1, int b2,
                                      const int32_t *browptr, const int32_t *bcolind,
                                      const uint16_t *bval, const uint16_t *X, int64_t ldx,
                                      const float *Y_in, int64_t ldy_in, double *Y, double *bound,
                                      double alpha, double beta, int base) {
    #pragma omp parallel
    {
        double *acc = (double *)malloc(sizeof(double) * (size_t)b1 * (size_t)N);
        double *mag = (double *)malloc(sizeof(double) * (size_t)b1 * (size_t)N);
        #pragma omp for schedule(dynamic, 1)
        for (int64_t I = 0; I < mb; ++I) {
            memset(acc, 0, sizeof(double) * (size_t)b1 * (size_t)N);
            memset(mag, 0, sizeof(double) * (size_t)b1 * (size_t)N);
            const int64_t qlo = (int64_t)browptr[I] - base, qhi = (int64_t)browptr[I + 1] - base;
            for (int64_t q = qlo; q < qhi; ++q) {
                const int64_t J = (int64_t)bcolind[q] - base;
                const uint16_t *blk = bval + q * (int64_t)b1 * b2;
                for (int r = 0; r < b1; ++r)
                    for (int c = 0; c < b2; ++c) {
                        const double v = bf16_to_f32(blk[r * b2 + c]);
                        const uint16_t *xr = X + (J * b2 + c) * ldx;
                        for (int64_t t = 0; t < N; ++t) {
                            double pr = v * (double)bf16_to_f32(xr[t]);
                            acc[(size_t)r * N + t] += pr;
                            mag[(size_t)r * N + t] += fabs(pr);
                        }
                    }
            }
            for (int r = 0; r < b1; ++r)
                for (int64_t t = 0; t < N; ++t) {
                    double yin = (beta != 0.0 && Y_in) ? (double)Y_in[(I * b1 + r) * ldy_in + t] : 0.0;
                    Y[(I * b1 + r) * N + t] = alpha * acc[(size_t)r * N + t] + beta * yin;
                    if (bound) bound[(I * b1 + r) * N + t] = fabs(alpha) * mag[(size_t)r * N + t] + fabs(beta * yin);
                }
        }
        free(acc); free(mag);
    }
}

/* ------------------------------------------------------------------------- */
/* Exclusive scan of counts into a position buffer: out[0] = base,            */
/* out[i+1] = out[i] + counts[i].  Returns the total, or -1 on int32 overflow. */
/* ------------------------------------------------------------------------- */
OR_EXPORT int64_t or_exclusive_scan_i32(int64_t n, const int32_t *counts, int32_t *out, int base) {
    int64_t run = base;
    out[0] = (int32_t)run;
    for (int64_t i = 0; i < n; ++i) {
        run += counts[i];
        if (run > INT32_MAX) return -1;
        out[i + 1] = (int32_t)run;
    }
    return run - base;
}

/* ------------------------------------------------------------------------- */
/* CSR / COO -> BSRRight((b1, b2)) conversion (src/convert.jl:302-388).         */
/*                                                                            */
/* 1. Decompose in storage order, dropping explicit zeros (convert.jl:316).   */
/* 2. dim2lvl: (i, j) -> (i / b1, j / b2, i % b1, j % b2) (formats.jl:429).   */
/* 3. Stable lexicographic sort of the level coordinates (convert.jl:343).    */
/* 4. Compose: level 1 dense over ceil(m/b1) block rows, level 2 compressed    */
/*    (block row pointer + sorted distinct block columns), levels 3-4 dense    */
/*    b1 x b2 tiles filled with zeros where no entry lands.  Within a run of   */
/*    equal coordinates the first value is kept (convert.jl:231-238, :222).    */
/* 5. Position and coordinate buffers shifted by the source origin            */
/*    (convert.jl:365-376).                                                    */
/*                                                                            */
/* Two-phase like the composer: call with browptr/bcolind/bval == NULL to get */
/* nnzb; call again with buffers of ceil(m/b1)+1, nnzb and nnzb*b1*b2.        */
/* ------------------------------------------------------------------------- */
typedef struct { uint64_t blk; uint32_t cell; int64_t p; } or_entry;

static int or_entry_cmp(const void *a, const void *b) {
    const or_entry *x = (const or_entry *)a, *y = (const or_entry *)b;
    if (x->blk != y->blk) return x->blk < y->blk ? -1 : 1;
    if (x->cell != y->cell) return x->cell < y->cell ? -1 : 1;
    if (x->p != y->p) return x->p < y->p ? -1 : 1;
    return 0;
}

static int or_is_zero(const void *val, int dtype, int64_t p) {
    if (dtype == OR_F64) return ((const double *)val)[p] == 0.0;
    if (dtype == OR_F32) return ((const float *)val)[p] == 0.0f;
    return (((const uint16_t *)val)[p] & 0x7fffu) == 0;
}

static int or_esize(int dtype) { return dtype == OR_F64 ? 8 : dtype == OR_F32 ? 4 : 2; }

/* rows[p] may be NULL when rowptr is given (CSR); exactly one of them is used. */
static int64_t or_to_bsr(int64_t m, int64_t n, int64_t nnz, int b1, int b2,
                         const int32_t *rowptr, const int32_t *rows, const int32_t *cols,
                         const void *val, int dtype, int base,
                         int32_t *browptr, int32_t *bcolind, void *bval) {
    const int64_t mb = (m + b1 - 1) / b1, nb = (n + b2 - 1) / b2;
    or_entry *e = (or_entry *)malloc(sizeof(or_entry) * (size_t)(nnz > 0 ? nnz : 1));
    int64_t ne = 0;
    if (rowptr) {
        for (int64_t i = 0; i < m; ++i)
            for (int64_t p = (int64_t)rowptr[i] - base; p < (int64_t)rowptr[i + 1] - base; ++p) {
                if (or_is_zero(val, dtype, p)) continue;
                const int64_t j = (int64_t)cols[p] - base;
                e[ne].blk = (uint64_t)(i / b1) * (uint64_t)nb + (uint64_t)(j / b2);
                e[ne].cell = (uint32_t)((i % b1) * b2 + (j % b2));
                e[ne].p = p; ++ne;
            }
    } else {
        for (int64_t p = 0; p < nnz; ++p) {
            if (or_is_zero(val, dtype, p)) continue;
            const int64_t i = (int64_t)rows[p] - base, j = (int64_t)cols[p] - base;
            e[ne].blk = (uint64_t)(i / b1) * (uint64_t)nb + (uint64_t)(j / b2);
            e[ne].cell = (uint32_t)((i % b1) * b2 + (j % b2));
            e[ne].p = p; ++ne;
        }
    }
    qsort(e, (size_t)ne, sizeof(or_entry), or_entry_cmp);
    int64_t nnzb = 0;
    for (int64_t t = 0; t < ne; ++t)
        if (t == 0 || e[t].blk != e[t - 1].blk) ++nnzb;
    if (browptr && bcolind && bval) {
        const int es = or_esize(dtype);
        const int64_t bsz = (int64_t)b1 * b2;
        memset(bval, 0, (size_t)(nnzb * bsz * es));
        int32_t *cnt = (int32_t *)calloc((size_t)(mb > 0 ? mb : 1), sizeof(int32_t));
        int64_t q = -1;
        for (int64_t t = 0; t < ne; ++t) {
            if (t == 0 || e[t].blk != e[t - 1].blk) {
                ++q;
                bcolind[q] = (int32_t)(e[t].blk % (uint64_t)nb) + base;
                cnt[e[t].blk / (uint64_t)nb] += 1;
            }
            if (t > 0 && e[t].blk == e[t - 1].blk && e[t].cell == e[t - 1].cell) continue;
            memcpy((char *)bval + (q * bsz + e[t].cell) * es,
                   (const char *)val + e[t].p * es, (size_t)es);
        }
        or_exclusive_scan_i32(mb, cnt, browptr, base);
        free(cnt);
    }
    free(e);
    return nnzb;
}

OR_EXPORT int64_t or_csr_to_bsr(int64_t m, int64_t n, int b1, int b2, const int32_t *rowptr,
                                const int32_t *colind, const void *val, int dtype, int base,
                                int32_t *browptr, int32_t *bcolind, void *bval) {
    const int64_t nnz = m > 0 ? (int64_t)rowptr[m] - base : 0;
    return or_to_bsr(m, n, nnz, b1, b2, rowptr, NULL, colind, val, dtype, base,
                     browptr, bcolind, bval);
}

OR_EXPORT int64_t or_coo_to_bsr(int64_t m, int64_t n, int64_t nnz, int b1, int b2,
                                const int32_t *rows, const int32_t *cols, const void *val,
                                int dtype, int base, int32_t *browptr, int32_t *bcolind,
                                void *bval) {
    return or_to_bsr(m, n, nnz, b1, b2, NULL, rows, cols, val, dtype, base,
                     browptr, bcolind, bval);
}
