// spmv_formats.cu -- SpMV for COO and CSC inputs on sm_100a.
//
// JLUST runs these without converting them: y is first scaled by beta (set to
// zero when beta is 0), then every stored entry adds alpha*v*x[col] into its
// row with an atomic add (ext/KernelAbstractionsExt/ops/spmv.jl:386-420; the
// COO walk with its segmented warp reduction, ops/_walker.jl:343-375).  The
// order in which a row's terms land is therefore not fixed, in the reference
// as here, and results are compared within tolerance.
//
// COO: a warp takes 32 consecutive entries; lanes holding the same row in a
// run of consecutive lanes add their terms with a fixed shuffle tree, and the
// first lane of each run adds the run's sum to y with one atomic (sorted COO,
// the composer's output, has long runs; unsorted input has runs of one).
// CSC: one lane per column of up to 16 entries, the warp for longer ones,
// one atomic per entry.  Out-of-range coordinates raise the device bounds
// flag and are skipped.
#include "common.cuh"

namespace jlb {

JLB_DEFINE_DEV_ERROR(spmvfmt)

namespace spmvfmt {

constexpr int kThreads = 256;

template <typename T>
__global__ void scale_y(int64_t m, T *__restrict__ y, T beta, int zero) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += stride)
        y[i] = zero ? T(0) : mul_rn(beta, y[i]);
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
coo_entries(int64_t nnz, int64_t m, int64_t n, const int32_t *__restrict__ rows,
            const int32_t *__restrict__ cols, const T *__restrict__ val,
            const T *__restrict__ x, T *__restrict__ y, T alpha, int base) {
    const int lane = threadIdx.x % kWarp;
    const int64_t warps = (int64_t)gridDim.x * (kThreads / kWarp);
    for (int64_t w = ((int64_t)blockIdx.x * kThreads + threadIdx.x) / kWarp; w * kWarp < nnz;
         w += warps) {
        const int64_t p = w * kWarp + lane;
        int64_t r = -1;
        T t = T(0);
        if (p < nnz) {
            r = (int64_t)ldg(rows + p) - base;
            const int64_t c = (int64_t)ldg(cols + p) - base;
            if (r < 0 || r >= m || c < 0 || c >= n) {
                dev_error(DEV_ERR_BOUNDS);
                r = -1;
            } else {
                t = mul_rn(mul_rn(alpha, ldg(val + p)), ldg(x + c));
            }
        }
        // runs of equal rows over consecutive lanes; `end` = first lane of the next run
        const int64_t prev = __shfl_up_sync(0xffffffffu, r, 1);
        const bool head = lane == 0 || prev != r;
        const unsigned heads = __ballot_sync(0xffffffffu, head);
        const unsigned after = heads & ~((2u << lane) - 1u);
        const int end = after ? __ffs(after) - 1 : kWarp;
#pragma unroll
        for (int d = 1; d < kWarp; d <<= 1) {
            const T o = __shfl_down_sync(0xffffffffu, t, d);
            if (lane + d < end) t = add_rn(t, o);
        }
        if (head && r >= 0) atomicAdd(y + r, t);
    }
}

// CSC: a warp takes 32 columns at a time.  Each lane scatters its own column
// when it has at most kLaneEntries entries (one lane per column keeps the
// lanes busy on short columns); the warp then scatters the longer ones one
// after another, lanes over entries.  Every term is alpha*v*x[j], added to
// its row atomically.
constexpr int kLaneEntries = 16;

template <typename T>
__global__ void __launch_bounds__(kThreads)
csc_columns(int64_t n, int64_t m, int64_t nnz, const int32_t *__restrict__ colptr,
            const int32_t *__restrict__ rowind, const T *__restrict__ val,
            const T *__restrict__ x, T *__restrict__ y, T alpha, int base) {
    const int lane = threadIdx.x % kWarp;
    const int64_t warps = (int64_t)gridDim.x * (kThreads / kWarp);
    for (int64_t jb = ((int64_t)blockIdx.x * kThreads + threadIdx.x) / kWarp * kWarp; jb < n;
         jb += warps * kWarp) {
        const int64_t j = jb + lane;
        int lo = 0, hi = 0;
        bool valid = j < n;
        if (valid) {
            lo = ldg(colptr + j) - base;
            hi = ldg(colptr + j + 1) - base;
            if (lo < 0 || hi > nnz || lo > hi) {
                dev_error(DEV_ERR_BOUNDS);
                valid = false;
            }
        }
        if (valid && hi - lo <= kLaneEntries) {
            const T xj = ldg(x + j);
            for (int p = lo; p < hi; ++p) {
                const int64_t r = (int64_t)ldg(rowind + p) - base;
                if (r < 0 || r >= m) {
                    dev_error(DEV_ERR_BOUNDS);
                    continue;
                }
                atomicAdd(y + r, mul_rn(mul_rn(alpha, ldg(val + p)), xj));
            }
        }
        unsigned rest = __ballot_sync(0xffffffffu, valid && hi - lo > kLaneEntries);
        while (rest) {
            const int src = __ffs(rest) - 1;
            rest &= rest - 1;
            const int clo = __shfl_sync(0xffffffffu, lo, src), chi = __shfl_sync(0xffffffffu, hi, src);
            const T xj = ldg(x + jb + src);
            for (int p = clo + lane; p < chi; p += kWarp) {
                const int64_t r = (int64_t)ldg(rowind + p) - base;
                if (r < 0 || r >= m) {
                    dev_error(DEV_ERR_BOUNDS);
                    continue;
                }
                atomicAdd(y + r, mul_rn(mul_rn(alpha, ldg(val + p)), xj));
            }
        }
    }
}

inline unsigned grid_for(int64_t items) {
    const int64_t g = ceil_div(items > 0 ? items : 1, kThreads);
    return (unsigned)(g < 148 * 16 ? g : 148 * 16);
}

template <typename T>
int launch(cudaStream_t st, bool csc, int base, int64_t m, int64_t n, int64_t nnz,
           const int32_t *a, const int32_t *b, const void *val, const void *x, void *y,
           double alpha, double beta) {
    if (m > 0) {
        scale_y<T><<<grid_for(m), kThreads, 0, st>>>(m, (T *)y, (T)beta, beta == 0.0);
        JLB_LAUNCH_CHECK("scale_y");
    }
    if (csc) {
        if (n > 0) {
            csc_columns<T><<<grid_for(n), kThreads, 0, st>>>(
                n, m, nnz, a, b, (const T *)val, (const T *)x, (T *)y, (T)alpha, base);
            JLB_LAUNCH_CHECK("csc_columns");
        }
    } else if (nnz > 0) {
        coo_entries<T><<<grid_for(nnz), kThreads, 0, st>>>(nnz, m, n, a, b, (const T *)val,
                                                          (const T *)x, (T *)y, (T)alpha, base);
        JLB_LAUNCH_CHECK("coo_entries");
    }
    return ok();
}

int args(int dtype, int idx_base, int64_t m, int64_t n, int64_t nnz, const void *val,
         const void *x, const void *y) {
    if (dtype != JLB_F32 && dtype != JLB_F64)
        return fail(JLB_ERR_UNSUPPORTED_VALUE_TYPE, "SpMV supports Float32 and Float64 (dtype %d)", dtype);
    if (idx_base != 0 && idx_base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (m < 0 || n < 0 || nnz < 0) return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "negative extent");
    if (nnz > INT32_MAX - 1) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "nnz exceeds Int32 positions");
    if (m > 0 && !y) return fail(JLB_ERR_INVALID_ARGUMENT, "null y");
    if (nnz > 0 && (!val || !x)) return fail(JLB_ERR_INVALID_ARGUMENT, "null values or x");
    return JLB_OK;
}

}  // namespace spmvfmt
}  // namespace jlb

using namespace jlb;

extern "C" JLB_API int jlb_coo_spmv(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                    int64_t nnz, const int32_t *rows, const int32_t *cols,
                                    const void *val, const void *x, void *y, double alpha,
                                    double beta) {
    int st = spmvfmt::args(dtype, idx_base, m, n, nnz, val, x, y);
    if (st) return st;
    if (nnz > 0 && (!rows || !cols)) return fail(JLB_ERR_INVALID_ARGUMENT, "null coordinates");
    if (dtype == JLB_F64)
        return spmvfmt::launch<double>(as_stream(stream), false, idx_base, m, n, nnz, rows, cols,
                                       val, x, y, alpha, beta);
    return spmvfmt::launch<float>(as_stream(stream), false, idx_base, m, n, nnz, rows, cols, val,
                                  x, y, alpha, beta);
}

extern "C" JLB_API int jlb_csc_spmv(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                    int64_t nnz, const int32_t *colptr, const int32_t *rowind,
                                    const void *val, const void *x, void *y, double alpha,
                                    double beta) {
    int st = spmvfmt::args(dtype, idx_base, m, n, nnz, val, x, y);
    if (st) return st;
    if (n > 0 && !colptr) return fail(JLB_ERR_INVALID_ARGUMENT, "null column pointer");
    if (nnz > 0 && !rowind) return fail(JLB_ERR_INVALID_ARGUMENT, "null row coordinates");
    if (dtype == JLB_F64)
        return spmvfmt::launch<double>(as_stream(stream), true, idx_base, m, n, nnz, colptr,
                                       rowind, val, x, y, alpha, beta);
    return spmvfmt::launch<float>(as_stream(stream), true, idx_base, m, n, nnz, colptr, rowind,
                                  val, x, y, alpha, beta);
}
