// spmv.cu -- CSR SpMV for sm_100a, plus CSR structure validation.
//
// One CTA owns a tile of kRows consecutive rows (one thread per row).  The
// tile's slice of the value and column arrays is contiguous, so the CTA first
// stages it into shared memory with 16-byte vector loads (cache-streaming, so
// the gathered x keeps L2), then:
//   phase A  rows of <= kShortMax entries: one thread sums its row in storage
//            order with separately rounded products and sums -- the same
//            operations, in the same order, as JLUST's CPU walker
//            (ext/KernelAbstractionsExt/ops/_walker.jl:111-146 and
//            ops/spmv.jl:154,161-178), hence bit-identical results;
//   phase B  longer rows: one warp per row, lane-strided partial sums and a
//            fixed xor-butterfly (deterministic, within tolerance).
// A tile whose slice exceeds kCap entries (it holds long rows) runs the same
// two phases straight from global memory.  This replaces the reference's
// per-row walker kernels with their VS heuristic (KA spmv.jl:296-323) and its
// atomic merge-based kernel (ext/CUDAExt/ops/spmv.jl:129-191): the choice of
// thread / warp per row is made per row from its length, and no atomics touch
// y, so results are deterministic.
#include "common.cuh"

#include <new>

namespace jlb {

JLB_DEFINE_DEV_ERROR(spmv)

namespace spmv {

constexpr int kRows = 256;      // rows per tile == threads per CTA
constexpr int kCap = 2048;      // entries staged per tile
constexpr int kShortMax = 32;   // longest row summed by a single thread

template <typename T>
struct Vec16;
template <>
struct Vec16<double> { using type = double2; };
template <>
struct Vec16<float> { using type = float4; };
template <>
struct Vec16<int32_t> { using type = int4; };

// Copies src[p0, p1) into dst[p - pa], pa <= p0.  With `vec`, pa must be a
// multiple of the 16-byte vector width and src 16-byte aligned; whole vectors
// below p1 are moved with 16-byte loads, the ragged end element by element.
// Every load stays inside [pa, p1), which lies inside the caller's array.
template <typename T>
__device__ __forceinline__ void stage_range(T *dst, const T *__restrict__ src, int64_t pa,
                                            int64_t p0, int64_t p1, bool vec) {
    constexpr int E = 16 / (int)sizeof(T);
    using V = typename Vec16<T>::type;
    const int tid = threadIdx.x, nt = blockDim.x;
    int64_t tail = p0;
    if (vec) {
        const int64_t vb = pa / E, ve = p1 / E;
        const V *s = reinterpret_cast<const V *>(src);
        V *d = reinterpret_cast<V *>(dst);
        for (int64_t v = vb + tid; v < ve; v += nt) d[v - vb] = __ldcs(s + v);
        tail = ve * E > p0 ? ve * E : p0;
    }
    for (int64_t p = tail + tid; p < p1; p += nt) dst[p - pa] = __ldcs(src + p);
}

template <typename T>
struct __align__(16) Smem {
    T val[kCap + 16 / sizeof(T)];
    int32_t col[kCap + 4];
    int32_t rp[kRows + 1];
    int32_t longrows[kRows];
    int nlong;
};

template <typename T, bool kBeta>
__device__ __forceinline__ void write_row(T *y, int64_t r, T acc, T alpha, T beta) {
    T out = mul_rn(alpha, acc);
    if (kBeta) out = add_rn(out, mul_rn(beta, y[r]));
    y[r] = out;
}

template <typename T, bool kBeta>
__global__ void __launch_bounds__(kRows)
spmv_tiles(int64_t m, const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
           const T *__restrict__ val, const T *__restrict__ x, T *__restrict__ y, T alpha,
           T beta, int base, int vec_ok) {
    __shared__ Smem<T> s;
    const int tid = threadIdx.x;
    const int64_t r0 = (int64_t)blockIdx.x * kRows;
    const int nrows = (int)((m - r0) < kRows ? (m - r0) : kRows);
    for (int i = tid; i <= nrows; i += kRows) s.rp[i] = rowptr[r0 + i] - base;
    if (tid == 0) s.nlong = 0;
    __syncthreads();

    const int64_t p0 = s.rp[0], p1 = s.rp[nrows];
    constexpr int EV = 16 / (int)sizeof(T);
    const bool staged = (p1 - p0) <= kCap;
    const int64_t pav = vec_ok ? (p0 & ~(int64_t)(EV - 1)) : p0;
    const int64_t pac = vec_ok ? (p0 & ~(int64_t)3) : p0;
    if (staged) {
        stage_range<T>(s.val, val, pav, p0, p1, vec_ok);
        stage_range<int32_t>(s.col, colind, pac, p0, p1, vec_ok);
        __syncthreads();
    }

    // Phase A: short rows, one thread each, storage order.
    if (tid < nrows) {
        const int lo = s.rp[tid], hi = s.rp[tid + 1];
        if (hi - lo <= kShortMax) {
            T acc = T(0);
            if (staged) {
                for (int k = lo; k < hi; ++k)
                    acc = add_rn(acc, mul_rn(s.val[k - pav], ldg(x + (s.col[k - pac] - base))));
            } else {
                for (int k = lo; k < hi; ++k)
                    acc = add_rn(acc, mul_rn(ldg(val + k), ldg(x + (ldg(colind + k) - base))));
            }
            write_row<T, kBeta>(y, r0 + tid, acc, alpha, beta);
        } else {
            s.longrows[atomicAdd(&s.nlong, 1)] = tid;
        }
    }
    __syncthreads();

    // Phase B: long rows, one warp each.
    const int warp = tid / kWarp, lane = tid % kWarp;
    for (int i = warp; i < s.nlong; i += kRows / kWarp) {
        const int t = s.longrows[i];
        const int lo = s.rp[t], hi = s.rp[t + 1];
        T acc = T(0);
        if (staged) {
            for (int k = lo + lane; k < hi; k += kWarp)
                acc = add_rn(acc, mul_rn(s.val[k - pav], ldg(x + (s.col[k - pac] - base))));
        } else {
            for (int k = lo + lane; k < hi; k += kWarp)
                acc = add_rn(acc, mul_rn(__ldcs(val + k), ldg(x + (__ldcs(colind + k) - base))));
        }
        acc = warp_sum(acc);
        if (lane == 0) write_row<T, kBeta>(y, r0 + t, acc, alpha, beta);
    }
}

template <typename T>
int launch(cudaStream_t st, int base, int64_t m, const int32_t *rowptr, const int32_t *colind,
           const void *val, const void *x, void *y, double alpha, double beta) {
    if (m == 0) return ok();
    const int vec_ok = aligned16(val) && aligned16(colind);
    const T a = (T)alpha, b = (T)beta;
    const unsigned grid = (unsigned)ceil_div(m, kRows);
    if (b == T(0))
        spmv_tiles<T, false><<<grid, kRows, 0, st>>>(m, rowptr, colind, (const T *)val,
                                                      (const T *)x, (T *)y, a, b, base, vec_ok);
    else
        spmv_tiles<T, true><<<grid, kRows, 0, st>>>(m, rowptr, colind, (const T *)val,
                                                     (const T *)x, (T *)y, a, b, base, vec_ok);
    JLB_LAUNCH_CHECK("spmv_tiles");
    return ok();
}

// ------------------------------------------------------------- validation
static __device__ int g_validate_flags;

__global__ void csr_validate_kernel(int64_t m, int64_t n, int64_t nnz,
                                    const int32_t *__restrict__ rowptr,
                                    const int32_t *__restrict__ colind, int base,
                                    int require_sorted, int32_t *__restrict__ stats) {
    // stats[0] = max row length, stats[1] = number of tiles above kCap entries
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < m; r += stride) {
        const int64_t lo = (int64_t)rowptr[r] - base, hi = (int64_t)rowptr[r + 1] - base;
        if (r == 0 && lo != 0) atomicOr(&g_validate_flags, 1);
        if (r == m - 1 && hi != nnz) atomicOr(&g_validate_flags, 2);
        if (hi < lo || lo < 0 || hi > nnz) { atomicOr(&g_validate_flags, 4); continue; }
        if (stats) {
            atomicMax(&stats[0], (int32_t)(hi - lo));
            if (r % kRows == 0) {
                const int64_t re = (r + kRows < m) ? r + kRows : m;
                const int64_t tn = (int64_t)rowptr[re] - base - lo;
                if (tn > kCap) atomicAdd(&stats[1], 1);
            }
        }
        int64_t prev = -1;
        for (int64_t k = lo; k < hi; ++k) {
            const int64_t c = (int64_t)colind[k] - base;
            if (c < 0 || c >= n) { atomicOr(&g_validate_flags, 8); break; }
            if (require_sorted && c <= prev) { atomicOr(&g_validate_flags, 16); break; }
            prev = c;
        }
    }
}

}  // namespace spmv

// Runs the validation kernel; on success optionally returns (max row, tiles
// above the staging capacity) through stats_host.
int csr_validate_impl(cudaStream_t st, int base, int64_t m, int64_t n, int64_t nnz,
                      const int32_t *rowptr, const int32_t *colind, int require_sorted,
                      int32_t *stats_dev, int32_t *stats_host) {
    if (m < 0 || n < 0 || nnz < 0) return fail(JLB_ERR_INVALID_ARGUMENT, "negative extent");
    if (base != 0 && base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (nnz > INT32_MAX - 1) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "nnz %lld exceeds Int32 positions", (long long)nnz);
    if (!rowptr || (nnz > 0 && !colind)) return fail(JLB_ERR_INVALID_ARGUMENT, "null index buffer");
    const int zero = 0;
    JLB_CUDA(cudaMemcpyToSymbolAsync(spmv::g_validate_flags, &zero, sizeof(int), 0,
                                     cudaMemcpyHostToDevice, st));
    if (stats_dev) JLB_CUDA(cudaMemsetAsync(stats_dev, 0, 2 * sizeof(int32_t), st));
    if (m > 0) {
        const unsigned grid = (unsigned)(ceil_div(m, 256) < 148 * 16 ? ceil_div(m, 256) : 148 * 16);
        spmv::csr_validate_kernel<<<grid, 256, 0, st>>>(m, n, nnz, rowptr, colind, base,
                                                        require_sorted, stats_dev);
        JLB_LAUNCH_CHECK("csr_validate_kernel");
    } else {
        int32_t first = 0;
        JLB_CUDA(cudaMemcpyAsync(&first, rowptr, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
        JLB_CUDA(cudaStreamSynchronize(st));
        if (first != base || nnz != 0)
            return fail(JLB_ERR_NONCANONICAL_STORAGE, "empty CSR must have rowptr == [idx_base] and nnz == 0");
    }
    int flags = 0;
    JLB_CUDA(cudaMemcpyFromSymbolAsync(&flags, spmv::g_validate_flags, sizeof(int), 0,
                                       cudaMemcpyDeviceToHost, st));
    if (stats_dev && stats_host)
        JLB_CUDA(cudaMemcpyAsync(stats_host, stats_dev, 2 * sizeof(int32_t),
                                 cudaMemcpyDeviceToHost, st));
    JLB_CUDA(cudaStreamSynchronize(st));
    if (flags & 1) return fail(JLB_ERR_NONCANONICAL_STORAGE, "rowptr[0] != idx_base");
    if (flags & 2) return fail(JLB_ERR_NONCANONICAL_STORAGE, "rowptr[m] != nnz + idx_base");
    if (flags & 4) return fail(JLB_ERR_NONCANONICAL_STORAGE, "rowptr is not non-decreasing within [idx_base, nnz+idx_base]");
    if (flags & 8) return fail(JLB_ERR_NONCANONICAL_STORAGE, "column index outside [idx_base, n+idx_base)");
    if (flags & 16) return fail(JLB_ERR_NONCANONICAL_STORAGE, "columns not strictly increasing within a row");
    return ok();
}

}  // namespace jlb

using namespace jlb;

extern "C" JLB_API int jlb_csr_validate(void *stream, int idx_base, int64_t m, int64_t n,
                                        int64_t nnz, const int32_t *rowptr,
                                        const int32_t *colind, int require_sorted) {
    return csr_validate_impl(as_stream(stream), idx_base, m, n, nnz, rowptr, colind,
                             require_sorted, nullptr, nullptr);
}

static int spmv_args(int dtype, int idx_base, int64_t m, int64_t n, int64_t nnz,
                     const int32_t *rowptr, const int32_t *colind, const void *val,
                     const void *x, const void *y) {
    if (dtype != JLB_F32 && dtype != JLB_F64)
        return fail(JLB_ERR_UNSUPPORTED_VALUE_TYPE, "SpMV supports Float32 and Float64 (dtype %d)", dtype);
    if (idx_base != 0 && idx_base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (m < 0 || n < 0 || nnz < 0) return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "negative extent");
    if (nnz > INT32_MAX - 1) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "nnz exceeds Int32 positions");
    if (m > 0 && (!rowptr || !y)) return fail(JLB_ERR_INVALID_ARGUMENT, "null rowptr or y");
    if (nnz > 0 && (!colind || !val || !x)) return fail(JLB_ERR_INVALID_ARGUMENT, "null colind, val or x");
    return JLB_OK;
}

extern "C" JLB_API int jlb_csr_spmv(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                    int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                                    const void *val, const void *x, void *y, double alpha,
                                    double beta) {
    int st = spmv_args(dtype, idx_base, m, n, nnz, rowptr, colind, val, x, y);
    if (st) return st;
    if (dtype == JLB_F64)
        return spmv::launch<double>(as_stream(stream), idx_base, m, rowptr, colind, val, x, y,
                                    alpha, beta);
    return spmv::launch<float>(as_stream(stream), idx_base, m, rowptr, colind, val, x, y, alpha,
                               beta);
}

struct jlb_spmv_plan_s {
    int dtype, base;
    int64_t m, n, nnz;
    const int32_t *rowptr, *colind;
    int64_t max_row;
    int64_t wide_tiles;
    int variant;
};

extern "C" JLB_API int jlb_spmv_plan_create(jlb_spmv_plan *plan, void *stream, int dtype,
                                            int idx_base, int64_t m, int64_t n, int64_t nnz,
                                            const int32_t *rowptr, const int32_t *colind) {
    if (!plan) return fail(JLB_ERR_INVALID_ARGUMENT, "null plan out-pointer");
    *plan = nullptr;
    int st = spmv_args(dtype, idx_base, m, n, nnz, rowptr, colind, (const void *)1,
                       (const void *)1, (void *)1);
    if (st) return st;
    int32_t *stats_dev = nullptr;
    JLB_CUDA(cudaMallocAsync((void **)&stats_dev, 2 * sizeof(int32_t), as_stream(stream)));
    int32_t stats[2] = {0, 0};
    st = csr_validate_impl(as_stream(stream), idx_base, m, n, nnz, rowptr, colind, 0, stats_dev,
                           stats);
    cudaFreeAsync(stats_dev, as_stream(stream));
    if (st) return st;
    jlb_spmv_plan p = new (std::nothrow) jlb_spmv_plan_s;
    if (!p) return fail(JLB_ERR_INVALID_ARGUMENT, "out of host memory");
    p->dtype = dtype; p->base = idx_base; p->m = m; p->n = n; p->nnz = nnz;
    p->rowptr = rowptr; p->colind = colind;
    p->max_row = stats[0];
    p->wide_tiles = stats[1];
    p->variant = (stats[0] <= spmv::kShortMax && stats[1] == 0) ? 0 : 1;
    *plan = p;
    return ok();
}

extern "C" JLB_API int jlb_spmv_plan_execute(jlb_spmv_plan p, void *stream, const void *val,
                                             const void *x, void *y, double alpha, double beta) {
    if (!p) return fail(JLB_ERR_INVALID_ARGUMENT, "null plan");
    int st = spmv_args(p->dtype, p->base, p->m, p->n, p->nnz, p->rowptr, p->colind, val, x, y);
    if (st) return st;
    if (p->dtype == JLB_F64)
        return spmv::launch<double>(as_stream(stream), p->base, p->m, p->rowptr, p->colind, val,
                                    x, y, alpha, beta);
    return spmv::launch<float>(as_stream(stream), p->base, p->m, p->rowptr, p->colind, val, x, y,
                               alpha, beta);
}

extern "C" JLB_API int jlb_spmv_plan_info(jlb_spmv_plan p, int64_t *max_row, double *mean_row,
                                          int *variant) {
    if (!p) return fail(JLB_ERR_INVALID_ARGUMENT, "null plan");
    if (max_row) *max_row = p->max_row;
    if (mean_row) *mean_row = p->m > 0 ? (double)p->nnz / (double)p->m : 0.0;
    if (variant) *variant = p->variant;
    return ok();
}

extern "C" JLB_API int jlb_spmv_plan_destroy(jlb_spmv_plan p) {
    delete p;
    return ok();
}
