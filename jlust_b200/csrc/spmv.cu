// spmv.cu -- CSR SpMV for sm_100a, plus CSR structure validation.
//
// One thread per row.  A row of up to kShortMax entries is summed by its
// thread in storage order with separately rounded products and sums -- the
// same operations, in the same order, as JLUST's CPU walker
// (ext/KernelAbstractionsExt/ops/_walker.jl:111-146 and ops/spmv.jl:154,
// 161-178), hence bit-identical results.  The thread reads its entries
// directly through the read-only path: the 32 rows of a warp occupy one
// contiguous slice of the value and column arrays, so the L1 turns the
// threads' strided reads into whole-line fetches and every byte of the
// slice crosses HBM once (measured on B200: 95% of the copy bandwidth on the
// 4096^2 Laplacian; staging the slice in shared memory first was slower).
// The x gathers of four entries are issued before their sums.
//
// Rows longer than kShortMax are found with a warp ballot and summed by the
// whole warp: lane-strided partial sums and a fixed xor-butterfly
// (deterministic, within tolerance).  No atomics touch y.  This replaces the
// reference's per-row walker kernels with their VS heuristic
// (KA spmv.jl:296-323) and its atomic merge-based kernel
// (ext/CUDAExt/ops/spmv.jl:129-191): thread or warp per row is chosen per row
// from its length.
#include "common.cuh"

#include <new>

namespace jlb {

JLB_DEFINE_DEV_ERROR(spmv)

namespace spmv {

constexpr int kThreads = 256;
constexpr int kShortMax = 32;   // longest row summed by a single thread
constexpr double kScalarMean = 12.0;   // thread per row up to this mean row length

template <typename T, bool kBeta>
__device__ __forceinline__ void write_row(T *y, int64_t r, T acc, T alpha, T beta) {
    T out = mul_rn(alpha, acc);
    if (kBeta) out = add_rn(out, mul_rn(beta, y[r]));
    y[r] = out;
}

// Sum of entries [lo, hi) in storage order.
template <typename T>
__device__ __forceinline__ T row_sum(int lo, int hi, const int32_t *__restrict__ colind,
                                     const T *__restrict__ val, const T *__restrict__ x, int base) {
    T acc = T(0);
    int k = lo;
    for (; k + 4 <= hi; k += 4) {
        const int c0 = ldg(colind + k), c1 = ldg(colind + k + 1);
        const int c2 = ldg(colind + k + 2), c3 = ldg(colind + k + 3);
        const T v0 = ldg(val + k), v1 = ldg(val + k + 1), v2 = ldg(val + k + 2), v3 = ldg(val + k + 3);
        const T x0 = ldg(x + (c0 - base)), x1 = ldg(x + (c1 - base));
        const T x2 = ldg(x + (c2 - base)), x3 = ldg(x + (c3 - base));
        acc = add_rn(acc, mul_rn(v0, x0));
        acc = add_rn(acc, mul_rn(v1, x1));
        acc = add_rn(acc, mul_rn(v2, x2));
        acc = add_rn(acc, mul_rn(v3, x3));
    }
    for (; k < hi; ++k) acc = add_rn(acc, mul_rn(ldg(val + k), ldg(x + (ldg(colind + k) - base))));
    return acc;
}

// kRowIds: DCSR, whose compressed outer level stores only the non-empty rows:
// `m` counts the stored rows, rowptr is the inner level's position buffer and
// row_ids[f] the row of stored row f (JLUST's DCSR walk,
// ext/KernelAbstractionsExt/ops/_walker.jl:323-342: rows not stored are not
// written).  Otherwise plain CSR with row_ids unused.
template <typename T, bool kBeta, bool kRowIds = false>
__global__ void __launch_bounds__(kThreads)
spmv_rows(int64_t m, const int32_t *__restrict__ rowptr, const int32_t *__restrict__ colind,
          const T *__restrict__ val, const T *__restrict__ x, T *__restrict__ y, T alpha, T beta,
          int base, const int32_t *__restrict__ row_ids = nullptr, int64_t nrows = 0) {
    const int64_t f = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    const int lane = threadIdx.x % kWarp;
    int lo = 0, hi = 0;
    int64_t r = f;
    bool live = f < m;
    if (live) {
        lo = ldg(rowptr + f) - base;
        hi = ldg(rowptr + f + 1) - base;
        if (kRowIds) {
            r = (int64_t)ldg(row_ids + f) - base;
            if (r < 0 || r >= nrows) {
                dev_error(DEV_ERR_BOUNDS);
                live = false;
            }
        }
    }
    const bool is_long = hi - lo > kShortMax;
    if (live && !is_long) write_row<T, kBeta>(y, r, row_sum<T>(lo, hi, colind, val, x, base), alpha, beta);
    unsigned longs = __ballot_sync(0xffffffffu, live && is_long);
    while (longs) {
        const int src = __ffs(longs) - 1;
        longs &= longs - 1;
        const int l = __shfl_sync(0xffffffffu, lo, src), h = __shfl_sync(0xffffffffu, hi, src);
        // lane-strided over the row, four entries of each lane in flight:
        // their columns and values, then their four x gathers, then the sums
        T acc = T(0);
        int k = l + lane;
        for (; k + 3 * kWarp < h; k += 4 * kWarp) {
            int c[4];
            T v[4], xv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                c[u] = __ldcs(colind + k + u * kWarp);
                v[u] = __ldcs(val + k + u * kWarp);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) xv[u] = ldg(x + (c[u] - base));
#pragma unroll
            for (int u = 0; u < 4; ++u) acc = add_rn(acc, mul_rn(v[u], xv[u]));
        }
        for (; k < h; k += kWarp)
            acc = add_rn(acc, mul_rn(__ldcs(val + k), ldg(x + (__ldcs(colind + k) - base))));
        acc = warp_sum(acc);
        if (lane == src) write_row<T, kBeta>(y, r, acc, alpha, beta);
    }
}

// ------------------------------------------------------- vector-per-row
// Four consecutive entries [q, q+4) of the value and column arrays: one
// 16-byte load of columns and 16-byte loads of values when the quad lies
// inside the arrays (q is a multiple of 4 and both arrays are 16-byte
// aligned), scalar loads of the valid entries otherwise.
template <typename T>
struct Quad {
    int c[4];
    T v[4];
};

template <typename T>
__device__ __forceinline__ void load_quad(Quad<T> &d, int q, int lo, int hi, int nnz,
                                          const int32_t *__restrict__ colind,
                                          const T *__restrict__ val) {
    if (q + 4 <= nnz) {
        const int4 c = __ldcs(reinterpret_cast<const int4 *>(colind + q));
        d.c[0] = c.x; d.c[1] = c.y; d.c[2] = c.z; d.c[3] = c.w;
        if constexpr (sizeof(T) == 8) {
            const double2 a = __ldcs(reinterpret_cast<const double2 *>(val + q));
            const double2 b = __ldcs(reinterpret_cast<const double2 *>(val + q + 2));
            d.v[0] = a.x; d.v[1] = a.y; d.v[2] = b.x; d.v[3] = b.y;
        } else {
            const float4 a = __ldcs(reinterpret_cast<const float4 *>(val + q));
            d.v[0] = a.x; d.v[1] = a.y; d.v[2] = a.z; d.v[3] = a.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const bool in = q + i >= lo && q + i < hi;
            d.c[i] = in ? ldg(colind + q + i) : 0;
            d.v[i] = in ? ldg(val + q + i) : T(0);
        }
    }
}

// Rows summed by groups of W lanes (W = 2 .. 32, the reference's warp-vector
// width VS, KA spmv.jl:296-323).  Lane l of a row's group takes the quads
// q = a0 + 4*l, a0 + 4*(l + W), ... (a0 = the row's first entry rounded down
// to a multiple of 4), two at a time, adds the products of the quads'
// entries that belong to the row in storage order, and the group adds its W
// partial sums with a fixed xor butterfly: deterministic, within tolerance
// of the sequential sum.  The W lanes of a group read 16*W contiguous bytes of columns and
// 32*W (fp64) or 16*W (fp32) of values per step.
template <int W, typename T>
__device__ __forceinline__ T group_sum(T v) {
#pragma unroll
    for (int o = W / 2; o > 0; o >>= 1) v = add_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <typename T, int W, bool kBeta>
__global__ void __launch_bounds__(kThreads)
spmv_vec(int64_t m, int nnz, const int32_t *__restrict__ rowptr,
         const int32_t *__restrict__ colind, const T *__restrict__ val,
         const T *__restrict__ x, T *__restrict__ y, T alpha, T beta, int base) {
    constexpr int kRowsPerCta = kThreads / W;
    const int lane = threadIdx.x % W;
    const int64_t stride = (int64_t)gridDim.x * kRowsPerCta;
    // every lane of a warp runs the same number of row iterations (the
    // stride is a whole number of warps' rows), so the butterfly below sees
    // the whole warp converged
    const int64_t first = (int64_t)blockIdx.x * kRowsPerCta + threadIdx.x / W;
    const int64_t warp_first = first - (threadIdx.x % kWarp) / W;
    for (int64_t r0 = warp_first; r0 < m; r0 += stride) {
        const int64_t r = r0 + (threadIdx.x % kWarp) / W;
        const bool live = r < m;
        int lo = 0, hi = 0;
        if (live) {
            lo = ldg(rowptr + r) - base;
            hi = ldg(rowptr + r + 1) - base;
        }
        T acc = T(0);
        // two quads of the lane in flight per step: both quads' loads, then
        // their eight x gathers, then the sums in entry order
        for (int q = (lo & ~3) + 4 * lane; q < hi; q += 8 * W) {
            Quad<T> d0, d1;
            const int q1 = q + 4 * W;
            load_quad<T>(d0, q, lo, hi, nnz, colind, val);
            if (q1 < hi) load_quad<T>(d1, q1, lo, hi, nnz, colind, val);
            T xs0[4], xs1[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                xs0[i] = (q + i >= lo && q + i < hi) ? ldg(x + (d0.c[i] - base)) : T(0);
                xs1[i] = (q1 + i < hi) ? ldg(x + (d1.c[i] - base)) : T(0);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (q + i >= lo && q + i < hi) acc = add_rn(acc, mul_rn(d0.v[i], xs0[i]));
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (q1 + i < hi) acc = add_rn(acc, mul_rn(d1.v[i], xs1[i]));
        }
        acc = group_sum<W>(acc);
        if (live && lane == 0) write_row<T, kBeta>(y, r, acc, alpha, beta);
    }
}

// CSR SpMV plus selector patches: the assembled CSR of a BlockSparseMatrix
// whose constant shifted-identity blocks were kept out of it.  Patch p adds
// val[p] * x[row - rows[2p] + cols[p]] to rows rows[2p] .. rows[2p+1].  Each
// row sums its CSR entries in storage order (one thread per row, also for
// long rows), the patches in patch order into a second sum, then adds the
// two: the operations of JLUST's patched kernel
// (ext/KernelAbstractionsExt/ops/block_periodic.jl:40-79).  A null rowptr
// means no CSR entries (a standalone ShiftedDiag tensor, whose one patch
// gives each row val * x[r + shift] as JLUST's walker does with a
// ShiftedDiag leaf, src/backends.jl:223-227); alpha scales the row (exact
// for alpha = 1, the BlockSparseMatrix case).
template <typename T, bool kBeta>
__global__ void __launch_bounds__(kThreads)
patched_rows(int64_t m, int64_t n, const int32_t *__restrict__ rowptr,
             const int32_t *__restrict__ colind, const T *__restrict__ val, int npatch,
             const int64_t *__restrict__ prows, const int64_t *__restrict__ pcols,
             const double *__restrict__ pvals, const T *__restrict__ x, T *__restrict__ y,
             T alpha, T beta, int base) {
    const int64_t r = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (r >= m) return;
    T acc = rowptr ? row_sum<T>(ldg(rowptr + r) - base, ldg(rowptr + r + 1) - base, colind, val,
                                x, base)
                   : T(0);
    bool bad = false;
    const T pacc = patch_sum<T>(r, npatch, prows, pcols, pvals, x, 0, n, bad);
    if (bad) dev_error(DEV_ERR_BOUNDS);
    T out = mul_rn(alpha, add_rn(acc, pacc));
    if (kBeta) out = add_rn(out, mul_rn(beta, y[r]));
    y[r] = out;
}

template <typename T>
int launch_patched(cudaStream_t st, int base, int64_t m, int64_t n, const int32_t *rowptr,
                   const int32_t *colind, const void *val, int npatch, const int64_t *prows,
                   const int64_t *pcols, const double *pvals, const void *x, void *y,
                   double alpha, double beta) {
    if (m == 0) return ok();
    const unsigned grid = (unsigned)ceil_div(m, kThreads);
    const T a = (T)alpha, b = (T)beta;
    if (b == T(0))
        patched_rows<T, false><<<grid, kThreads, 0, st>>>(m, n, rowptr, colind, (const T *)val,
                                                          npatch, prows, pcols, pvals,
                                                          (const T *)x, (T *)y, a, b, base);
    else
        patched_rows<T, true><<<grid, kThreads, 0, st>>>(m, n, rowptr, colind, (const T *)val,
                                                         npatch, prows, pcols, pvals,
                                                         (const T *)x, (T *)y, a, b, base);
    JLB_LAUNCH_CHECK("patched_rows");
    return ok();
}

template <typename T>
int launch_dcsr(cudaStream_t st, int base, int64_t nrows, int64_t nfib, const int32_t *fibptr,
                const int32_t *row_ids, const int32_t *colind, const void *val, const void *x,
                void *y, double alpha, double beta) {
    if (nfib == 0) return ok();
    const T a = (T)alpha, b = (T)beta;
    const unsigned grid = (unsigned)ceil_div(nfib, kThreads);
    if (b == T(0))
        spmv_rows<T, false, true><<<grid, kThreads, 0, st>>>(nfib, fibptr, colind, (const T *)val,
                                                              (const T *)x, (T *)y, a, b, base,
                                                              row_ids, nrows);
    else
        spmv_rows<T, true, true><<<grid, kThreads, 0, st>>>(nfib, fibptr, colind, (const T *)val,
                                                             (const T *)x, (T *)y, a, b, base,
                                                             row_ids, nrows);
    JLB_LAUNCH_CHECK("spmv_rows (DCSR)");
    return ok();
}

template <typename T, int W>
void launch_vec(cudaStream_t st, int base, int64_t m, int64_t nnz, const int32_t *rowptr,
                const int32_t *colind, const T *val, const T *x, T *y, T a, T b) {
    constexpr int kRowsPerCta = kThreads / W;
    const int64_t need = ceil_div(m, kRowsPerCta);
    const unsigned grid = (unsigned)(need < 148 * 16 ? need : 148 * 16);
    if (b == T(0))
        spmv_vec<T, W, false><<<grid, kThreads, 0, st>>>(m, (int)nnz, rowptr, colind, val, x, y, a, b, base);
    else
        spmv_vec<T, W, true><<<grid, kThreads, 0, st>>>(m, (int)nnz, rowptr, colind, val, x, y, a, b, base);
}

// ------------------------------------------------------ banded, staged x
// Variant 1, for banded structure: a CTA takes kBandRows consecutive rows,
// whose columns all lie in [r0 - lbw, r1 + ubw) (lbw, ubw: the matrix's
// lower and upper bandwidths, from the plan), and stages that window of x in
// shared memory with one bulk copy (cp.async.bulk, completion on an
// mbarrier) before summing.  Rows are summed as variant 0 sums them (a
// thread per row of up to kShortMax entries in storage order -- bit-exact --
// the warp for longer rows), reading x from shared memory; a column outside
// the window (structure changed since the plan) reads x from global memory.
// The wait for the copy is bounded: past it the device error word is set and
// x is read from global memory; the copy is waited for (bounded) again
// before the CTA exits.
constexpr int kBandRowsPerThread = 4;
constexpr int kBandRows = kThreads * kBandRowsPerThread;
constexpr size_t kBandMaxSmem = 110 * 1024;   // two CTAs an SM
constexpr long long kBandWaitCycles = 2000000000ll;   // ~1 s

__device__ __forceinline__ bool band_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ bool band_wait(uint32_t bar) {
    const long long t0 = clock64();
    while (!band_try_wait(bar, 0))
        if (clock64() - t0 > kBandWaitCycles) return false;
    return true;
}

// x window of the CTA's rows: first column (a 16-byte boundary) and bytes (a
// multiple of 16; the last 16-byte block may extend past x's end inside the
// block that holds its last element)
template <typename T>
__host__ __device__ inline void band_window(int64_t r0, int64_t r1, int64_t n, int64_t lbw,
                                            int64_t ubw, int64_t &w0, int64_t &bytes) {
    constexpr int64_t kPer16 = 16 / (int64_t)sizeof(T);
    int64_t a = r0 - lbw, b = r1 + ubw;
    if (a < 0) a = 0;
    if (b > n) b = n;
    a &= ~(kPer16 - 1);
    w0 = a;
    bytes = b > a ? (((b - a) * (int64_t)sizeof(T) + 15) & ~(int64_t)15) : 0;
}

template <typename T, bool kBeta>
__global__ void __launch_bounds__(kThreads)
spmv_band(int64_t m, int64_t n, const int32_t *__restrict__ rowptr,
          const int32_t *__restrict__ colind, const T *__restrict__ val, const T *__restrict__ x,
          T *__restrict__ y, T alpha, T beta, int base, int64_t lbw, int64_t ubw) {
    extern __shared__ __align__(16) unsigned char band_smem[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ int s_ok;
    const int lane = threadIdx.x % kWarp;
    const int64_t r0 = (int64_t)blockIdx.x * kBandRows;
    const int64_t r1 = r0 + kBandRows < m ? r0 + kBandRows : m;
    int64_t w0, bytes;
    band_window<T>(r0, r1, n, lbw, ubw, w0, bytes);
    const T *xs = reinterpret_cast<const T *>(band_smem);
    const uint32_t bar_a = static_cast<uint32_t>(__cvta_generic_to_shared(&bar));
    if (threadIdx.x == 0) {
        s_ok = 1;
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_a) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0 && bytes > 0) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_a),
                     "r"((uint32_t)bytes)
                     : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
            ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(band_smem))), "l"(x + w0),
            "r"((uint32_t)bytes), "r"(bar_a)
            : "memory");
    }
    if (bytes > 0 && !band_wait(bar_a)) {
        s_ok = 0;
        dev_error(DEV_ERR_TIMEOUT);
    }
    __syncthreads();
    const bool staged = s_ok != 0;
    const int64_t wn = bytes / (int64_t)sizeof(T);
    auto xat = [&](int c) -> T {   // c: 0-based column
        const int64_t i = (int64_t)c - w0;
        return staged && i >= 0 && i < wn ? xs[i] : ldg(x + c);
    };
#pragma unroll 1
    for (int j = 0; j < kBandRowsPerThread; ++j) {
        const int64_t r = r0 + (int64_t)j * kThreads + threadIdx.x;
        const bool live = r < r1;
        int lo = 0, hi = 0;
        if (live) {
            lo = ldg(rowptr + r) - base;
            hi = ldg(rowptr + r + 1) - base;
        }
        const bool is_long = hi - lo > kShortMax;
        if (live && !is_long) {
            T acc = T(0);
            for (int k = lo; k < hi; ++k) acc = add_rn(acc, mul_rn(ldg(val + k), xat(ldg(colind + k) - base)));
            write_row<T, kBeta>(y, r, acc, alpha, beta);
        }
        unsigned longs = __ballot_sync(0xffffffffu, live && is_long);
        while (longs) {
            const int src = __ffs(longs) - 1;
            longs &= longs - 1;
            const int l = __shfl_sync(0xffffffffu, lo, src), h = __shfl_sync(0xffffffffu, hi, src);
            T acc = T(0);
            for (int k = l + lane; k < h; k += kWarp)
                acc = add_rn(acc, mul_rn(__ldcs(val + k), xat(__ldcs(colind + k) - base)));
            acc = warp_sum(acc);
            if (lane == src) write_row<T, kBeta>(y, r, acc, alpha, beta);   // lane src's own row
        }
    }
    // a copy that outlived the bounded wait lands before the CTA exits
    if (!staged && threadIdx.x == 0 && !band_wait(bar_a)) dev_error(DEV_ERR_TIMEOUT);
}

// Launches variant 1 when the window fits; false otherwise (the caller then
// runs variant 0).
template <typename T>
bool launch_band(cudaStream_t st, int base, int64_t m, int64_t n, const int32_t *rowptr,
                 const int32_t *colind, const T *val, const T *x, T *y, T a, T b, int64_t lbw,
                 int64_t ubw) {
    const int64_t span = kBandRows + lbw + ubw + 16;
    if (lbw < 0 || ubw < 0 || span * (int64_t)sizeof(T) > (int64_t)kBandMaxSmem || !aligned16(x))
        return false;
    const size_t smem = (size_t)(((span * (int64_t)sizeof(T)) + 15) & ~(int64_t)15);
    const unsigned grid = (unsigned)ceil_div(m, kBandRows);
    if (b == T(0)) {
        if (cudaFuncSetAttribute(spmv_band<T, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return false;
        spmv_band<T, false><<<grid, kThreads, smem, st>>>(m, n, rowptr, colind, val, x, y, a, b, base,
                                                          lbw, ubw);
    } else {
        if (cudaFuncSetAttribute(spmv_band<T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return false;
        spmv_band<T, true><<<grid, kThreads, smem, st>>>(m, n, rowptr, colind, val, x, y, a, b, base,
                                                         lbw, ubw);
    }
    return true;
}

template <typename T>
int launch(cudaStream_t st, int base, int64_t m, int64_t nnz, const int32_t *rowptr,
           const int32_t *colind, const void *val, const void *x, void *y, double alpha,
           double beta) {
    if (m == 0) return ok();
    const T a = (T)alpha, b = (T)beta;
    const unsigned grid = (unsigned)ceil_div(m, kThreads);
    if (b == T(0))
        spmv_rows<T, false><<<grid, kThreads, 0, st>>>(m, rowptr, colind, (const T *)val,
                                                        (const T *)x, (T *)y, a, b, base);
    else
        spmv_rows<T, true><<<grid, kThreads, 0, st>>>(m, rowptr, colind, (const T *)val,
                                                       (const T *)x, (T *)y, a, b, base);
    JLB_LAUNCH_CHECK("spmv_rows");
    return ok();
}

// Variant 0: a thread per row (bit-exact for rows of up to kShortMax entries),
// the warp for longer rows.  Variant 1: the same sums with x staged in shared
// memory per block of rows (banded structure; needs the bandwidths and a
// window that fits, else variant 0 runs).  Variant W in {2, 4, 8, 16, 32}:
// groups of W lanes per row; they need 16-byte aligned colind and val (else
// variant 0 runs).
template <typename T>
int launch_variant(cudaStream_t st, int base, int64_t m, int64_t nnz, const int32_t *rowptr,
                   const int32_t *colind, const void *val, const void *x, void *y, double alpha,
                   double beta, int variant, int64_t n = 0, int64_t lbw = -1, int64_t ubw = -1) {
    if (m == 0) return ok();
    if (variant == 1) {
        if (launch_band<T>(st, base, m, n, rowptr, colind, (const T *)val, (const T *)x, (T *)y,
                           (T)alpha, (T)beta, lbw, ubw)) {
            JLB_LAUNCH_CHECK("spmv_band");
            return ok();
        }
        variant = 0;
    }
    if (variant != 0 && aligned16(colind) && aligned16(val)) {
        const T a = (T)alpha, b = (T)beta;
        const T *v = (const T *)val, *xx = (const T *)x;
        T *yy = (T *)y;
        switch (variant) {
            case 2: launch_vec<T, 2>(st, base, m, nnz, rowptr, colind, v, xx, yy, a, b); break;
            case 4: launch_vec<T, 4>(st, base, m, nnz, rowptr, colind, v, xx, yy, a, b); break;
            case 8: launch_vec<T, 8>(st, base, m, nnz, rowptr, colind, v, xx, yy, a, b); break;
            case 16: launch_vec<T, 16>(st, base, m, nnz, rowptr, colind, v, xx, yy, a, b); break;
            default: launch_vec<T, 32>(st, base, m, nnz, rowptr, colind, v, xx, yy, a, b); break;
        }
        JLB_LAUNCH_CHECK("spmv_vec");
        return ok();
    }
    return launch<T>(st, base, m, nnz, rowptr, colind, val, x, y, alpha, beta);
}


// ------------------------------------------------------------- validation
static __device__ int g_validate_flags;
constexpr int kValidateStats = 5;

__global__ void csr_validate_kernel(int64_t m, int64_t n, int64_t nnz,
                                    const int32_t *__restrict__ rowptr,
                                    const int32_t *__restrict__ colind, int base,
                                    int require_sorted, int32_t *__restrict__ stats) {
    // stats[0] = max row length, stats[1] = rows longer than kShortMax,
    // stats[2] = entries in those rows, stats[3] / stats[4] = lower / upper
    // bandwidth (max of row - column / column - row over the entries)
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < m; r += stride) {
        const int64_t lo = (int64_t)rowptr[r] - base, hi = (int64_t)rowptr[r + 1] - base;
        if (r == 0 && lo != 0) atomicOr(&g_validate_flags, 1);
        if (r == m - 1 && hi != nnz) atomicOr(&g_validate_flags, 2);
        if (hi < lo || lo < 0 || hi > nnz) { atomicOr(&g_validate_flags, 4); continue; }
        if (stats) {
            atomicMax(&stats[0], (int32_t)(hi - lo));
            if (hi - lo > kShortMax) {
                atomicAdd(&stats[1], 1);
                atomicAdd(&stats[2], (int32_t)(hi - lo));
            }
        }
        int64_t prev = -1, below = 0, above = 0;
        for (int64_t k = lo; k < hi; ++k) {
            const int64_t c = (int64_t)colind[k] - base;
            if (c < 0 || c >= n) { atomicOr(&g_validate_flags, 8); break; }
            if (require_sorted && c <= prev) { atomicOr(&g_validate_flags, 16); break; }
            prev = c;
            if (r - c > below) below = r - c;
            if (c - r > above) above = c - r;
        }
        if (stats) {
            if (below > 0) atomicMax(&stats[3], (int32_t)(below < INT32_MAX ? below : INT32_MAX));
            if (above > 0) atomicMax(&stats[4], (int32_t)(above < INT32_MAX ? above : INT32_MAX));
        }
    }
}

}  // namespace spmv

// Runs the validation kernel; on success optionally returns (max row length,
// rows longer than kShortMax, entries in them) through stats_host.
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
    if (stats_dev) JLB_CUDA(cudaMemsetAsync(stats_dev, 0, spmv::kValidateStats * sizeof(int32_t), st));
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
        JLB_CUDA(cudaMemcpyAsync(stats_host, stats_dev, spmv::kValidateStats * sizeof(int32_t),
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
        return spmv::launch<double>(as_stream(stream), idx_base, m, nnz, rowptr, colind, val, x,
                                    y, alpha, beta);
    return spmv::launch<float>(as_stream(stream), idx_base, m, nnz, rowptr, colind, val, x, y,
                               alpha, beta);
}

extern "C" JLB_API int jlb_dcsr_spmv(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                     int64_t nfib, int64_t nnz, const int32_t *fibptr,
                                     const int32_t *row_ids, const int32_t *colind,
                                     const void *val, const void *x, void *y, double alpha,
                                     double beta) {
    int st = spmv_args(dtype, idx_base, nfib, n, nnz, fibptr, colind, val, x, y);
    if (st) return st;
    if (m < 0 || nfib > m) return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "more stored rows than rows");
    if (nfib > 0 && !row_ids) return fail(JLB_ERR_INVALID_ARGUMENT, "null row coordinates");
    if (dtype == JLB_F64)
        return spmv::launch_dcsr<double>(as_stream(stream), idx_base, m, nfib, fibptr, row_ids,
                                         colind, val, x, y, alpha, beta);
    return spmv::launch_dcsr<float>(as_stream(stream), idx_base, m, nfib, fibptr, row_ids, colind,
                                    val, x, y, alpha, beta);
}

extern "C" JLB_API int jlb_csr_patched_spmv(void *stream, int dtype, int idx_base, int64_t m,
                                            int64_t n, int64_t nnz, const int32_t *rowptr,
                                            const int32_t *colind, const void *val, int npatch,
                                            const int64_t *patch_rows, const int64_t *patch_cols,
                                            const double *patch_vals, const void *x, void *y,
                                            double alpha, double beta) {
    if (!rowptr && nnz > 0) return fail(JLB_ERR_INVALID_ARGUMENT, "null rowptr with entries");
    static const int32_t no_rows = 0;   // lets a null rowptr pass the common checks
    int st = spmv_args(dtype, idx_base, m, n, nnz, rowptr ? rowptr : &no_rows, colind, val, x, y);
    if (st) return st;
    if (npatch < 0 || (npatch > 0 && (!patch_rows || !patch_cols || !patch_vals)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "bad patch arrays");
    if (npatch > 0 && !x) return fail(JLB_ERR_INVALID_ARGUMENT, "null x");
    if (dtype == JLB_F64)
        return spmv::launch_patched<double>(as_stream(stream), idx_base, m, n, rowptr, colind,
                                            val, npatch, patch_rows, patch_cols, patch_vals, x,
                                            y, alpha, beta);
    return spmv::launch_patched<float>(as_stream(stream), idx_base, m, n, rowptr, colind, val,
                                       npatch, patch_rows, patch_cols, patch_vals, x, y, alpha,
                                       beta);
}

struct jlb_spmv_plan_s {
    int dtype, base;
    int64_t m, n, nnz;
    const int32_t *rowptr, *colind;
    int64_t max_row;
    int64_t long_rows;
    int64_t long_nnz;
    int64_t lbw, ubw;   // lower / upper bandwidth
    int variant;
};

namespace jlb {
namespace spmv {
// Kernel variant from the row-length profile: a thread per row while every
// row is short and rows are short on average (bit-exact with the CPU
// walker), otherwise groups of W lanes per row with W from the mean row
// length (the reference's warp-vector table, KA spmv.jl:296-323, scaled by
// the four entries a lane loads at once).
int choose_variant(int64_t m, int64_t nnz, int64_t max_row, int64_t long_nnz) {
    if (m == 0) return 0;
    const double mean = (double)nnz / (double)m;
    // measured on B200 (fp64): the thread per row wins on regular short rows
    // (5-point Laplacian, bands of 5 and 17 entries) and on power-law rows
    // (its warp path takes the long ones); groups of 4 lanes win on rows of
    // 16 to about 100 entries when no row is long (random columns; bands of
    // 33 and 65 entries: 2.3x and 1.17x variant 0); with longer rows present
    // the two are level on random columns (both bound by the x gathers' L1
    // sector throughput), and variant 0 keeps its bit-exact short rows.
    // Variant 1 (x staged per block of rows) is never picked: it was slower
    // than variant 0 on every banded matrix measured.
    (void)long_nnz;
    if (max_row <= kShortMax && mean <= kScalarMean) return 0;
    if (mean >= kScalarMean && mean < 96.0 && max_row <= 4 * kShortMax) return 4;
    return 0;
}
}  // namespace spmv
}  // namespace jlb

extern "C" JLB_API int jlb_spmv_plan_create(jlb_spmv_plan *plan, void *stream, int dtype,
                                            int idx_base, int64_t m, int64_t n, int64_t nnz,
                                            const int32_t *rowptr, const int32_t *colind) {
    if (!plan) return fail(JLB_ERR_INVALID_ARGUMENT, "null plan out-pointer");
    *plan = nullptr;
    int st = spmv_args(dtype, idx_base, m, n, nnz, rowptr, colind, (const void *)1,
                       (const void *)1, (void *)1);
    if (st) return st;
    int32_t *stats_dev = nullptr;
    JLB_CUDA(cudaMallocAsync((void **)&stats_dev, spmv::kValidateStats * sizeof(int32_t),
                             as_stream(stream)));
    int32_t stats[spmv::kValidateStats] = {0, 0, 0, 0, 0};
    st = csr_validate_impl(as_stream(stream), idx_base, m, n, nnz, rowptr, colind, 0, stats_dev,
                           stats);
    cudaFreeAsync(stats_dev, as_stream(stream));
    if (st) return st;
    jlb_spmv_plan p = new (std::nothrow) jlb_spmv_plan_s;
    if (!p) return fail(JLB_ERR_INVALID_ARGUMENT, "out of host memory");
    p->dtype = dtype; p->base = idx_base; p->m = m; p->n = n; p->nnz = nnz;
    p->rowptr = rowptr; p->colind = colind;
    p->max_row = stats[0];
    p->long_rows = stats[1];
    p->long_nnz = stats[2];
    p->lbw = stats[3];
    p->ubw = stats[4];
    p->variant = spmv::choose_variant(m, nnz, p->max_row, p->long_nnz);
    *plan = p;
    return ok();
}

extern "C" JLB_API int jlb_spmv_plan_set_variant(jlb_spmv_plan p, int variant) {
    if (!p) return fail(JLB_ERR_INVALID_ARGUMENT, "null plan");
    if (variant != 0 && variant != 1 && variant != 2 && variant != 4 && variant != 8 &&
        variant != 16 && variant != 32)
        return fail(JLB_ERR_INVALID_ARGUMENT,
                    "SpMV variant must be 0, 1, 2, 4, 8, 16 or 32 (got %d)", variant);
    p->variant = variant;
    return ok();
}

extern "C" JLB_API int jlb_spmv_plan_execute(jlb_spmv_plan p, void *stream, const void *val,
                                             const void *x, void *y, double alpha, double beta) {
    if (!p) return fail(JLB_ERR_INVALID_ARGUMENT, "null plan");
    int st = spmv_args(p->dtype, p->base, p->m, p->n, p->nnz, p->rowptr, p->colind, val, x, y);
    if (st) return st;
    if (p->dtype == JLB_F64)
        return spmv::launch_variant<double>(as_stream(stream), p->base, p->m, p->nnz, p->rowptr,
                                            p->colind, val, x, y, alpha, beta, p->variant, p->n,
                                            p->lbw, p->ubw);
    return spmv::launch_variant<float>(as_stream(stream), p->base, p->m, p->nnz, p->rowptr,
                                       p->colind, val, x, y, alpha, beta, p->variant, p->n, p->lbw,
                                       p->ubw);
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
