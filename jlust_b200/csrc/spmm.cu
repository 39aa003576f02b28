// spmm.cu -- CSR SpMM (C = alpha*A*B + beta*C) for sm_100a.
//
// Fast path (B and C row-major, 16-byte aligned rows): a group of 16 lanes
// owns one output row; each lane owns 16 bytes of every 16*16-byte column
// chunk of C (64 fp32 / 32 fp64 columns), so every stored entry of A costs one
// coalesced 256-byte read of a B row.  The group loads 16 (column, value)
// pairs at a time and broadcasts them with shuffles.  Per output element the
// sum runs over the row's entries in storage order with separately rounded
// products and sums: the same operations as JLUST's Tiled SpMM body
// (ext/KernelAbstractionsExt/ops/spmm.jl:272-292), hence bit-identical.
// Groups run independently (no block barriers), one row each.  Rows longer
// than kLong entries go to a second kernel that splits each into 16
// contiguous segments, one per group of a CTA, whose partial sums are added
// in segment order (deterministic, within tolerance).  No atomics touch C.
//
// Generic path (any order / alignment): one thread per output element, the
// same storage-order sum.
#include "common.cuh"

namespace jlb {

JLB_DEFINE_DEV_ERROR(spmm)

namespace spmm {

constexpr int kThreads = 256;
constexpr int kGroup = 16;                     // lanes per row
constexpr int kGroups = kThreads / kGroup;     // rows in flight per CTA
constexpr int kLong = 256;                     // longer rows use the whole CTA

template <typename T>
struct V16;
template <>
struct V16<float> {
    using type = float4;
    static constexpr int E = 4;
    __device__ static float get(const float4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
    __device__ static void set(float4 &v, int i, float x) { if (i == 0) v.x = x; else if (i == 1) v.y = x; else if (i == 2) v.z = x; else v.w = x; }
};
template <>
struct V16<double> {
    using type = double2;
    static constexpr int E = 2;
    __device__ static double get(const double2 &v, int i) { return i == 0 ? v.x : v.y; }
    __device__ static void set(double2 &v, int i, double x) { if (i == 0) v.x = x; else v.y = x; }
};

// Accumulates, for one output row and one column chunk, the entries [lo, hi)
// in storage order into acc[E].  `lane` is the lane within the 16-lane group;
// `width_ok` says whether this lane's columns lie inside k.
template <typename T>
__device__ __forceinline__ void group_accumulate(T (&acc)[V16<T>::E], int lo, int hi,
                                                 const int32_t *__restrict__ colind,
                                                 const T *__restrict__ val,
                                                 const T *__restrict__ B, int64_t ldb,
                                                 int64_t col0, bool width_ok, int base,
                                                 unsigned gmask, int lane) {
    using VT = typename V16<T>::type;
    constexpr int E = V16<T>::E;
    for (int kb = lo; kb < hi; kb += kGroup) {
        const int mk = kb + lane;
        int32_t mc = 0;
        T mv = T(0);
        if (mk < hi) {
            mc = __ldcs(colind + mk) - base;
            mv = __ldcs(val + mk);
        }
        const int n = (hi - kb) < kGroup ? (hi - kb) : kGroup;
        int j = 0;
        for (; j + 4 <= n; j += 4) {
            int32_t c[4];
            T v[4];
            VT b[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                c[u] = __shfl_sync(gmask, mc, j + u, kGroup);
                v[u] = __shfl_sync(gmask, mv, j + u, kGroup);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (width_ok) b[u] = __ldg(reinterpret_cast<const VT *>(B + (int64_t)c[u] * ldb + col0));
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (width_ok) {
#pragma unroll
                    for (int e = 0; e < E; ++e) acc[e] = add_rn(acc[e], mul_rn(v[u], V16<T>::get(b[u], e)));
                }
        }
        for (; j < n; ++j) {
            const int32_t c = __shfl_sync(gmask, mc, j, kGroup);
            const T v = __shfl_sync(gmask, mv, j, kGroup);
            if (width_ok) {
                const VT b = __ldg(reinterpret_cast<const VT *>(B + (int64_t)c * ldb + col0));
#pragma unroll
                for (int e = 0; e < E; ++e) acc[e] = add_rn(acc[e], mul_rn(v, V16<T>::get(b, e)));
            }
        }
    }
}

template <typename T, bool kBeta>
__device__ __forceinline__ void store_chunk(T *C, int64_t ldc, int64_t row, int64_t col0,
                                            const T (&acc)[V16<T>::E], T alpha, T beta) {
    using VT = typename V16<T>::type;
    constexpr int E = V16<T>::E;
    VT *dst = reinterpret_cast<VT *>(C + row * ldc + col0);
    VT out;
    VT old;
    if (kBeta) old = *dst;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        T o = mul_rn(alpha, acc[e]);
        if (kBeta) o = add_rn(o, mul_rn(beta, V16<T>::get(old, e)));
        V16<T>::set(out, e, o);
    }
    *dst = out;
}

// Short rows: one 16-lane group per row, no block-level synchronisation
// (rows of a power-law matrix differ widely in length, and a barrier would
// make every group of a CTA wait for its slowest row).  Rows longer than
// kLong are left to spmm_long_rows.
template <typename T, bool kBeta>
__global__ void __launch_bounds__(kThreads)
spmm_rowmajor(int64_t m, int64_t k, const int32_t *__restrict__ rowptr,
              const int32_t *__restrict__ colind, const T *__restrict__ val,
              const T *__restrict__ B, int64_t ldb, T *__restrict__ C, int64_t ldc, T alpha,
              T beta, int base) {
    constexpr int E = V16<T>::E;
    constexpr int CW = kGroup * E;  // columns per chunk
    const int tid = threadIdx.x;
    const int lane = tid % kGroup;
    const unsigned gmask = (tid % kWarp < kGroup) ? 0x0000ffffu : 0xffff0000u;
    const int64_t r = (int64_t)blockIdx.x * kGroups + tid / kGroup;
    if (r >= m) return;
    const int lo = ldg(rowptr + r) - base, hi = ldg(rowptr + r + 1) - base;
    if (hi - lo > kLong) return;
    for (int64_t c0 = 0; c0 < k; c0 += CW) {
        const int64_t col0 = c0 + (int64_t)lane * E;
        const bool width_ok = col0 < k;
        T acc[E];
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] = T(0);
        group_accumulate<T>(acc, lo, hi, colind, val, B, ldb, col0, width_ok, base, gmask, lane);
        if (width_ok) store_chunk<T, kBeta>(C, ldc, r, col0, acc, alpha, beta);
    }
}

constexpr int kScanRows = 4096;   // rows a long-row CTA inspects

// Long rows: each CTA inspects kScanRows rows and computes every row longer
// than kLong with all 16 groups, one contiguous segment each, the partial
// sums added in segment order (deterministic).
template <typename T, bool kBeta>
__global__ void __launch_bounds__(kThreads)
spmm_long_rows(int64_t m, int64_t k, const int32_t *__restrict__ rowptr,
               const int32_t *__restrict__ colind, const T *__restrict__ val,
               const T *__restrict__ B, int64_t ldb, T *__restrict__ C, int64_t ldc, T alpha,
               T beta, int base) {
    constexpr int E = V16<T>::E;
    constexpr int CW = kGroup * E;
    __shared__ int64_t s_long[kScanRows];
    __shared__ int s_nlong;
    __shared__ T s_part[kGroups][CW];
    const int tid = threadIdx.x;
    const int g = tid / kGroup, lane = tid % kGroup;
    const unsigned gmask = (tid % kWarp < kGroup) ? 0x0000ffffu : 0xffff0000u;
    const int64_t r0 = (int64_t)blockIdx.x * kScanRows;
    if (tid == 0) s_nlong = 0;
    __syncthreads();
    for (int i = tid; i < kScanRows && r0 + i < m; i += kThreads) {
        const int64_t r = r0 + i;
        if (ldg(rowptr + r + 1) - ldg(rowptr + r) > kLong) s_long[atomicAdd(&s_nlong, 1)] = r;
    }
    __syncthreads();
    for (int i = 0; i < s_nlong; ++i) {
        const int64_t r = s_long[i];
        const int lo = ldg(rowptr + r) - base, hi = ldg(rowptr + r + 1) - base;
        const int seg = (hi - lo + kGroups - 1) / kGroups;
        const int slo = lo + g * seg < hi ? lo + g * seg : hi;
        const int shi = slo + seg < hi ? slo + seg : hi;
        for (int64_t c0 = 0; c0 < k; c0 += CW) {
            const int64_t col0 = c0 + (int64_t)lane * E;
            const bool width_ok = col0 < k;
            T acc[E];
#pragma unroll
            for (int e = 0; e < E; ++e) acc[e] = T(0);
            group_accumulate<T>(acc, slo, shi, colind, val, B, ldb, col0, width_ok, base, gmask, lane);
#pragma unroll
            for (int e = 0; e < E; ++e) s_part[g][lane * E + e] = acc[e];
            __syncthreads();
            if (g == 0 && width_ok) {
                T tot[E];
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    tot[e] = s_part[0][lane * E + e];
                    for (int q = 1; q < kGroups; ++q) tot[e] = add_rn(tot[e], s_part[q][lane * E + e]);
                }
                store_chunk<T, kBeta>(C, ldc, r, col0, tot, alpha, beta);
            }
            __syncthreads();
        }
    }
}

// Generic layouts: one thread per output element.
template <typename T>
__global__ void spmm_generic(int64_t m, int64_t k, const int32_t *__restrict__ rowptr,
                             const int32_t *__restrict__ colind, const T *__restrict__ val,
                             const T *__restrict__ B, int64_t ldb, int b_order,
                             T *__restrict__ C, int64_t ldc, int c_order, T alpha, T beta,
                             int base, int has_beta) {
    const int64_t total = m * k;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        int64_t r, t;
        if (c_order == JLB_ROW_MAJOR) { r = idx / k; t = idx % k; }
        else { t = idx / m; r = idx % m; }
        const int lo = rowptr[r] - base, hi = rowptr[r + 1] - base;
        T acc = T(0);
        for (int p = lo; p < hi; ++p) {
            const int64_t c = (int64_t)ldg(colind + p) - base;
            const T bv = b_order == JLB_ROW_MAJOR ? ldg(B + c * ldb + t) : ldg(B + c + t * ldb);
            acc = add_rn(acc, mul_rn(ldg(val + p), bv));
        }
        T *dst = c_order == JLB_ROW_MAJOR ? C + r * ldc + t : C + r + t * ldc;
        T o = mul_rn(alpha, acc);
        if (has_beta) o = add_rn(o, mul_rn(beta, *dst));
        *dst = o;
    }
}

template <typename T>
int launch(cudaStream_t st, int base, int64_t m, int64_t k, const int32_t *rowptr,
           const int32_t *colind, const void *val, const void *B, int64_t ldb, int b_order,
           void *C, int64_t ldc, int c_order, double alpha, double beta) {
    if (m == 0 || k == 0) return ok();
    constexpr int E = V16<T>::E;
    const T a = (T)alpha, b = (T)beta;
    const bool fast = b_order == JLB_ROW_MAJOR && c_order == JLB_ROW_MAJOR && k % E == 0 &&
                      ldb % E == 0 && ldc % E == 0 && aligned16(B) && aligned16(C);
    if (fast) {
        const unsigned grid = (unsigned)ceil_div(m, kGroups);
        const unsigned grid_long = (unsigned)ceil_div(m, kScanRows);
        if (b == T(0)) {
            spmm_rowmajor<T, false><<<grid, kThreads, 0, st>>>(m, k, rowptr, colind, (const T *)val,
                                                               (const T *)B, ldb, (T *)C, ldc, a, b, base);
            spmm_long_rows<T, false><<<grid_long, kThreads, 0, st>>>(
                m, k, rowptr, colind, (const T *)val, (const T *)B, ldb, (T *)C, ldc, a, b, base);
        } else {
            spmm_rowmajor<T, true><<<grid, kThreads, 0, st>>>(m, k, rowptr, colind, (const T *)val,
                                                              (const T *)B, ldb, (T *)C, ldc, a, b, base);
            spmm_long_rows<T, true><<<grid_long, kThreads, 0, st>>>(
                m, k, rowptr, colind, (const T *)val, (const T *)B, ldb, (T *)C, ldc, a, b, base);
        }
        JLB_LAUNCH_CHECK("spmm_rowmajor");
    } else {
        const int64_t total = m * k;
        const unsigned grid = (unsigned)(ceil_div(total, 256) < 148 * 32 ? ceil_div(total, 256) : 148 * 32);
        spmm_generic<T><<<grid, 256, 0, st>>>(m, k, rowptr, colind, (const T *)val, (const T *)B,
                                              ldb, b_order, (T *)C, ldc, c_order, a, b, base,
                                              b != T(0));
        JLB_LAUNCH_CHECK("spmm_generic");
    }
    return ok();
}

}  // namespace spmm
}  // namespace jlb

using namespace jlb;

extern "C" JLB_API int jlb_csr_spmm(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                    int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                                    const void *val, int64_t k, const void *B, int64_t ldb,
                                    int b_order, void *C, int64_t ldc, int c_order, double alpha,
                                    double beta) {
    if (dtype != JLB_F32 && dtype != JLB_F64)
        return fail(JLB_ERR_UNSUPPORTED_VALUE_TYPE, "SpMM supports Float32 and Float64 (dtype %d)", dtype);
    if (idx_base != 0 && idx_base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (m < 0 || n < 0 || nnz < 0 || k < 0) return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "negative extent");
    if (nnz > INT32_MAX - 1) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "nnz exceeds Int32 positions");
    if ((b_order != JLB_ROW_MAJOR && b_order != JLB_COL_MAJOR) ||
        (c_order != JLB_ROW_MAJOR && c_order != JLB_COL_MAJOR))
        return fail(JLB_ERR_INVALID_ARGUMENT, "order must be JLB_ROW_MAJOR or JLB_COL_MAJOR");
    if (ldb < (b_order == JLB_ROW_MAJOR ? k : n) || ldc < (c_order == JLB_ROW_MAJOR ? k : m))
        return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "leading dimension smaller than the operand");
    if (m > 0 && k > 0 && (!rowptr || !C)) return fail(JLB_ERR_INVALID_ARGUMENT, "null rowptr or C");
    if (nnz > 0 && k > 0 && (!colind || !val || !B)) return fail(JLB_ERR_INVALID_ARGUMENT, "null colind, val or B");
    if (dtype == JLB_F64)
        return spmm::launch<double>(as_stream(stream), idx_base, m, k, rowptr, colind, val, B, ldb,
                                    b_order, C, ldc, c_order, alpha, beta);
    return spmm::launch<float>(as_stream(stream), idx_base, m, k, rowptr, colind, val, B, ldb,
                               b_order, C, ldc, c_order, alpha, beta);
}
