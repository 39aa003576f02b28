// spmm.cu -- CSR SpMM (C = alpha*A*B + beta*C) for sm_100a.
//
// Fast path (B and C row-major, 16-byte aligned rows).  A group of 8 lanes
// holds a 256-byte column chunk of one output row (64 fp32 / 32 fp64 columns):
// each lane owns two 16-byte vectors, so every stored entry of A costs one
// 256-byte gather of a B row in two coalesced 128-byte halves.
//
// The work is bound by how many B-row gathers are in flight, and power-law
// matrices have mostly 1-entry rows, so a group does not work row by row.  It
// owns a contiguous range of rows, balanced by rows + entries (each group
// finds its range with an 8-ary search of the row pointer), and streams
// through the range's entries in storage order with kDepth gathers always in
// flight, across row boundaries: entry i+kDepth is issued while entry i is
// accumulated, and a row's chunk of C is stored when its last entry has been
// added.  Per output element the sum runs over the row's entries in storage
// order with separately rounded products and sums: the same operations as
// JLUST's Tiled SpMM body (ext/KernelAbstractionsExt/ops/spmm.jl:272-292),
// hence bit-identical.  B rows bypass L1 (ld.global.cg); the sequential index
// streams stay in L1.
//
// Rows longer than kLong entries are skipped by the stream and computed by a
// second kernel that splits each into contiguous segments, one per group of a
// CTA, whose partial sums are added in segment order (deterministic, within
// tolerance).  No atomics touch C.
//
// Generic path (any order / alignment): one thread per output element, the
// same storage-order sum.
#include "common.cuh"

namespace jlb {

JLB_DEFINE_DEV_ERROR(spmm)

namespace spmm {

constexpr int kThreads = 256;
constexpr int kGroup = 8;                      // lanes per row
constexpr int kVec = 2;                        // 16-byte vectors per lane per B row
constexpr int kGroups = kThreads / kGroup;     // groups per CTA
constexpr int kLong = 256;                     // longer rows go to spmm_long_rows
constexpr int kDepth = 4;                      // B-row gathers in flight per group
constexpr int kMinWork = 64;                   // rows + entries per group, at least

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

// Columns a lane owns inside a chunk of kGroup*kVec vectors: vector w of lane
// l sits at vector index w*kGroup + l, so each load instruction of the group
// covers kGroup consecutive vectors (128 contiguous bytes).
template <typename T>
struct Lanes {
    static constexpr int E = V16<T>::E;
    static constexpr int CW = kGroup * kVec * E;   // columns per chunk
    __device__ static int64_t col(int64_t c0, int lane, int w) { return c0 + ((int64_t)w * kGroup + lane) * E; }
};

// One in-flight entry: its value and this lane's part of its B row.
template <typename T>
struct Slot {
    T v;
    typename V16<T>::type b[kVec];
};

template <typename T>
__device__ __forceinline__ void issue(Slot<T> &s, int p, const int32_t *__restrict__ colind,
                                      const T *__restrict__ val, const T *__restrict__ B,
                                      int64_t ldb, int64_t c0, int base, int lane,
                                      const bool (&ok)[kVec]) {
    using VT = typename V16<T>::type;
    const int64_t c = (int64_t)(ldg(colind + p) - base);
    s.v = ldg(val + p);
    const T *row = B + c * ldb;
#pragma unroll
    for (int w = 0; w < kVec; ++w)
        if (ok[w]) s.b[w] = __ldcg(reinterpret_cast<const VT *>(row + Lanes<T>::col(c0, lane, w)));
}

template <typename T>
__device__ __forceinline__ void accumulate(T (&acc)[kVec][V16<T>::E], const Slot<T> &s,
                                           const bool (&ok)[kVec]) {
#pragma unroll
    for (int w = 0; w < kVec; ++w)
        if (ok[w]) {
#pragma unroll
            for (int e = 0; e < V16<T>::E; ++e)
                acc[w][e] = add_rn(acc[w][e], mul_rn(s.v, V16<T>::get(s.b[w], e)));
        }
}

// Accumulates entries [lo, hi) of one row, in storage order, into acc for the
// chunk starting at column c0, kDepth gathers in flight.
template <typename T>
__device__ __forceinline__ void range_accumulate(T (&acc)[kVec][V16<T>::E], int lo, int hi,
                                                 const int32_t *__restrict__ colind,
                                                 const T *__restrict__ val,
                                                 const T *__restrict__ B, int64_t ldb,
                                                 int64_t c0, int64_t k, int base, int lane) {
    bool ok[kVec];
#pragma unroll
    for (int w = 0; w < kVec; ++w) ok[w] = Lanes<T>::col(c0, lane, w) < k;
    Slot<T> s[kDepth];
#pragma unroll
    for (int u = 0; u < kDepth; ++u)
        if (lo + u < hi) issue(s[u], lo + u, colind, val, B, ldb, c0, base, lane, ok);
    for (int p = lo; p < hi; p += kDepth) {
#pragma unroll
        for (int u = 0; u < kDepth; ++u) {
            const int q = p + u;
            if (q < hi) {
                accumulate(acc, s[u], ok);
                if (q + kDepth < hi) issue(s[u], q + kDepth, colind, val, B, ldb, c0, base, lane, ok);
            }
        }
    }
}

template <typename T, bool kBeta>
__device__ __forceinline__ void store_chunk(T *C, int64_t ldc, int64_t row, int64_t c0, int64_t k,
                                            const T (&acc)[kVec][V16<T>::E], T alpha, T beta,
                                            int lane) {
    using VT = typename V16<T>::type;
    constexpr int E = V16<T>::E;
#pragma unroll
    for (int w = 0; w < kVec; ++w) {
        const int64_t col = Lanes<T>::col(c0, lane, w);
        if (col >= k) continue;
        VT *dst = reinterpret_cast<VT *>(C + row * ldc + col);
        VT out;
        VT old;
        if (kBeta) old = *dst;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            T o = mul_rn(alpha, acc[w][e]);
            if (kBeta) o = add_rn(o, mul_rn(beta, V16<T>::get(old, e)));
            V16<T>::set(out, e, o);
        }
        *dst = out;
    }
}

template <typename T>
__device__ __forceinline__ void zero(T (&acc)[kVec][V16<T>::E]) {
#pragma unroll
    for (int w = 0; w < kVec; ++w)
#pragma unroll
        for (int e = 0; e < V16<T>::E; ++e) acc[w][e] = T(0);
}

__device__ __forceinline__ unsigned group_mask(int tid) {
    return ((1u << kGroup) - 1u) << ((tid % kWarp) / kGroup * kGroup);
}

// Smallest rows r0, r1 in [0, m] with r + rowptr[r] - base >= t0 (resp. t1):
// both 8-ary searches run together, each lane of the group probing one point
// of each interval per step (about log9(m) dependent loads).
__device__ __forceinline__ void find_rows(int64_t m, const int32_t *__restrict__ rowptr, int base,
                                          int64_t t0, int64_t t1, int lane, unsigned gmask,
                                          int shift, int64_t &r0, int64_t &r1) {
    int64_t lo0 = 0, hi0 = m, lo1 = 0, hi1 = m;
    while (lo0 < hi0 || lo1 < hi1) {
        const int64_t p0 = lo0 + (hi0 - lo0) * (lane + 1) / 9;
        const int64_t p1 = lo1 + (hi1 - lo1) * (lane + 1) / 9;
        const bool q0 = lo0 < hi0 && p0 + (ldg(rowptr + p0) - base) >= t0;
        const bool q1 = lo1 < hi1 && p1 + (ldg(rowptr + p1) - base) >= t1;
        const unsigned b0 = (__ballot_sync(gmask, q0) >> shift) & ((1u << kGroup) - 1u);
        const unsigned b1 = (__ballot_sync(gmask, q1) >> shift) & ((1u << kGroup) - 1u);
        if (lo0 < hi0) {
            const int64_t span = hi0 - lo0;
            if (b0) {
                const int f = __ffs(b0) - 1;
                hi0 = lo0 + span * (f + 1) / 9;
                if (f > 0) lo0 = lo0 + span * f / 9 + 1;
            } else {
                lo0 = lo0 + span * 8 / 9 + 1;
            }
        }
        if (lo1 < hi1) {
            const int64_t span = hi1 - lo1;
            if (b1) {
                const int f = __ffs(b1) - 1;
                hi1 = lo1 + span * (f + 1) / 9;
                if (f > 0) lo1 = lo1 + span * f / 9 + 1;
            } else {
                lo1 = lo1 + span * 8 / 9 + 1;
            }
        }
    }
    r0 = lo0;
    r1 = lo1;
}

// Moves the issue cursor to the first entry of the next row in (r, re) that
// has entries and at most kLong of them; r == re when there is none.  e holds
// the end of row r on entry.
__device__ __forceinline__ void issue_seek(int64_t &r, int &p, int &e, int64_t re,
                                           const int32_t *__restrict__ rowptr, int base) {
    for (;;) {
        if (++r >= re) return;
        const int lo = e;
        e = ldg(rowptr + r + 1) - base;
        if (e > lo && e - lo <= kLong) {
            p = lo;
            return;
        }
    }
}

// Short rows: each group streams through the entries of its row range (rows
// longer than kLong excluded) with kDepth B-row gathers in flight, storing
// each row's chunk of C when its last entry is in, and the chunk of every
// empty row as alpha * 0 (+ beta * C).
template <typename T, bool kBeta>
__global__ void __launch_bounds__(kThreads, 3)
spmm_stream(int64_t m, int64_t k, const int32_t *__restrict__ rowptr,
            const int32_t *__restrict__ colind, const T *__restrict__ val,
            const T *__restrict__ B, int64_t ldb, T *__restrict__ C, int64_t ldc, T alpha, T beta,
            int base) {
    const int tid = threadIdx.x;
    const int lane = tid % kGroup;
    const unsigned gmask = group_mask(tid);
    const int shift = (tid % kWarp) / kGroup * kGroup;
    const int64_t groups = (int64_t)gridDim.x * kGroups;
    const int64_t g = (int64_t)blockIdx.x * kGroups + tid / kGroup;
    const int64_t total = m + (int64_t)(ldg(rowptr + m) - base);
    int64_t rs, re;
    find_rows(m, rowptr, base, total * g / groups, total * (g + 1) / groups, lane, gmask, shift,
              rs, re);
    if (rs >= re) return;
    const int first = ldg(rowptr + rs) - base;

    for (int64_t c0 = 0; c0 < k; c0 += Lanes<T>::CW) {
        bool ok[kVec];
#pragma unroll
        for (int w = 0; w < kVec; ++w) ok[w] = Lanes<T>::col(c0, lane, w) < k;
        T acc[kVec][V16<T>::E];
        zero(acc);

        // consume cursor: row rc, next entry cp, row end ce.  Rows before the
        // first short non-empty one are stored now (empty) or skipped (long).
        int64_t rc = rs - 1;
        int cp = first, ce = first;
        for (;;) {
            if (++rc >= re) break;
            const int lo = ce;
            ce = ldg(rowptr + rc + 1) - base;
            if (ce - lo > kLong || ce < lo) continue;
            if (ce == lo) {
                store_chunk<T, kBeta>(C, ldc, rc, c0, k, acc, alpha, beta, lane);
                continue;
            }
            cp = lo;
            break;
        }
        // issue cursor, kDepth entries ahead of the consume cursor
        int64_t ri = rc;
        int ip = cp, ie = ce;
        Slot<T> s[kDepth];
        bool have[kDepth];
#pragma unroll
        for (int u = 0; u < kDepth; ++u) {
            have[u] = ri < re;
            if (have[u]) {
                issue(s[u], ip, colind, val, B, ldb, c0, base, lane, ok);
                if (++ip >= ie) issue_seek(ri, ip, ie, re, rowptr, base);
            }
        }
        while (have[0]) {
#pragma unroll
            for (int u = 0; u < kDepth; ++u) {
                if (!have[u]) continue;
                accumulate(acc, s[u], ok);
                if (++cp >= ce) {
                    store_chunk<T, kBeta>(C, ldc, rc, c0, k, acc, alpha, beta, lane);
                    zero(acc);
                    for (;;) {
                        if (++rc >= re) break;
                        const int lo = ce;
                        ce = ldg(rowptr + rc + 1) - base;
                        if (ce - lo > kLong || ce < lo) continue;
                        if (ce == lo) {
                            store_chunk<T, kBeta>(C, ldc, rc, c0, k, acc, alpha, beta, lane);
                            continue;
                        }
                        cp = lo;
                        break;
                    }
                }
                have[u] = ri < re;
                if (have[u]) {
                    issue(s[u], ip, colind, val, B, ldb, c0, base, lane, ok);
                    if (++ip >= ie) issue_seek(ri, ip, ie, re, rowptr, base);
                }
            }
        }
    }
}

template <typename T, bool kBeta>
int stream_grid() {
    static int per_sm = 0, sms = 0;
    if (!per_sm) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, spmm_stream<T, kBeta>, kThreads, 0) != cudaSuccess ||
            per_sm < 1) {
            per_sm = 1;
            sms = 148;
        }
    }
    return per_sm * sms;
}

constexpr int kScanRows = 4096;   // rows a long-row CTA inspects

// Long rows: each CTA inspects kScanRows rows and computes every row longer
// than kLong with all of its groups, one contiguous segment each, the partial
// sums added in segment order (deterministic).
template <typename T, bool kBeta>
__global__ void __launch_bounds__(kThreads)
spmm_long_rows(int64_t m, int64_t k, const int32_t *__restrict__ rowptr,
               const int32_t *__restrict__ colind, const T *__restrict__ val,
               const T *__restrict__ B, int64_t ldb, T *__restrict__ C, int64_t ldc, T alpha,
               T beta, int base) {
    constexpr int E = V16<T>::E;
    __shared__ int64_t s_long[kScanRows];
    __shared__ int s_nlong;
    __shared__ T s_part[kGroups][kVec * kGroup * E];
    const int tid = threadIdx.x;
    const int g = tid / kGroup, lane = tid % kGroup;
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
        for (int64_t c0 = 0; c0 < k; c0 += Lanes<T>::CW) {
            T acc[kVec][E];
            zero(acc);
            range_accumulate<T>(acc, slo, shi, colind, val, B, ldb, c0, k, base, lane);
#pragma unroll
            for (int w = 0; w < kVec; ++w)
#pragma unroll
                for (int e = 0; e < E; ++e) s_part[g][(w * kGroup + lane) * E + e] = acc[w][e];
            __syncthreads();
            if (g == 0) {
                T tot[kVec][E];
#pragma unroll
                for (int w = 0; w < kVec; ++w)
#pragma unroll
                    for (int e = 0; e < E; ++e) {
                        const int idx = (w * kGroup + lane) * E + e;
                        tot[w][e] = s_part[0][idx];
                        for (int q = 1; q < kGroups; ++q) tot[w][e] = add_rn(tot[w][e], s_part[q][idx]);
                    }
                store_chunk<T, kBeta>(C, ldc, r, c0, k, tot, alpha, beta, lane);
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
int launch(cudaStream_t st, int base, int64_t m, int64_t nnz, int64_t k, const int32_t *rowptr,
           const int32_t *colind, const void *val, const void *B, int64_t ldb, int b_order,
           void *C, int64_t ldc, int c_order, double alpha, double beta) {
    if (m == 0 || k == 0) return ok();
    constexpr int E = V16<T>::E;
    const T a = (T)alpha, b = (T)beta;
    const bool fast = b_order == JLB_ROW_MAJOR && c_order == JLB_ROW_MAJOR && k % E == 0 &&
                      ldb % E == 0 && ldc % E == 0 && aligned16(B) && aligned16(C);
    if (fast) {
        const unsigned grid_long = (unsigned)ceil_div(m, kScanRows);
        const int64_t need = ceil_div(m + nnz, (int64_t)kGroups * kMinWork);
        if (b == T(0)) {
            const int64_t full = stream_grid<T, false>();
            spmm_stream<T, false><<<(unsigned)(need < full ? need : full), kThreads, 0, st>>>(
                m, k, rowptr, colind, (const T *)val, (const T *)B, ldb, (T *)C, ldc, a, b, base);
            spmm_long_rows<T, false><<<grid_long, kThreads, 0, st>>>(
                m, k, rowptr, colind, (const T *)val, (const T *)B, ldb, (T *)C, ldc, a, b, base);
        } else {
            const int64_t full = stream_grid<T, true>();
            spmm_stream<T, true><<<(unsigned)(need < full ? need : full), kThreads, 0, st>>>(
                m, k, rowptr, colind, (const T *)val, (const T *)B, ldb, (T *)C, ldc, a, b, base);
            spmm_long_rows<T, true><<<grid_long, kThreads, 0, st>>>(
                m, k, rowptr, colind, (const T *)val, (const T *)B, ldb, (T *)C, ldc, a, b, base);
        }
        JLB_LAUNCH_CHECK("spmm_stream");
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
        return spmm::launch<double>(as_stream(stream), idx_base, m, nnz, k, rowptr, colind, val, B, ldb,
                                    b_order, C, ldc, c_order, alpha, beta);
    return spmm::launch<float>(as_stream(stream), idx_base, m, nnz, k, rowptr, colind, val, B, ldb,
                               b_order, C, ldc, c_order, alpha, beta);
}
