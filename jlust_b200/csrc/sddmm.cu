// sddmm.cu -- sampled dense-dense product over a CSR pattern, sm_100a.
//
// Fast path (A row-major with 16-byte aligned rows, or column-major as
// Julia stores it; the K x n operand B stored with each column j contiguous
// -- Julia's column-major K x n, or a row-major n x K array -- with 16-byte
// aligned columns): one warp per pattern row i keeps A(i, :) in registers (16 bytes per
// lane per 32*16-byte chunk of K); every stored position (i, j) costs one
// coalesced read of B(:, j) and a fixed-order warp reduction.  Positions are
// processed four at a time so four B columns are in flight per warp.  Results
// are written back 32 positions at a time, coalesced.
//
// Generic path (any layouts): one warp per row, one lane per stored position,
// each lane summing k = 0..K-1 in order with separately rounded products and
// sums -- the operations of JLUST's SDDMM leaf (KA sddmm.jl:23-36).
#include "common.cuh"

namespace jlb {

JLB_DEFINE_DEV_ERROR(sddmm)

namespace sddmm {

constexpr int kThreads = 256;

template <typename T>
struct V16;
template <>
struct V16<float> {
    using type = float4;
    static constexpr int E = 4;
    __device__ static float dot(const float4 &a, const float4 &b) {
        float s = mul_rn(a.x, b.x);
        s = add_rn(s, mul_rn(a.y, b.y));
        s = add_rn(s, mul_rn(a.z, b.z));
        return add_rn(s, mul_rn(a.w, b.w));
    }
};
template <>
struct V16<double> {
    using type = double2;
    static constexpr int E = 2;
    __device__ static double dot(const double2 &a, const double2 &b) {
        return add_rn(mul_rn(a.x, b.x), mul_rn(a.y, b.y));
    }
};

template <typename T>
__device__ __forceinline__ T finish(T dot, T s, T old, T alpha, T beta, int mode, bool has_beta) {
    T o = mul_rn(alpha, dot);
    if (mode == JLB_SDDMM_MUL) o = mul_rn(o, s);
    if (has_beta) o = add_rn(o, mul_rn(beta, old));
    return o;
}

// A(i, kk .. kk+E-1) as one vector: a 16-byte load of a row-major A, or E
// scalar loads of a column-major A (Julia's layout, element (i, kk) at
// i + kk*lda).  Consecutive rows go to the warps of one CTA, so the 32-byte
// sectors of a column-major A are shared by eight neighbouring rows in L1.
template <typename T, bool kColA>
__device__ __forceinline__ typename V16<T>::type load_a(const T *__restrict__ A, int64_t lda,
                                                        int64_t i, int64_t kk) {
    using VT = typename V16<T>::type;
    if (!kColA) return __ldcs(reinterpret_cast<const VT *>(A + i * lda + kk));
    T e[V16<T>::E];
#pragma unroll
    for (int u = 0; u < V16<T>::E; ++u) e[u] = __ldg(A + i + (kk + u) * lda);
    if constexpr (V16<T>::E == 4) return make_float4(e[0], e[1], e[2], e[3]);
    else return make_double2(e[0], e[1]);
}

template <typename T, int NC, bool kColA>
__global__ void __launch_bounds__(kThreads)
sddmm_fast(int64_t m, int64_t K, const int32_t *__restrict__ rowptr,
           const int32_t *__restrict__ colind, const T *__restrict__ A, int64_t lda,
           const T *__restrict__ B, int64_t ldb, const T *__restrict__ S, T *__restrict__ out,
           int mode, T alpha, T beta, int has_beta, int base) {
    using VT = typename V16<T>::type;
    constexpr int E = V16<T>::E;
    constexpr int CW = kWarp * E;
    const int lane = threadIdx.x % kWarp;
    const int64_t warps = (int64_t)gridDim.x * (kThreads / kWarp);
    for (int64_t i = (int64_t)blockIdx.x * (kThreads / kWarp) + threadIdx.x / kWarp; i < m; i += warps) {
        VT a[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int64_t kk = (int64_t)c * CW + (int64_t)lane * E;
            if (kk < K) a[c] = load_a<T, kColA>(A, lda, i, kk);
        }
        const int lo = rowptr[i] - base, hi = rowptr[i + 1] - base;
        for (int pb = lo; pb < hi; pb += kWarp) {
            const int mp = pb + lane;
            int32_t mc = 0;
            if (mp < hi) mc = __ldcs(colind + mp) - base;
            const int n = (hi - pb) < kWarp ? (hi - pb) : kWarp;
            T mine = T(0);
            int j = 0;
            for (; j + 4 <= n; j += 4) {
                T part[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int64_t cj = __shfl_sync(0xffffffffu, mc, j + u);
                    part[u] = T(0);
#pragma unroll
                    for (int c = 0; c < NC; ++c) {
                        const int64_t kk = (int64_t)c * CW + (int64_t)lane * E;
                        if (kk < K) {
                            const VT b = __ldg(reinterpret_cast<const VT *>(B + cj * ldb + kk));
                            part[u] = add_rn(part[u], V16<T>::dot(a[c], b));
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const T d = warp_sum(part[u]);
                    if (lane == j + u) mine = d;
                }
            }
            for (; j < n; ++j) {
                const int64_t cj = __shfl_sync(0xffffffffu, mc, j);
                T part = T(0);
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const int64_t kk = (int64_t)c * CW + (int64_t)lane * E;
                    if (kk < K) {
                        const VT b = __ldg(reinterpret_cast<const VT *>(B + cj * ldb + kk));
                        part = add_rn(part, V16<T>::dot(a[c], b));
                    }
                }
                const T d = warp_sum(part);
                if (lane == j) mine = d;
            }
            if (mp < hi) {
                const T s = (mode == JLB_SDDMM_MUL) ? __ldcs(S + mp) : T(0);
                const T old = has_beta ? out[mp] : T(0);
                out[mp] = finish(mine, s, old, alpha, beta, mode, has_beta != 0);
            }
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
sddmm_generic(int64_t m, int64_t K, const int32_t *__restrict__ rowptr,
              const int32_t *__restrict__ colind, const T *__restrict__ A, int64_t lda,
              int a_order, const T *__restrict__ B, int64_t ldb, int b_order,
              const T *__restrict__ S, T *__restrict__ out, int mode, T alpha, T beta,
              int has_beta, int base) {
    const int lane = threadIdx.x % kWarp;
    const int64_t warps = (int64_t)gridDim.x * (kThreads / kWarp);
    for (int64_t i = (int64_t)blockIdx.x * (kThreads / kWarp) + threadIdx.x / kWarp; i < m; i += warps) {
        const int lo = rowptr[i] - base, hi = rowptr[i + 1] - base;
        for (int p = lo + lane; p < hi; p += kWarp) {
            const int64_t j = (int64_t)colind[p] - base;
            T dot = T(0);
            for (int64_t kk = 0; kk < K; ++kk) {
                const T av = a_order == JLB_ROW_MAJOR ? ldg(A + i * lda + kk) : ldg(A + i + kk * lda);
                const T bv = b_order == JLB_ROW_MAJOR ? ldg(B + kk * ldb + j) : ldg(B + kk + j * ldb);
                dot = add_rn(dot, mul_rn(av, bv));
            }
            const T s = (mode == JLB_SDDMM_MUL) ? S[p] : T(0);
            const T old = has_beta ? out[p] : T(0);
            out[p] = finish(dot, s, old, alpha, beta, mode, has_beta != 0);
        }
    }
}

template <typename T>
int launch(cudaStream_t st, int base, int64_t m, int64_t K, const int32_t *rowptr,
           const int32_t *colind, const void *A, int64_t lda, int a_order, const void *B,
           int64_t ldb, int b_order, const void *S, void *out, int mode, double alpha,
           double beta) {
    if (m == 0) return ok();
    constexpr int E = V16<T>::E;
    constexpr int CW = kWarp * E;
    const T a = (T)alpha, b = (T)beta;
    const int has_beta = b != T(0);
    const int64_t warps_needed = m;
    const unsigned grid = (unsigned)(ceil_div(warps_needed, kThreads / kWarp) < 148 * 64
                                         ? ceil_div(warps_needed, kThreads / kWarp)
                                         : 148 * 64);
    const int nc = (int)ceil_div(K, CW);
    // B(:, j) contiguous (the K x n operand column-major: JLUST's native
    // layout, or a row-major n x K array); A row-major or column-major
    const bool a_fast = (a_order == JLB_ROW_MAJOR && lda % E == 0 && aligned16(A)) ||
                        a_order == JLB_COL_MAJOR;
    const bool fast = a_fast && b_order == JLB_COL_MAJOR && K % E == 0 && ldb % E == 0 &&
                      aligned16(B) && nc >= 1 && nc <= 4;
#define JLB_SDDMM_FAST(NC, CA)                                                                 \
    sddmm_fast<T, NC, CA><<<grid, kThreads, 0, st>>>(m, K, rowptr, colind, (const T *)A, lda,  \
                                                     (const T *)B, ldb, (const T *)S,          \
                                                     (T *)out, mode, a, b, has_beta, base)
    if (fast && a_order == JLB_ROW_MAJOR) {
        switch (nc) {
            case 1: JLB_SDDMM_FAST(1, false); break;
            case 2: JLB_SDDMM_FAST(2, false); break;
            case 3: JLB_SDDMM_FAST(3, false); break;
            default: JLB_SDDMM_FAST(4, false); break;
        }
        JLB_LAUNCH_CHECK("sddmm_fast");
    } else if (fast) {
        switch (nc) {
            case 1: JLB_SDDMM_FAST(1, true); break;
            case 2: JLB_SDDMM_FAST(2, true); break;
            case 3: JLB_SDDMM_FAST(3, true); break;
            default: JLB_SDDMM_FAST(4, true); break;
        }
        JLB_LAUNCH_CHECK("sddmm_fast (column-major A)");
    } else {
        sddmm_generic<T><<<grid, kThreads, 0, st>>>(m, K, rowptr, colind, (const T *)A, lda,
                                                    a_order, (const T *)B, ldb, b_order,
                                                    (const T *)S, (T *)out, mode, a, b,
                                                    has_beta, base);
        JLB_LAUNCH_CHECK("sddmm_generic");
    }
#undef JLB_SDDMM_FAST
    return ok();
}

}  // namespace sddmm
}  // namespace jlb

using namespace jlb;

extern "C" JLB_API int jlb_sddmm(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                 int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                                 int64_t K, const void *A, int64_t lda, int a_order,
                                 const void *B, int64_t ldb, int b_order, const void *S,
                                 void *out, int mode, double alpha, double beta) {
    if (dtype != JLB_F32 && dtype != JLB_F64)
        return fail(JLB_ERR_UNSUPPORTED_VALUE_TYPE, "SDDMM supports Float32 and Float64 (dtype %d)", dtype);
    if (idx_base != 0 && idx_base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (mode != JLB_SDDMM_ADD && mode != JLB_SDDMM_MUL) return fail(JLB_ERR_INVALID_ARGUMENT, "bad SDDMM mode %d", mode);
    if (m < 0 || n < 0 || nnz < 0 || K < 0) return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "negative extent");
    if (nnz > INT32_MAX - 1) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "nnz exceeds Int32 positions");
    if ((a_order != JLB_ROW_MAJOR && a_order != JLB_COL_MAJOR) ||
        (b_order != JLB_ROW_MAJOR && b_order != JLB_COL_MAJOR))
        return fail(JLB_ERR_INVALID_ARGUMENT, "order must be JLB_ROW_MAJOR or JLB_COL_MAJOR");
    if (lda < (a_order == JLB_ROW_MAJOR ? K : m) || ldb < (b_order == JLB_ROW_MAJOR ? n : K))
        return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "leading dimension smaller than the operand");
    if (m > 0 && !rowptr) return fail(JLB_ERR_INVALID_ARGUMENT, "null rowptr");
    if (nnz > 0 && (!colind || !out || (K > 0 && (!A || !B)) || (mode == JLB_SDDMM_MUL && !S)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null colind, A, B, S or out");
    if (dtype == JLB_F64)
        return sddmm::launch<double>(as_stream(stream), idx_base, m, K, rowptr, colind, A, lda,
                                     a_order, B, ldb, b_order, S, out, mode, alpha, beta);
    return sddmm::launch<float>(as_stream(stream), idx_base, m, K, rowptr, colind, A, lda,
                                a_order, B, ldb, b_order, S, out, mode, alpha, beta);
}
