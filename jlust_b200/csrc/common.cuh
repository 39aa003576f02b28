// common.cuh -- helpers shared by the translation units of libjlust_b200.so.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdarg.h>

#include "../../include/jlust_b200.h"

namespace jlb {

// ---------------------------------------------------------------- host errors
// Records `status` and a formatted message as the calling thread's last error
// (implemented in api.cu) and returns `status`, so call sites can write
// `return fail(JLB_ERR_..., "...")`.
int fail(int status, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int ok();  // clears the thread's last error, returns JLB_OK

// Checks a CUDA runtime result; on failure records JLB_ERR_CUDA with the
// CUDA error string and the call site.
int cuda_check(cudaError_t e, const char *what);

#define JLB_CUDA(call)                                              \
    do {                                                            \
        cudaError_t _e = (call);                                    \
        if (_e != cudaSuccess) return ::jlb::cuda_check(_e, #call); \
    } while (0)

#define JLB_LAUNCH_CHECK(what)                                       \
    do {                                                             \
        cudaError_t _e = cudaGetLastError();                         \
        if (_e != cudaSuccess) return ::jlb::cuda_check(_e, what);   \
    } while (0)

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

inline size_t dtype_size(int dtype) {
    return dtype == JLB_F64 ? 8 : dtype == JLB_F32 ? 4 : dtype == JLB_BF16 ? 2 : 0;
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------ device errors
// Kernels report a bounded wait that gave up, or a bounds check that failed,
// by OR-ing a bit into a per-translation-unit device word.  The host reads and
// clears every unit's word in jlb_device_status().
enum DevErr : int {
    DEV_ERR_TIMEOUT = 1,      // an mbarrier / flag wait exceeded its limit
    DEV_ERR_BOUNDS = 2,       // an index outside the declared extents
    DEV_ERR_OVERFLOW = 4,     // an int32 position buffer overflowed
    DEV_ERR_ORDER = 8,        // coordinates out of the order the format declares
};

// Per-unit accessors, defined once per .cu file by JLB_DEFINE_DEV_ERROR.
int take_dev_error_spmv();
int take_dev_error_spmm();
int take_dev_error_sddmm();
int take_dev_error_bsr();
int take_dev_error_convert();
int take_dev_error_halo();
int take_dev_error_spmvfmt();
int take_dev_error_bbm();
int take_dev_error_spgemm();

#define JLB_DEFINE_DEV_ERROR(unit)                                           \
    static __device__ int g_dev_error;                                       \
    __device__ __forceinline__ void dev_error(int bit) {                     \
        atomicOr(&g_dev_error, bit);                                         \
    }                                                                        \
    int take_dev_error_##unit() {                                            \
        int v = 0;                                                           \
        if (cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int)) != cudaSuccess) \
            return -1;                                                       \
        if (v) {                                                             \
            int z = 0;                                                       \
            if (cudaMemcpyToSymbol(g_dev_error, &z, sizeof(int)) != cudaSuccess) \
                return -1;                                                   \
        }                                                                    \
        return v;                                                            \
    }

// ------------------------------------------------------ exact arithmetic ops
// Separately rounded multiply and add.  nvcc contracts a*b + c into an FMA
// unless told otherwise; these intrinsics are never contracted, which keeps
// the kernels bit-identical to the reference's uncontracted sums.
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

template <typename T>
__device__ __forceinline__ T ldg(const T *p) { return __ldg(p); }

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
    return __uint_as_float(((uint32_t)h) << 16);
}

// Warp sum with a fixed xor-butterfly order (deterministic for a given
// assignment of values to lanes).
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = add_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

constexpr int kWarp = 32;

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

namespace conv {
// Exclusive scan of n int32 counts into out[0..n] (out[0] = base), with a
// workspace of scan_ws(n) bytes (convert.cu).
size_t scan_ws(int64_t n);
int scan(cudaStream_t st, int64_t n, const int32_t *counts, int32_t *out, int base, void *ws,
         size_t ws_bytes);
}  // namespace conv

// Sum over selector patches of row r in patch order, from zero: patch p
// covers rows rows[2p] .. rows[2p+1] (inclusive) and adds
// vals[p] * x[col_off + r - rows[2p] + cols[p]] (JLUST's _apply_patches,
// ext/KernelAbstractionsExt/ops/block_periodic.jl:39-49).  A column outside
// [0, n) is skipped and sets bad.
template <typename T>
__device__ __forceinline__ T patch_sum(int64_t r, int npatch, const int64_t *__restrict__ rows,
                                       const int64_t *__restrict__ cols,
                                       const double *__restrict__ vals, const T *__restrict__ x,
                                       int64_t col_off, int64_t n, bool &bad) {
    T acc = T(0);
    for (int p = 0; p < npatch; ++p) {
        const int64_t r0 = ldg(rows + 2 * p), r1 = ldg(rows + 2 * p + 1);
        if (r < r0 || r > r1) continue;
        const int64_t c = r - r0 + ldg(cols + p);
        if (c < 0 || c >= n) {
            bad = true;
            continue;
        }
        acc = add_rn(acc, mul_rn((T)ldg(vals + p), ldg(x + col_off + c)));
    }
    return acc;
}

}  // namespace jlb
