// halo.cu -- row-partitioned SpMV fused with its halo exchange over NVLink
// peer memory, for the iterative x <- A x of a banded matrix split across GPUs
// (one process per GPU).
//
// Rank r keeps x in two device buffers (double buffering), each laid out as
// [lower halo (h) | own rows (R) | upper halo (h)].  Step t reads buffer t%2
// and writes buffer (t+1)%2.  In one launch:
//   * the first blocks compute the boundary rows: a block whose rows read the
//     lower halo first waits until the lower neighbour has published step t's
//     halo (flag from_lower >= t), likewise for the upper halo;
//   * the remaining blocks compute the interior rows (which read no halo
//     entry).  Boundary blocks go first so that each step publishes its halo
//     early, with the peer stores and system-scope fences overlapping the
//     interior rows instead of adding to the end of the step; a neighbour's
//     next step then finds the flag already raised;
//   * every boundary row's result is stored into this rank's next buffer and,
//     for the first h rows, into the lower neighbour's next buffer (its upper
//     halo), for the last h rows into the upper neighbour's (its lower halo),
//     through peer pointers (CUDA IPC mappings over NVLink);
//   * when the last block of a side has stored its values (release fence at
//     system scope, then a count), that block raises the neighbour's flag to
//     t+1 with a system-scope release store.
// A neighbour's step-t halo writes target this rank's buffer (t+1)%2 = (t-1)%2
// only after this rank published step t, i.e. after this rank's step-t
// boundary rows (the only readers of that halo) finished -- so no halo is
// overwritten while being read.
//
// Consecutive steps are launched with programmatic dependent launch: step t+1
// reads its rows of A while step t drains and waits for step t's completion
// (griddepcontrol.wait) before reading x.
//
// Every wait is bounded (timeout_ns of the GPU's global timer): on expiry the
// block records DEV_ERR_TIMEOUT, computes with what it has and publishes, so
// the launch ends and jlb_device_status() reports the failure.
// Row sums are formed exactly as by spmv_rows (thread per row, storage order),
// so the partitioned iteration is bit-identical to the single-GPU one.
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cstring>

namespace jlb {

JLB_DEFINE_DEV_ERROR(halo)

namespace halo {

constexpr int kThreads = 256;

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ int ld_acquire_sys(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(int *p, int v) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits (bounded) until *flag >= target; returns false on timeout.
__device__ bool wait_flag(const int *flag, int target, uint64_t timeout_ns) {
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(flag) < target) {
        if (globaltimer() - t0 > timeout_ns) return false;
        __nanosleep(64);
    }
    return true;
}

template <typename T>
__device__ __forceinline__ T row_sum_coherent(int lo, int hi, const int32_t *__restrict__ colind,
                                              const T *__restrict__ val, const T *x, int base) {
    // x is read through L2 (ld.cg): halo entries were written by a peer GPU.
    T acc = T(0);
    for (int k = lo; k < hi; ++k)
        acc = add_rn(acc, mul_rn(ldg(val + k), __ldcg(x + (ldg(colind + k) - base))));
    return acc;
}

template <typename T>
__device__ __forceinline__ T row_sum_ro(int lo, int hi, const int32_t *__restrict__ colind,
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

struct Args {
    int64_t R, h;                 // own rows, halo width
    int64_t i0, i1;               // interior rows [i0, i1)
    int64_t interior_blocks;      // blocks covering [i0, i1)
    int64_t lower_blocks;         // blocks covering [0, i0)
    int64_t upper_blocks;         // blocks covering [i1, R)
    const int32_t *rowptr, *colind;
    const void *val;
    const void *x;                // this rank's buffer t%2
    void *y;                      // this rank's buffer (t+1)%2
    void *lower_next, *upper_next;  // neighbours' buffers (t+1)%2, or null
    int *my_flags;                // [from_lower, from_upper, done_lower, done_upper]
    int *lower_flag, *upper_flag; // neighbours' from_upper / from_lower, or null
    int step, base;
    uint64_t timeout_ns;
};

// Programmatic dependent launch: the next step's grid may start while this
// one drains; it reads its rows of A (independent of x) first and waits for
// this grid's completion (griddepcontrol.wait) before touching x.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

constexpr int kPre = 8;   // entries per row read before the wait

template <typename T>
__global__ void __launch_bounds__(kThreads) halo_step(Args a) {
    const T *val = (const T *)a.val;
    const T *x = (const T *)a.x;
    T *y = (T *)a.y;
    const int64_t b = blockIdx.x;
    const int64_t nbound = a.lower_blocks + a.upper_blocks;
    pdl_trigger();
    if (b >= nbound) {
        const int64_t r = a.i0 + (b - nbound) * kThreads + threadIdx.x;
        int lo = 0, hi = 0;
        int c[kPre];
        T v[kPre];
        if (r < a.i1) {
            lo = ldg(a.rowptr + r) - a.base;
            hi = ldg(a.rowptr + r + 1) - a.base;
#pragma unroll
            for (int j = 0; j < kPre; ++j)
                if (lo + j < hi) {
                    c[j] = ldg(a.colind + lo + j) - a.base;
                    v[j] = ldg(val + lo + j);
                }
        }
        pdl_wait();
        if (r < a.i1) {
            // storage order: the prefetched entries, then any further ones
            T acc = T(0);
#pragma unroll
            for (int j = 0; j < kPre; ++j)
                if (lo + j < hi) acc = add_rn(acc, mul_rn(v[j], ldg(x + c[j])));
            for (int k = lo + kPre; k < hi; ++k)
                acc = add_rn(acc, mul_rn(ldg(val + k), ldg(x + (ldg(a.colind + k) - a.base))));
            y[a.h + r] = acc;
        }
        return;
    }
    pdl_wait();
    // Boundary blocks: side 0 = rows [0, i0) (lower halo), side 1 = [i1, R).
    const int side = b < a.lower_blocks ? 0 : 1;
    const int64_t sb = side == 0 ? b : b - a.lower_blocks;
    const int64_t nb = side == 0 ? a.lower_blocks : a.upper_blocks;
    const int64_t first = side == 0 ? 0 : a.i1, last = side == 0 ? a.i0 : a.R;
    if (threadIdx.x == 0) {
        const int *peer_published = side == 0 ? &a.my_flags[0] : &a.my_flags[1];
        const bool has_peer = side == 0 ? (a.lower_next != nullptr) : (a.upper_next != nullptr);
        if (has_peer && !wait_flag(peer_published, a.step, a.timeout_ns)) dev_error(DEV_ERR_TIMEOUT);
    }
    __syncthreads();
    const int64_t r = first + sb * kThreads + threadIdx.x;
    if (r < last) {
        const int lo = ldg(a.rowptr + r) - a.base, hi = ldg(a.rowptr + r + 1) - a.base;
        const T v = row_sum_coherent<T>(lo, hi, a.colind, val, x, a.base);
        y[a.h + r] = v;
        // first h own rows -> lower neighbour's upper halo; last h -> upper's lower halo
        if (a.lower_next && r < a.h) ((T *)a.lower_next)[a.h + a.R + r] = v;
        if (a.upper_next && r >= a.R - a.h) ((T *)a.upper_next)[r - (a.R - a.h)] = v;
    }
    // Publish: the last block of each side, after every block of that side
    // fenced its peer stores, raises the peer's flag.
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        int *done = side == 0 ? &a.my_flags[2] : &a.my_flags[3];
        const int old = atomicAdd(done, 1);
        if ((int64_t)old == (int64_t)(a.step + 1) * nb - 1) {
            __threadfence_system();
            int *peer_flag = side == 0 ? a.lower_flag : a.upper_flag;
            if (peer_flag) st_release_sys(peer_flag, a.step + 1);
        }
    }
}

}  // namespace halo
}  // namespace jlb

using namespace jlb;

extern "C" JLB_API int jlb_halo_spmv_steps(void *stream, int dtype, int idx_base, int64_t R,
                                           int64_t h, int64_t interior_lo, int64_t interior_hi,
                                           const int32_t *rowptr, const int32_t *colind,
                                           const void *val, void *const *x_bufs,
                                           void *const *lower_bufs, void *const *upper_bufs,
                                           int *my_flags, int *lower_flag, int *upper_flag,
                                           int first_step, int nsteps, uint64_t timeout_ns) {
    if (dtype != JLB_F32 && dtype != JLB_F64)
        return fail(JLB_ERR_UNSUPPORTED_VALUE_TYPE, "halo SpMV supports Float32 and Float64");
    if (idx_base != 0 && idx_base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (R < 0 || h < 0 || interior_lo < 0 || interior_hi > R || interior_lo > interior_hi)
        return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "bad row ranges");
    if (first_step < 0 || nsteps < 0) return fail(JLB_ERR_INVALID_ARGUMENT, "negative step");
    if (!x_bufs || !x_bufs[0] || !x_bufs[1])
        return fail(JLB_ERR_INVALID_ARGUMENT, "x_bufs must hold two buffers");
    const bool lower = lower_bufs != nullptr, upper = upper_bufs != nullptr;
    if (lower != (lower_flag != nullptr) || upper != (upper_flag != nullptr))
        return fail(JLB_ERR_INVALID_ARGUMENT, "neighbour buffers and flag must be given together");
    if ((lower && (!lower_bufs[0] || !lower_bufs[1])) || (upper && (!upper_bufs[0] || !upper_bufs[1])))
        return fail(JLB_ERR_INVALID_ARGUMENT, "neighbour buffers must be two pointers");
    if (lower && interior_lo < h)
        return fail(JLB_ERR_INVALID_ARGUMENT, "rows feeding the lower neighbour must be boundary rows");
    if (upper && R - interior_hi < h)
        return fail(JLB_ERR_INVALID_ARGUMENT, "rows feeding the upper neighbour must be boundary rows");
    if ((lower || upper) && R < 2 * h)
        return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "each rank needs at least 2*h rows");
    if (R == 0 || nsteps == 0) return ok();
    if (!rowptr || !colind || !val || !my_flags) return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    halo::Args a;
    a.R = R; a.h = h; a.i0 = interior_lo; a.i1 = interior_hi;
    a.interior_blocks = ceil_div(interior_hi - interior_lo, halo::kThreads);
    a.lower_blocks = ceil_div(interior_lo, halo::kThreads);
    a.upper_blocks = ceil_div(R - interior_hi, halo::kThreads);
    a.rowptr = rowptr; a.colind = colind; a.val = val; a.my_flags = my_flags;
    a.lower_flag = lower_flag; a.upper_flag = upper_flag;
    a.base = idx_base; a.timeout_ns = timeout_ns;
    const int64_t grid = a.interior_blocks + a.lower_blocks + a.upper_blocks;
    cudaStream_t st = as_stream(stream);
    for (int t = first_step; t < first_step + nsteps; ++t) {
        a.step = t;
        a.x = x_bufs[t % 2];
        a.y = x_bufs[(t + 1) % 2];
        a.lower_next = lower ? lower_bufs[(t + 1) % 2] : nullptr;
        a.upper_next = upper ? upper_bufs[(t + 1) % 2] : nullptr;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(halo::kThreads);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (dtype == JLB_F64) JLB_CUDA(cudaLaunchKernelEx(&cfg, halo::halo_step<double>, a));
        else JLB_CUDA(cudaLaunchKernelEx(&cfg, halo::halo_step<float>, a));
    }
    return ok();
}

// Base and offset of a device pointer inside its cudaMalloc allocation (an
// IPC handle names the allocation, so peers add the offset themselves).
static int alloc_base(void *ptr, void **base) {
    static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return fail(JLB_ERR_CUDA, "cuMemGetAddressRange is unavailable");
        fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
    }
    CUdeviceptr b = 0;
    size_t sz = 0;
    CUresult r = fn(&b, &sz, reinterpret_cast<CUdeviceptr>(ptr));
    if (r != CUDA_SUCCESS) return fail(JLB_ERR_CUDA, "cuMemGetAddressRange failed (%d)", (int)r);
    *base = reinterpret_cast<void *>(b);
    return JLB_OK;
}

extern "C" JLB_API int jlb_ipc_handle(void *ptr, void *handle_out, uint64_t *offset_out) {
    if (!ptr || !handle_out || !offset_out) return fail(JLB_ERR_INVALID_ARGUMENT, "null pointer");
    void *base = nullptr;
    int r = alloc_base(ptr, &base);
    if (r) return r;
    cudaIpcMemHandle_t hdl;
    JLB_CUDA(cudaIpcGetMemHandle(&hdl, base));
    memcpy(handle_out, &hdl, sizeof(hdl));
    *offset_out = (uint64_t)((char *)ptr - (char *)base);
    return ok();
}

extern "C" JLB_API int jlb_ipc_open(const void *handle, void **base_out) {
    if (!base_out || !handle) return fail(JLB_ERR_INVALID_ARGUMENT, "null pointer");
    cudaIpcMemHandle_t hdl;
    memcpy(&hdl, handle, sizeof(hdl));
    JLB_CUDA(cudaIpcOpenMemHandle(base_out, hdl, cudaIpcMemLazyEnablePeerAccess));
    return ok();
}

extern "C" JLB_API int jlb_ipc_close(void *base) {
    if (base) JLB_CUDA(cudaIpcCloseMemHandle(base));
    return ok();
}
