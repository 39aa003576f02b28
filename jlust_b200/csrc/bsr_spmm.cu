// bsr_spmm.cu -- BSR (64 x 64 bf16 blocks) x dense bf16 -> fp32 on sm_100a
// tensor cores: TMA-fed shared-memory tiles, tcgen05.mma, TMEM accumulators.
//
// Formulation.  For block row I, C[I*64 : I*64+64, :] = sum over stored blocks
// (I, J) of A_IJ (64 x 64) x B[J*64 : J*64+64, :].  The MMA computes the
// transpose, D = B_J^T x A_IJ^T, so that the long side of the output (the N
// columns of C) is the MMA's M = 128 dimension and the 64 rows of the block are
// its N = 64 dimension:
//   MMA A operand  (M=128 x K=16)  = B[J*64 + k, t*128 + m]   -- "MN-major":
//                   m is contiguous in B's rows; a TMA box of 64 B-columns x
//                   64 B-rows with 128-byte swizzle is exactly the canonical
//                   MN-major SW128 atom stack (LBO = 8 KB between the two
//                   64-column boxes of an M-tile, SBO = 1 KB between 8-row
//                   groups of K).
//   MMA B operand  (N=64 x K=16)   = A_IJ[n, k]                 -- "K-major":
//                   the block's rows are 128-byte rows of a TMA box with
//                   128-byte swizzle (SBO = 1 KB; K advances 32 bytes per
//                   16-element step inside the swizzle atom).
//   D (fp32, TMEM) lane m, column n  = C[I*64 + n, t*128 + m].
// Each CTA accumulates a whole block row (N/128 M-tiles x 64 TMEM columns),
// double-buffered so the epilogue of one block row overlaps the MMAs of the
// next.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner and MMA
// issuer, warps 2-5 = epilogue (warp w reads TMEM lanes 32*(w%4) .. +31).  No
// cluster multicast is used anywhere.  Every mbarrier wait is bounded: on
// expiry the kernel raises the device error word, all roles leave their
// loops, the producer waits (bounded) for its outstanding copies, the MMA
// issuer waits (bounded) for its outstanding MMAs and TMEM is freed.
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace jlb {

JLB_DEFINE_DEV_ERROR(bsr)

namespace bsr {

constexpr int kBS = 64;                        // block size on the tensor path
constexpr int kThreads = 192;
constexpr uint32_t kATileBytes = kBS * kBS * 2;  // 8 KB
constexpr uint32_t kBoxBytes = 64 * 128;         // one 64-col x 64-row bf16 box
constexpr long long kTimeoutCycles = 4000000000ll;  // ~2 s at 2 GHz

// ---------------------------------------------------------------- PTX glue
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
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

// Bounded wait for the phase of parity `parity`.  Returns false when the
// kernel is aborting (another role gave up) or when this wait gave up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > kTimeoutCycles) {
            *abort_flag = 1;
            dev_error(DEV_ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Shared-memory matrix descriptor for 128-byte-swizzled operands
// (start address, leading and stride byte offsets in 16-byte units,
// descriptor version 1, layout SWIZZLE_128B).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor: bf16 x bf16 -> f32, A MN-major, B K-major, M=128, N=64.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (0u << 16) |
                            ((64u >> 3) << 17) | ((128u >> 4) << 24);

#define JLB_TMEM_LD32(taddr, r)                                                              \
    asm volatile(                                                                            \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "                                            \
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"                            \
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"          \
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),           \
          "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),         \
          "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),     \
          "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),     \
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),     \
          "=r"(r[30]), "=r"(r[31])                                                           \
        : "r"(taddr)                                                                         \
        : "memory")

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

constexpr int kMaxStages = 8;

struct Ctl {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t mma_done;
    uint32_t tmem_base;
    int abort;
};

// Waits without looking at the abort flag (used while draining on exit).
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kTimeoutCycles) {
            dev_error(DEV_ERR_TIMEOUT);
            return;
        }
    }
}

__device__ __forceinline__ uint32_t tmem_cols_for(int n_mt) {
    const uint32_t need = 2u * (uint32_t)n_mt * 64u;
    uint32_t c = 32;
    while (c < need) c <<= 1;
    return c;
}

__global__ void __launch_bounds__(kThreads, 1)
bsr_spmm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            int64_t mb, const int32_t *__restrict__ browptr, const int32_t *__restrict__ bcolind,
            int base, int n_mt, int stages, float *__restrict__ C, int64_t ldc, float alpha,
            float beta, int has_beta) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;
    uint8_t *tiles = smem_raw + pad;
    const uint32_t tiles_u32 = raw + pad;
    const uint32_t stage_bytes = kATileBytes + (uint32_t)n_mt * 2u * kBoxBytes;
    Ctl *ctl = reinterpret_cast<Ctl *>(tiles + (size_t)stages * stage_bytes);
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const uint32_t ncols = tmem_cols_for(n_mt);
    const int64_t N = (int64_t)n_mt * 128;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(&ctl->full[s]), 1);
            mbar_init(smem_u32(&ctl->empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&ctl->tfull[b]), 1);
            mbar_init(smem_u32(&ctl->tempty[b]), 4);
        }
        mbar_init(smem_u32(&ctl->mma_done), 1);
        ctl->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&ctl->tmem_base)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;
    volatile int *abort_flag = &ctl->abort;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------ TMA producer
        int stage = 0;
        uint32_t pe = 1;
        uint32_t fills[kMaxStages];
        for (int s = 0; s < kMaxStages; ++s) fills[s] = 0;
        bool ok = true;
        for (int64_t I = blockIdx.x; I < mb && ok; I += gridDim.x) {
            const int q0 = browptr[I] - base, q1 = browptr[I + 1] - base;
            for (int q = q0; q < q1; ++q) {
                if (!mbar_wait(smem_u32(&ctl->empty[stage]), pe, abort_flag)) { ok = false; break; }
                const uint32_t full = smem_u32(&ctl->full[stage]);
                mbar_arrive_expect_tx(full, stage_bytes);
                const uint32_t sA = tiles_u32 + (uint32_t)stage * stage_bytes;
                tma_load_2d(sA, &tmA, full, 0, q * kBS);
                const int J = bcolind[q] - base;
                for (int c = 0; c < 2 * n_mt; ++c)
                    tma_load_2d(sA + kATileBytes + (uint32_t)c * kBoxBytes, &tmB, full, c * 64, J * kBS);
                fills[stage] += 1;
                if (++stage == stages) { stage = 0; pe ^= 1; }
            }
        }
        // Let every copy this thread issued land before the CTA can exit.
        for (int s = 0; s < stages; ++s)
            if (fills[s]) mbar_drain(smem_u32(&ctl->full[s]), (fills[s] - 1u) & 1u);
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------- MMA issuer
        int stage = 0;
        uint32_t pf = 0;
        uint32_t te_phase[2] = {1u, 1u};
        int buf = 0;
        bool ok = true;
        for (int64_t I = blockIdx.x; I < mb && ok; I += gridDim.x) {
            const int q0 = browptr[I] - base, q1 = browptr[I + 1] - base;
            if (q1 <= q0) continue;
            if (!mbar_wait(smem_u32(&ctl->tempty[buf]), te_phase[buf], abort_flag)) { ok = false; break; }
            te_phase[buf] ^= 1u;
            tc_fence_after();
            const uint32_t dbase = tmem + (uint32_t)(buf * n_mt * 64);
            for (int q = q0; q < q1; ++q) {
                if (!mbar_wait(smem_u32(&ctl->full[stage]), pf, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t sA = tiles_u32 + (uint32_t)stage * stage_bytes;
                const uint32_t sB = sA + kATileBytes;
                for (int t = 0; t < n_mt; ++t) {
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint64_t adesc = sdesc_sw128(sB + (uint32_t)t * 2u * kBoxBytes + (uint32_t)s * 2048u, kBoxBytes, 1024u);
                        const uint64_t bdesc = sdesc_sw128(sA + (uint32_t)s * 32u, 16u, 1024u);
                        tc_mma(dbase + (uint32_t)t * 64u, adesc, bdesc, kIdesc, (q > q0 || s > 0) ? 1u : 0u);
                    }
                }
                tc_commit(smem_u32(&ctl->empty[stage]));
                if (++stage == stages) { stage = 0; pf ^= 1; }
            }
            if (!ok) break;
            tc_commit(smem_u32(&ctl->tfull[buf]));
            buf ^= 1;
        }
        // All MMAs of this thread complete before TMEM can be freed.
        tc_commit(smem_u32(&ctl->mma_done));
        mbar_drain(smem_u32(&ctl->mma_done), 0);
    } else if (warp >= 2) {
        // --------------------------------------------------------- epilogue
        const int qd = warp & 3;  // TMEM lane quarter this warp may read
        uint32_t tf_phase[2] = {0u, 0u};
        int buf = 0;
        for (int64_t I = blockIdx.x; I < mb; I += gridDim.x) {
            const int q0 = browptr[I] - base, q1 = browptr[I + 1] - base;
            const int64_t row0 = I * kBS;
            if (q1 <= q0) {
                for (int64_t idx = threadIdx.x - 64; idx < (int64_t)kBS * N; idx += 128) {
                    float *dst = C + (row0 + idx / N) * ldc + idx % N;
                    *dst = has_beta ? add_rn(mul_rn(alpha, 0.0f), mul_rn(beta, *dst)) : mul_rn(alpha, 0.0f);
                }
                continue;
            }
            if (!mbar_wait(smem_u32(&ctl->tfull[buf]), tf_phase[buf], abort_flag)) break;
            tf_phase[buf] ^= 1u;
            tc_fence_after();
            for (int t = 0; t < n_mt; ++t) {
                const int64_t col = (int64_t)t * 128 + qd * 32 + lane;
#pragma unroll 1
                for (int h = 0; h < 2; ++h) {
                    uint32_t r[32];
                    const uint32_t taddr = tmem + ((uint32_t)(qd * 32) << 16) +
                                           (uint32_t)(buf * n_mt * 64 + t * 64 + h * 32);
                    JLB_TMEM_LD32(taddr, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int n = 0; n < 32; ++n) {
                        float *dst = C + (row0 + h * 32 + n) * ldc + col;
                        float v = mul_rn(alpha, __uint_as_float(r[n]));
                        if (has_beta) v = add_rn(v, mul_rn(beta, *dst));
                        *dst = v;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&ctl->tempty[buf]));
            buf ^= 1;
        }
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols)
                     : "memory");
    }
}

// SIMT kernel for shapes outside the tensor path: one thread per output
// element, blocks then in-block columns in storage order with separately
// rounded products and sums (the order of the reference's fused CPU loop,
// src/block_sparse.jl:177-188).
__global__ void bsr_spmm_simt(int64_t mb, int bs, const int32_t *__restrict__ browptr,
                              const int32_t *__restrict__ bcolind,
                              const uint16_t *__restrict__ bval, int64_t N,
                              const uint16_t *__restrict__ B, int64_t ldb, float *__restrict__ C,
                              int64_t ldc, float alpha, float beta, int has_beta, int base) {
    const int64_t total = mb * bs * N;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += stride) {
        const int64_t r = idx / N, t = idx % N;
        const int64_t I = r / bs, rr = r % bs;
        const int q0 = browptr[I] - base, q1 = browptr[I + 1] - base;
        float acc = 0.0f;
        for (int q = q0; q < q1; ++q) {
            const int64_t J = (int64_t)bcolind[q] - base;
            const uint16_t *a = bval + ((int64_t)q * bs + rr) * bs;
            for (int c = 0; c < bs; ++c) {
                const float v = bf16_bits_to_f32(__ldg(a + c));
                const float x = bf16_bits_to_f32(__ldg(B + (J * bs + c) * ldb + t));
                acc = add_rn(acc, mul_rn(v, x));
            }
        }
        float *dst = C + r * ldc + t;
        float o = mul_rn(alpha, acc);
        if (has_beta) o = add_rn(o, mul_rn(beta, *dst));
        *dst = o;
    }
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

static int make_map(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                    uint64_t row_bytes) {
    auto fn = encode_fn();
    if (!fn) return fail(JLB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {64, 64};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(JLB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return JLB_OK;
}

bool tc_eligible(int bs, int64_t N, int64_t ldb, const void *bval, const void *B, int64_t nnzb,
                 int64_t nb) {
    return bs == kBS && N % 128 == 0 && N >= 128 && N <= 512 && ldb % 8 == 0 && aligned16(bval) &&
           aligned16(B) && nnzb > 0 && nnzb * kBS < (int64_t)UINT32_MAX && nb * kBS < (int64_t)INT32_MAX;
}

}  // namespace bsr
}  // namespace jlb

using namespace jlb;

extern "C" JLB_API int jlb_bsr_spmm(void *stream, int idx_base, int64_t mb, int64_t nb,
                                    int64_t nnzb, int bs, const int32_t *browptr,
                                    const int32_t *bcolind, const void *bval, int64_t N,
                                    const void *B, int64_t ldb, float *C, int64_t ldc,
                                    double alpha, double beta) {
    if (idx_base != 0 && idx_base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (mb < 0 || nb < 0 || nnzb < 0 || N < 0 || bs <= 0)
        return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "negative extent or block size");
    if (ldb < N || ldc < N) return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "leading dimension smaller than N");
    if (nnzb > INT32_MAX - 1) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "nnzb exceeds Int32 positions");
    if (mb == 0 || N == 0) return ok();
    if (!browptr || !C || (nnzb > 0 && (!bcolind || !bval || !B)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    cudaStream_t st = as_stream(stream);
    const float a = (float)alpha, b = (float)beta;
    if (bsr::tc_eligible(bs, N, ldb, bval, B, nnzb, nb)) {
        CUtensorMap tmA, tmB;
        int r = bsr::make_map(&tmA, bval, 64, (uint64_t)nnzb * 64, 128);
        if (r) return r;
        r = bsr::make_map(&tmB, B, (uint64_t)N, (uint64_t)nb * 64, (uint64_t)ldb * 2);
        if (r) return r;
        const int n_mt = (int)(N / 128);
        const uint32_t stage_bytes = bsr::kATileBytes + (uint32_t)n_mt * 2u * bsr::kBoxBytes;
        const size_t budget = 227 * 1024 - 1024 - sizeof(bsr::Ctl) - 64;
        int stages = (int)(budget / stage_bytes);
        if (stages > bsr::kMaxStages) stages = bsr::kMaxStages;
        if (stages < 2) return fail(JLB_ERR_UNSUPPORTED_FORMAT, "N too large for the staging buffers");
        const size_t smem = (size_t)stages * stage_bytes + 1024 + sizeof(bsr::Ctl) + 64;
        int dev = 0, sms = 148;
        JLB_CUDA(cudaGetDevice(&dev));
        JLB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        JLB_CUDA(cudaFuncSetAttribute(bsr::bsr_spmm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        const unsigned grid = (unsigned)(mb < sms ? mb : sms);
        bsr::bsr_spmm_tc<<<grid, bsr::kThreads, smem, st>>>(tmA, tmB, mb, browptr, bcolind, idx_base,
                                                            n_mt, stages, C, ldc, a, b, b != 0.0f);
        JLB_LAUNCH_CHECK("bsr_spmm_tc");
        return ok();
    }
    const int64_t total = mb * bs * N;
    const unsigned grid = (unsigned)(ceil_div(total, 256) < 148 * 32 ? ceil_div(total, 256) : 148 * 32);
    bsr::bsr_spmm_simt<<<grid, 256, 0, st>>>(mb, bs, browptr, bcolind, (const uint16_t *)bval, N,
                                             (const uint16_t *)B, ldb, C, ldc, a, b, b != 0.0f,
                                             idx_base);
    JLB_LAUNCH_CHECK("bsr_spmm_simt");
    return ok();
}
