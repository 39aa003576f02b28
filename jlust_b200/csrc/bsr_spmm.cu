// bsr_spmm.cu -- BSR (64 x 64 bf16 blocks) x dense bf16 -> fp32 on sm_100a
// tensor cores: TMA-fed shared-memory tiles, tcgen05.mma, TMEM accumulators.
//
// Formulation.  Block rows are taken in pairs (I, I+1).  A pair's blocks are
// walked as the merge of the two rows' block-column lists (each row's blocks
// in its storage order): a group is one block column J with the block of row
// I, of row I+1 or of both.  For a group the MMA computes
//   D (M = 128 x N) += A_pair (128 x 64) x B_J (64 x N)
// with
//   A operand (M=128 x K=16, K-major) = the two 64 x 64 blocks stacked, row
//       I's in rows 0-63 and row I+1's in rows 64-127: two 128-byte-swizzled
//       TMA boxes back to back (SBO = 1 KB between 8-row groups, K advancing
//       32 bytes per 16-element step inside the swizzle atom).  A row with no
//       block in J gets a box loaded from outside the value array, which TMA
//       fills with zeros.
//   B operand (N x K=16, MN-major) = B[J*64 + k, n]: N/64 boxes of 64 B-columns
//       x 64 B-rows with 128-byte swizzle, the canonical MN-major atom stack
//       (LBO = 8 KB between 64-column boxes, SBO = 1 KB between 8-row groups
//       of K); up to 256 columns per MMA.
//   D (fp32, TMEM) lane m, column n = C[I*64 + m, n].
// So a block column both rows hold costs one B slab load and one set of MMAs
// for two blocks (the band of a block-banded matrix), and every MMA is
// 128 x N x 16: four per group for N <= 256.  Each CTA accumulates a whole
// pair (N TMEM columns), double-buffered for N <= 256 so that the epilogue of
// one pair overlaps the MMAs of the next.
//
// Work split.  One CTA per SM (or per block row when there are fewer), each
// with a contiguous range of block rows holding an equal share of the units
// (block rows + stored blocks), found by a binary search over browptr in the
// prologue; the range's rows are paired from its first row.  Cycling pairs
// over the grid instead left SMs with 4 pairs next to SMs with 3 (1024 block
// rows on 148 SMs), a 14% tail.
//
// Warp roles (224 threads): warps 0 and 6 = TMA producers (alternate groups;
// each walks the same merge), warp 1 = TMEM owner and MMA issuer, warps 2-5 =
// epilogue (warp w reads TMEM lanes 32*(w%4) .. +31, i.e. C rows).  No cluster
// multicast is used anywhere.  Every mbarrier wait is bounded: on expiry the
// kernel raises the device error word, all roles leave their loops, every
// copy issued is waited for (bounded) before exit, the MMA issuer waits
// (bounded) for its outstanding MMAs and TMEM is freed.
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace jlb {

JLB_DEFINE_DEV_ERROR(bsr)

namespace bsr {

constexpr int kBS = 64;                        // block size on the tensor path
constexpr int kThreads = 224;                  // 7 warps: see the kernel's role split
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

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int32_t x, int32_t y, int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
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


// The four K-steps (K = 64) of one group into one accumulator, from one asm
// block: the descriptors' low (address) words advance by the K-step's offset
// in 16-byte units -- 32 bytes of the K-major A operand (2), 2048 bytes of
// the MN-major B operand (128) -- so that the issuing thread spends a few
// register moves per MMA.  `first` == 0 makes the first K-step overwrite the
// accumulator.
__device__ __forceinline__ void tc_mma_k64(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi,
                                           uint32_t b_lo, uint32_t b_hi, uint32_t idesc,
                                           uint32_t first) {
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t.reg .b64 a, b;\n\t.reg .b32 t, u;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "setp.eq.b32 q, %5, %5;\n\t"
        "mov.b64 a, {%1, %2};\n\t"
        "mov.b64 b, {%3, %4};\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %6, p;\n\t"
        "add.u32 t, %1, 2;\n\tadd.u32 u, %3, 128;\n\t"
        "mov.b64 a, {t, %2};\n\tmov.b64 b, {u, %4};\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %6, q;\n\t"
        "add.u32 t, %1, 4;\n\tadd.u32 u, %3, 256;\n\t"
        "mov.b64 a, {t, %2};\n\tmov.b64 b, {u, %4};\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %6, q;\n\t"
        "add.u32 t, %1, 6;\n\tadd.u32 u, %3, 384;\n\t"
        "mov.b64 a, {t, %2};\n\tmov.b64 b, {u, %4};\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %6, q;\n\t}"
        ::"r"(d_tmem), "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(first), "r"(idesc)
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

// Instruction descriptor: bf16 x bf16 -> f32, A K-major, B MN-major, M = 128,
// N columns (a multiple of 16, at most 256).
__host__ __device__ constexpr uint32_t idesc_for(uint32_t n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (0u << 15) | (1u << 16) | ((n >> 3) << 17) |
           ((128u >> 4) << 24);
}

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
    long long last_fill[2][kMaxStages];  // per producer: last group index copied into each stage
    int64_t row0, row1;                  // this CTA's block rows [row0, row1)
    uint32_t ginfo[kMaxStages];          // the stage's group: bit 1 last of its pair
    uint32_t tmem_base;
    int abort;
};

// First block row of CTA c's share when G CTAs split the block rows by work
// units u(r) = r + (browptr[r] - base) (one unit per block row for its
// epilogue, one per stored block): the smallest r with u(r) >= c * U / G,
// U = u(mb) = mb + nnzb.  u is strictly increasing, so CTA 0 starts at row 0,
// the last CTA ends at row mb, and neighbouring CTAs' ranges meet.
__device__ int64_t share_start(const int32_t *__restrict__ browptr, int64_t mb, int base,
                               int64_t c, int64_t G) {
    const int64_t U = mb + (int64_t)(browptr[mb] - base);
    const int64_t target = U * c / G;
    int64_t lo = 0, hi = mb;               // answer in [lo, hi]
    while (lo < hi) {
        const int64_t mid = (lo + hi) / 2;
        if (mid + (int64_t)(browptr[mid] - base) >= target) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

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

__host__ __device__ inline uint32_t tmem_cols_for(int n, int nbuf) {
    const uint32_t need = (uint32_t)(n * nbuf);
    uint32_t c = 32;
    while (c < need) c <<= 1;
    return c;
}

// Block-column merge of a pair of block rows: rows a = I and b = I+1 (b
// absent when has_b is false).  next() yields the groups in order: the
// smallest head block column, with each row whose head it is (each row's
// blocks stay in their storage order, sorted or not).
struct PairMerge {
    const int32_t *bcolind;
    int base;
    int qa, qa1, qb, qb1;
    // block columns of the next four entries of each row (INT_MAX past the
    // row's end): each load is issued three steps before its value is needed
    int a0, a1, a2, a3, b0, b1, b2, b3;

    __device__ __forceinline__ int col(int q, int q1) const {
        return q < q1 ? __ldg(bcolind + q) - base : INT_MAX;
    }
    __device__ void init(const int32_t *__restrict__ browptr, const int32_t *__restrict__ bc,
                         int64_t I, bool has_b, int b0_) {
        bcolind = bc;
        base = b0_;
        qa = browptr[I] - base;
        qa1 = browptr[I + 1] - base;
        if (has_b) {
            qb = qa1;
            qb1 = browptr[I + 2] - base;
        } else {
            qb = qb1 = 0;
        }
        a0 = col(qa, qa1); a1 = col(qa + 1, qa1); a2 = col(qa + 2, qa1); a3 = col(qa + 3, qa1);
        b0 = col(qb, qb1); b1 = col(qb + 1, qb1); b2 = col(qb + 2, qb1); b3 = col(qb + 3, qb1);
    }
    __device__ bool done() const { return qa >= qa1 && qb >= qb1; }
    // group: block column J, entries of row a / row b (-1 when absent)
    __device__ void next(int &J, int &ea, int &eb) {
        J = a0 < b0 ? a0 : b0;
        ea = (qa < qa1 && a0 == J) ? qa : -1;
        eb = (qb < qb1 && b0 == J) ? qb : -1;
        if (ea >= 0) {
            ++qa;
            a0 = a1; a1 = a2; a2 = a3; a3 = col(qa + 3, qa1);
        }
        if (eb >= 0) {
            ++qb;
            b0 = b1; b1 = b2; b2 = b3; b3 = col(qb + 3, qb1);
        }
    }
};

template <int N>
__global__ void __launch_bounds__(kThreads, 1)
bsr_spmm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            int64_t mb, const int32_t *__restrict__ browptr, const int32_t *__restrict__ bcolind,
            int base, int stages, int64_t zero_row, float *__restrict__ C, int64_t ldc,
            float alpha, float beta, int has_beta, int b_slab3d) {
    constexpr int kNBuf = 2 * N <= 512 ? 2 : 1;            // accumulators in TMEM
    constexpr int kChunks = N <= 256 ? 1 : 2;               // MMAs per K-step
    constexpr int kN0 = N <= 256 ? N : 256;                 // columns of the first MMA
    constexpr uint32_t kStageBytes = 2 * kATileBytes + (uint32_t)(N / 64) * kBoxBytes;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;
    uint8_t *tiles = smem_raw + pad;
    const uint32_t tiles_u32 = raw + pad;
    Ctl *ctl = reinterpret_cast<Ctl *>(tiles + (size_t)stages * kStageBytes);
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const uint32_t ncols = tmem_cols_for(N, kNBuf);

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(&ctl->full[s]), 1);
            mbar_init(smem_u32(&ctl->empty[s]), 1);
            ctl->last_fill[0][s] = ctl->last_fill[1][s] = -1;
        }
        ctl->row0 = share_start(browptr, mb, base, blockIdx.x, gridDim.x);
        ctl->row1 = share_start(browptr, mb, base, blockIdx.x + 1, gridDim.x);
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
    // The CTA's block rows, taken in pairs (I, I+1) from row0; a last row
    // without a partner inside the range forms a pair of its own.
    const int64_t row0 = ctl->row0, row1 = ctl->row1;

    if ((warp == 0 || warp == 6) && lane == 0) {
        // ------------------------------------------------------ TMA producers
        // Two producer threads take alternate groups (one thread's loop --
        // barrier wait, expect-tx, TMA issues -- costs about as much as a
        // group's MMAs).  Both walk the same merge; group k of the CTA goes to
        // stage k % stages with empty-barrier phase parity (k / stages) & 1 ^ 1,
        // both kept as running counters.
        const int pid = warp == 0 ? 0 : 1;
        long long k = 0;
        int stage = 0;
        uint32_t pe = 1u;
        bool ok = true;
        for (int64_t I = row0; I < row1 && ok; I += 2) {
            PairMerge mg;
            mg.init(browptr, bcolind, I, I + 1 < row1, base);
            while (!mg.done()) {
                int J, ea, eb;
                mg.next(J, ea, eb);
                const bool last = mg.done();
                if ((int)(k & 1) == pid) {
                    if (!mbar_wait(smem_u32(&ctl->empty[stage]), pe, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sA = tiles_u32 + (uint32_t)stage * kStageBytes;
                    const uint32_t full = smem_u32(&ctl->full[stage]);
                    ctl->ginfo[stage] = (last ? 2u : 0u);
                    mbar_arrive_expect_tx(full, kStageBytes);
                    // a missing block: a box wholly past the value array, filled with zeros
                    tma_load_2d(sA, &tmA, full, 0, ea >= 0 ? ea * kBS : (int32_t)zero_row);
                    tma_load_2d(sA + kATileBytes, &tmA, full, 0, eb >= 0 ? eb * kBS : (int32_t)zero_row);
                    if (b_slab3d) {
                        // the whole slab, its N/64 column boxes stacked, in one copy
                        tma_load_3d(sA + 2 * kATileBytes, &tmB, full, 0, J * kBS, 0);
                    } else {
#pragma unroll
                        for (int c = 0; c < N / 64; ++c)
                            tma_load_2d(sA + 2 * kATileBytes + (uint32_t)c * kBoxBytes, &tmB, full,
                                        c * 64, J * kBS);
                    }
                    ctl->last_fill[pid][stage] = k;
                }
                ++k;
                if (++stage == stages) { stage = 0; pe ^= 1u; }
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------- MMA issuer
        int stage = 0;
        uint32_t pf = 0;
        uint32_t te_phase[2] = {1u, 1u};
        int buf = 0;
        bool ok = true;
        const uint64_t adesc0 = sdesc_sw128(tiles_u32, 16u, 1024u);
        const uint64_t bdesc0 = sdesc_sw128(tiles_u32 + 2 * kATileBytes, kBoxBytes, 1024u);
        const uint32_t a_hi = (uint32_t)(adesc0 >> 32), b_hi = (uint32_t)(bdesc0 >> 32);
        constexpr uint32_t kId0 = idesc_for(kN0);
        constexpr uint32_t kId1 = idesc_for(N - kN0 > 0 ? N - kN0 : 16);
        for (int64_t I = row0; I < row1 && ok; I += 2) {
            const int q0 = browptr[I] - base;
            const int q2 = browptr[I + 1 < row1 ? I + 2 : I + 1] - base;
            if (q2 <= q0) continue;                      // no blocks: the epilogue writes it
            if (!mbar_wait(smem_u32(&ctl->tempty[buf]), te_phase[buf], abort_flag)) { ok = false; break; }
            te_phase[buf] ^= 1u;
            tc_fence_after();
            const uint32_t dbase = tmem + (uint32_t)(buf * N);
            uint32_t first = 0;
            for (;;) {
                if (!mbar_wait(smem_u32(&ctl->full[stage]), pf, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t last = ctl->ginfo[stage] & 2u;
                // the stage's descriptors: only the low (address) word moves,
                // without carry (addresses below 256 KB)
                const uint32_t soff = (uint32_t)stage * kStageBytes >> 4;
                const uint32_t a_lo = (uint32_t)adesc0 + soff, b_lo = (uint32_t)bdesc0 + soff;
                tc_mma_k64(dbase, a_lo, a_hi, b_lo, b_hi, kId0, first);
                if (kChunks == 2)
                    tc_mma_k64(dbase + (uint32_t)kN0, a_lo, a_hi, b_lo + (uint32_t)(4 * kBoxBytes >> 4),
                               b_hi, kId1, first);
                tc_commit(smem_u32(&ctl->empty[stage]));
                if (++stage == stages) { stage = 0; pf ^= 1; }
                first = 1;
                if (last) break;
            }
            if (!ok) break;
            tc_commit(smem_u32(&ctl->tfull[buf]));
            buf = (buf + 1) % kNBuf;
        }
        // All MMAs of this thread complete before TMEM can be freed.
        tc_commit(smem_u32(&ctl->mma_done));
        mbar_drain(smem_u32(&ctl->mma_done), 0);
    } else if (warp >= 2 && warp < 6) {
        // --------------------------------------------------------- epilogue
        // warp q (= warp % 4) owns TMEM lanes 32q .. 32q+31: C rows I*64 + 32q
        // + lane, N columns in 32-column loads, stored as 16-byte vectors
        const int qd = warp & 3;
        uint32_t tf_phase[2] = {0u, 0u};
        int buf = 0;
        for (int64_t I = row0; I < row1; I += 2) {
            const int64_t rlim = I + 1 < row1 ? I + 2 : I + 1;
            const int q0 = browptr[I] - base;
            const int q2 = browptr[rlim] - base;
            const int64_t nrows = rlim * kBS;           // end of this pair's C rows
            const int64_t row = I * kBS + qd * 32 + lane;
            if (q2 <= q0) {
                if (row < nrows)
                    for (int64_t c = 0; c < N; ++c) {
                        float *dst = C + row * ldc + c;
                        *dst = has_beta ? add_rn(mul_rn(alpha, 0.0f), mul_rn(beta, *dst))
                                        : mul_rn(alpha, 0.0f);
                    }
                continue;
            }
            if (!mbar_wait(smem_u32(&ctl->tfull[buf]), tf_phase[buf], abort_flag)) break;
            tf_phase[buf] ^= 1u;
            tc_fence_after();
#pragma unroll 1
            for (int c0 = 0; c0 < N; c0 += 32) {
                uint32_t r[32];
                const uint32_t taddr = tmem + ((uint32_t)(qd * 32) << 16) + (uint32_t)(buf * N + c0);
                JLB_TMEM_LD32(taddr, r);
                tmem_wait_ld();
                if (row < nrows) {
                    float4 *dst = reinterpret_cast<float4 *>(C + row * ldc + c0);
#pragma unroll
                    for (int v = 0; v < 8; ++v) {
                        float4 o;
                        o.x = mul_rn(alpha, __uint_as_float(r[4 * v + 0]));
                        o.y = mul_rn(alpha, __uint_as_float(r[4 * v + 1]));
                        o.z = mul_rn(alpha, __uint_as_float(r[4 * v + 2]));
                        o.w = mul_rn(alpha, __uint_as_float(r[4 * v + 3]));
                        if (has_beta) {
                            const float4 old = dst[v];
                            o.x = add_rn(o.x, mul_rn(beta, old.x));
                            o.y = add_rn(o.y, mul_rn(beta, old.y));
                            o.z = add_rn(o.z, mul_rn(beta, old.z));
                            o.w = add_rn(o.w, mul_rn(beta, old.w));
                        }
                        dst[v] = o;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&ctl->tempty[buf]));
            buf = (buf + 1) % kNBuf;
        }
    }

    __syncthreads();
    // every copy issued lands before the CTA can exit (they all have when the
    // MMA issuer consumed every stage; an aborted run may leave some in flight)
    if (threadIdx.x == 0)
        for (int st = 0; st < stages; ++st) {
            const long long lf = ctl->last_fill[0][st] > ctl->last_fill[1][st] ? ctl->last_fill[0][st]
                                                                               : ctl->last_fill[1][st];
            if (lf >= 0) mbar_drain(smem_u32(&ctl->full[st]), (uint32_t)((lf / stages) & 1));
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

// B as a 3-D tensor {64 columns, rows, N/64 column boxes} (strides ldb * 2
// and 128 bytes), so that one box {64, 64, N/64} is a whole 64-row slab laid
// out box after box, as the 2-D boxes would put it.  False when the driver
// refuses the layout.
static bool make_map_b3(CUtensorMap *map, const void *B, int64_t N, uint64_t rows, uint64_t ldb) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {64, rows, (cuuint64_t)(N / 64)};
    cuuint64_t strides[2] = {ldb * 2, 128};
    cuuint32_t box[3] = {64, 64, (cuuint32_t)(N / 64)};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(B), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_eligible(int bs, int64_t N, int64_t ldb, const void *bval, const void *B, int64_t nnzb,
                 int64_t nb, const float *C, int64_t ldc) {
    // TMA coordinates are int32: the zero-filled box starts at row nnzb * 64
    return bs == kBS && N % 128 == 0 && N >= 128 && N <= 512 && ldb % 8 == 0 && aligned16(bval) &&
           aligned16(B) && aligned16(C) && ldc % 4 == 0 && nnzb > 0 &&
           nnzb * kBS + kBS < (int64_t)INT32_MAX && nb * kBS < (int64_t)INT32_MAX;
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
    if (bsr::tc_eligible(bs, N, ldb, bval, B, nnzb, nb, C, ldc)) {
        CUtensorMap tmA, tmB;
        int r = bsr::make_map(&tmA, bval, 64, (uint64_t)nnzb * 64, 128);
        if (r) return r;
        const int b3 = bsr::make_map_b3(&tmB, B, N, (uint64_t)nb * 64, (uint64_t)ldb) ? 1 : 0;
        if (!b3) {
            r = bsr::make_map(&tmB, B, (uint64_t)N, (uint64_t)nb * 64, (uint64_t)ldb * 2);
            if (r) return r;
        }
        const uint32_t stage_bytes = 2 * bsr::kATileBytes + (uint32_t)(N / 64) * bsr::kBoxBytes;
        const size_t budget = 227 * 1024 - 1024 - sizeof(bsr::Ctl) - 64;
        int stages = (int)(budget / stage_bytes);
        if (stages > bsr::kMaxStages) stages = bsr::kMaxStages;
        if (stages < 2) return fail(JLB_ERR_UNSUPPORTED_FORMAT, "N too large for the staging buffers");
        const size_t smem = (size_t)stages * stage_bytes + 1024 + sizeof(bsr::Ctl) + 64;
        int dev = 0, sms = 148;
        JLB_CUDA(cudaGetDevice(&dev));
        JLB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        const unsigned grid = (unsigned)(mb < sms ? mb : sms);
        const int64_t zero_row = nnzb * 64;       // a box wholly past the values: zeros
#define JLB_BSR_TC(NN)                                                                          \
    JLB_CUDA(cudaFuncSetAttribute(bsr::bsr_spmm_tc<NN>,                                         \
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));    \
    bsr::bsr_spmm_tc<NN><<<grid, bsr::kThreads, smem, st>>>(tmA, tmB, mb, browptr, bcolind,     \
                                                            idx_base, stages, zero_row, C, ldc, \
                                                            a, b, b != 0.0f, b3)
        switch (N) {
            case 128: JLB_BSR_TC(128); break;
            case 256: JLB_BSR_TC(256); break;
            case 384: JLB_BSR_TC(384); break;
            default: JLB_BSR_TC(512); break;
        }
#undef JLB_BSR_TC
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
