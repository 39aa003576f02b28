// sort.cuh -- per-bucket sorts of entry indices by (coordinate, storage
// index) on sm_100a, shared by the conversions and SpGEMM.  Include after the
// translation unit's JLB_DEFINE_DEV_ERROR: the kernels report through its
// dev_error.  Everything here has internal linkage, one copy per unit.
//
// Keys are 64-bit, coordinate << 32 | storage index, so they are unique and
// any correct sort gives the same order.  Buckets of up to kThreadKeys
// entries are insertion-sorted by one thread.  Larger ones go through an
// ascending bitonic network run on positions [0, len) of a power-of-two
// network (positions past len act as +infinity and are never touched): up to
// kWarpKeys entries by one warp in shared memory, up to kCtaKeys by one CTA
// in shared memory, longer ones (up to kMaxSortKeys) by one CTA in place in
// global memory, gathering the coordinate per comparison.
#pragma once
#include "common.cuh"

namespace jlb {
namespace seg {
namespace {

constexpr int kSortThreads = 256;
constexpr int kWarpKeys = 256;
constexpr int kLongThreads = 1024;
constexpr int kCtaKeys = 16384;   // 128 KB of keys
constexpr int64_t kMaxSortKeys = (int64_t)1 << 24;   // longest row the global-memory sort takes

__device__ __forceinline__ uint64_t entry_key(const int32_t *__restrict__ cols, int base,
                                              int32_t e) {
    return ((uint64_t)(uint32_t)(ldg(cols + e) - base) << 32) | (uint32_t)e;
}

// One step pair of the network: the partner of i in step (k, j), or -1.
template <typename I>
__device__ __forceinline__ I bitonic_partner(I i, I k, I j, I len) {
    const I l = j == (k >> 1) ? (i ^ (k - 1)) : (i ^ j);
    return (l > i && l < len) ? l : I(-1);
}

struct WarpSync {
    __device__ __forceinline__ void operator()() const { __syncwarp(); }
};
struct BlockSync {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

// Ascending sort of s[0, len) by the threads tid, tid + nthr, ...; sync()
// separates the steps and must be reached by all of them.
template <typename Sync>
__device__ void bitonic_smem(uint64_t *s, int len, int tid, int nthr, Sync sync) {
    int P = 1;
    while (P < len) P <<= 1;
    for (int k = 2; k <= P; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < P; i += nthr) {
                const int l = bitonic_partner<int>(i, k, j, len);
                if (l < 0) continue;
                const uint64_t a = s[i], b = s[l];
                if (a > b) {
                    s[i] = b;
                    s[l] = a;
                }
            }
            sync();
        }
}

__device__ __forceinline__ int warp_isum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

constexpr int kThreadKeys = 16;

// Sorts every bucket of up to kWarpKeys entries and counts its distinct
// columns into cnt[r]; longer rows are appended to `long_rows`.  A warp takes
// 32 rows at a time: each lane sorts its own row when it has at most
// kThreadKeys entries (insertion sort in registers and local memory), then the
// warp sorts the others one after another in shared memory.  The keys are
// unique, so both sorts give the same order.
__global__ void __launch_bounds__(kSortThreads)
sort_short_rows(int64_t m, const int32_t *__restrict__ offs, int32_t *__restrict__ ent,
                const int32_t *__restrict__ cols, int base, int32_t *__restrict__ cnt,
                int32_t *__restrict__ long_rows, int32_t *__restrict__ n_long, int64_t long_cap) {
    __shared__ uint64_t s_keys[kSortThreads / kWarp][kWarpKeys];
    const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
    uint64_t *s = s_keys[warp];
    const int64_t nwarps = (int64_t)gridDim.x * (kSortThreads / kWarp);
    for (int64_t rb = ((int64_t)blockIdx.x * (kSortThreads / kWarp) + warp) * kWarp; rb < m;
         rb += nwarps * kWarp) {
        const int64_t r = rb + lane;
        int lo = 0, len = 0;
        if (r < m) {
            lo = ldg(offs + r);
            len = ldg(offs + r + 1) - lo;
        }
        if (r < m && len <= kThreadKeys) {
            uint64_t k[kThreadKeys];
            for (int i = 0; i < len; ++i) {
                const uint64_t key = entry_key(cols, base, ent[lo + i]);
                int j = i;
                while (j > 0 && k[j - 1] > key) {
                    k[j] = k[j - 1];
                    --j;
                }
                k[j] = key;
            }
            int u = 0;
            for (int i = 0; i < len; ++i) {
                ent[lo + i] = (int32_t)(uint32_t)k[i];
                u += (i == 0 || (k[i] >> 32) != (k[i - 1] >> 32));
            }
            cnt[r] = u;
        }
        unsigned rest = __ballot_sync(0xffffffffu, r < m && len > kThreadKeys);
        while (rest) {
            const int src = __ffs(rest) - 1;
            rest &= rest - 1;
            const int64_t rr = rb + src;
            const int rlo = __shfl_sync(0xffffffffu, lo, src);
            const int rlen = __shfl_sync(0xffffffffu, len, src);
            if (rlen > kWarpKeys) {
                if (lane == 0) {
                    const int q = atomicAdd(n_long, 1);
                    if (q < long_cap) long_rows[q] = (int32_t)rr;
                    else dev_error(DEV_ERR_OVERFLOW);
                }
                continue;
            }
            for (int i = lane; i < rlen; i += kWarp) s[i] = entry_key(cols, base, ent[rlo + i]);
            __syncwarp();
            bitonic_smem(s, rlen, lane, kWarp, WarpSync{});
            int u = 0;
            for (int i = lane; i < rlen; i += kWarp) {
                ent[rlo + i] = (int32_t)(uint32_t)s[i];
                u += (i == 0 || (s[i] >> 32) != (s[i - 1] >> 32));
            }
            u = warp_isum(u);
            if (lane == 0) cnt[rr] = u;
            __syncwarp();
        }
    }
}

__device__ __forceinline__ int block_isum(int v, int *s_red) {
    const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
    v = warp_isum(v);
    if (lane == 0) s_red[warp] = v;
    __syncthreads();
    int t = 0;
    for (int w = 0; w < (int)(blockDim.x / kWarp); ++w) t += s_red[w];
    __syncthreads();
    return t;
}

// Sorts the buckets listed in long_rows, one CTA per row.
__global__ void __launch_bounds__(kLongThreads)
sort_long_rows(const int32_t *__restrict__ offs, int32_t *ent, const int32_t *__restrict__ cols,
               int base, int32_t *__restrict__ cnt, const int32_t *__restrict__ long_rows,
               const int32_t *__restrict__ n_long, int64_t long_cap) {
    extern __shared__ uint64_t s_dyn[];
    __shared__ int s_red[kLongThreads / kWarp];
    const int tid = threadIdx.x;
    int nl = *n_long;
    if (nl > long_cap) nl = (int)long_cap;
    for (int b = blockIdx.x; b < nl; b += gridDim.x) {
        const int32_t r = long_rows[b];
        const int lo = ldg(offs + r), len = ldg(offs + r + 1) - lo;
        int u = 0;
        if (len > kMaxSortKeys) {
            if (tid == 0) {
                dev_error(DEV_ERR_OVERFLOW);
                cnt[r] = 0;
            }
            continue;
        }
        if (len <= kCtaKeys) {
            for (int i = tid; i < len; i += kLongThreads) s_dyn[i] = entry_key(cols, base, ent[lo + i]);
            __syncthreads();
            bitonic_smem(s_dyn, len, tid, kLongThreads, BlockSync{});
            for (int i = tid; i < len; i += kLongThreads) {
                ent[lo + i] = (int32_t)(uint32_t)s_dyn[i];
                u += (i == 0 || (s_dyn[i] >> 32) != (s_dyn[i - 1] >> 32));
            }
        } else {
            // In place in global memory: the same network on entry indices,
            // each comparison gathering both columns.
            int32_t *e = ent + lo;
            const int64_t n64 = len;
            int64_t P = 1;
            while (P < n64) P <<= 1;
            for (int64_t k = 2; k <= P; k <<= 1)
                for (int64_t j = k >> 1; j > 0; j >>= 1) {
                    for (int64_t i = tid; i < P; i += kLongThreads) {
                        const int64_t l = bitonic_partner<int64_t>(i, k, j, n64);
                        if (l < 0) continue;
                        const int32_t ea = e[i], eb = e[l];
                        if (entry_key(cols, base, ea) > entry_key(cols, base, eb)) {
                            e[i] = eb;
                            e[l] = ea;
                        }
                    }
                    __syncthreads();
                }
            for (int i = tid; i < len; i += kLongThreads)
                u += (i == 0 || ldg(cols + e[i]) != ldg(cols + e[i - 1]));
        }
        u = block_isum(u, s_red);
        if (tid == 0) cnt[r] = u;
        __syncthreads();
    }
}

}  // namespace
}  // namespace seg
}  // namespace jlb
