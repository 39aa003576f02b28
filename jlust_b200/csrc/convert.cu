// convert.cu -- GPU CSR/COO -> BSRRight((b1, b2)) conversion and position
// scans for sm_100a, bit-exact with JLUST's CPU convert_format
// (src/convert.jl:302-388) using the level extents of
// dim2lvl(...; as_size=true) (src/formats.jl:204-220): ceil(m/b1) block rows,
// b1 x b2 row-major tiles.
//
// Layout of the work: one CTA per block row I.  The block columns J that hold
// at least one nonzero entry of rows [I*b1, I*b1+b1) are marked in a
// shared-memory bitmap (windows of kWinBits block columns when the matrix is
// wider); popcounts give the per-block-row block counts, an exclusive scan
// gives the block row pointer, and in the fill pass a prefix of the bitmap
// words gives every J its rank -- its slot in the block column array, which
// is therefore ascending as the composer's sorted output is.  Values are
// copied bit for bit into zero-filled tiles.
//
// COO input is first bucketed by block row (count, scan, scatter of entry
// indices).  Duplicate coordinates resolve exactly as the composer's stable
// sort does -- the nonzero entry with the lowest storage index wins -- via an
// atomicMin over the storage index per tile cell, then a second pass that
// writes the winner's value.
#include "common.cuh"

#include <mutex>

namespace jlb {

JLB_DEFINE_DEV_ERROR(convert)

namespace conv {

constexpr int kThreads = 256;
constexpr int kConvThreads = 1024;   // threads of the CSR/COO -> BSR kernels (one CTA per block row)
constexpr int kScanItems = 8;
constexpr int kScanTile = kThreads * kScanItems;
constexpr int64_t kWinBits = 163840;  // block columns per bitmap window (bitmap + prefix = 40 KB)
constexpr int kWinWords = (int)(kWinBits / 32);

// ------------------------------------------------------------------ scans
template <int NT = kThreads>
__device__ __forceinline__ int64_t block_exclusive_scan(int64_t v, int64_t *s_warp, int64_t &total) {
    const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
    int64_t x = v;
#pragma unroll
    for (int o = 1; o < kWarp; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == kWarp - 1) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int64_t w = lane < NT / kWarp ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < kWarp; o <<= 1) {
            const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < NT / kWarp) s_warp[lane] = w;
    }
    __syncthreads();
    total = s_warp[NT / kWarp - 1];
    const int64_t before = warp > 0 ? s_warp[warp - 1] : 0;
    __syncthreads();
    return before + x - v;
}

__global__ void __launch_bounds__(kThreads)
scan_tile_sums(int64_t n, const int32_t *__restrict__ counts, int64_t *__restrict__ sums) {
    __shared__ int64_t s_warp[kThreads / kWarp];
    const int64_t t0 = (int64_t)blockIdx.x * kScanTile;
    int64_t v = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const int64_t i = t0 + (int64_t)threadIdx.x * kScanItems + j;
        if (i < n) v += counts[i];
    }
    int64_t total;
    block_exclusive_scan(v, s_warp, total);
    if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kThreads)
scan_sums_single(int64_t ntiles, int64_t *__restrict__ sums) {
    __shared__ int64_t s_warp[kThreads / kWarp];
    int64_t carry = 0;
    for (int64_t c0 = 0; c0 < ntiles; c0 += kThreads) {
        const int64_t i = c0 + threadIdx.x;
        const int64_t v = i < ntiles ? sums[i] : 0;
        int64_t total;
        const int64_t ex = block_exclusive_scan(v, s_warp, total);
        if (i < ntiles) sums[i] = carry + ex;
        carry += total;
    }
}

__global__ void __launch_bounds__(kThreads)
scan_tiles_final(int64_t n, const int32_t *counts, int32_t *out, const int64_t *__restrict__ sums,
                 int base) {
    __shared__ int64_t s_warp[kThreads / kWarp];
    const int64_t t0 = (int64_t)blockIdx.x * kScanTile;
    int32_t items[kScanItems];
    int64_t v = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const int64_t i = t0 + (int64_t)threadIdx.x * kScanItems + j;
        items[j] = i < n ? counts[i] : 0;
        v += items[j];
    }
    int64_t total;
    int64_t run = block_exclusive_scan(v, s_warp, total) + sums[blockIdx.x] + base;
    // `out` may alias `counts + 1`: every element is read above and written
    // below by the same thread.
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const int64_t i = t0 + (int64_t)threadIdx.x * kScanItems + j;
        run += items[j];
        if (i < n) {
            if (run > INT32_MAX) dev_error(DEV_ERR_OVERFLOW);
            out[i + 1] = (int32_t)run;
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) out[0] = base;
}

size_t scan_ws(int64_t n) { return (size_t)(ceil_div(n > 0 ? n : 1, kScanTile) * sizeof(int64_t)); }

int scan(cudaStream_t st, int64_t n, const int32_t *counts, int32_t *out, int base, void *ws,
         size_t ws_bytes) {
    if (ws_bytes < scan_ws(n) || (!ws && n > 0))
        return fail(JLB_ERR_WORKSPACE, "scan workspace %zu < %zu bytes", ws_bytes, scan_ws(n));
    if (n == 0) {
        JLB_CUDA(cudaMemcpyAsync(out, &base, sizeof(int32_t), cudaMemcpyHostToDevice, st));
        // The host value must outlive the async copy.
        JLB_CUDA(cudaStreamSynchronize(st));
        return ok();
    }
    const int64_t ntiles = ceil_div(n, kScanTile);
    int64_t *sums = (int64_t *)ws;
    scan_tile_sums<<<(unsigned)ntiles, kThreads, 0, st>>>(n, counts, sums);
    scan_sums_single<<<1, kThreads, 0, st>>>(ntiles, sums);
    scan_tiles_final<<<(unsigned)ntiles, kThreads, 0, st>>>(n, counts, out, sums, base);
    JLB_LAUNCH_CHECK("exclusive_scan");
    return ok();
}

// ------------------------------------------------------------ value helpers
// ES = bytes per value (8 fp64, 4 fp32, 2 bf16); the conversion kernels are
// compiled per value size so that these are single loads and stores.
template <int ES>
__device__ __forceinline__ bool is_zero(const void *val, int64_t p) {
    if (ES == 8) return reinterpret_cast<const double *>(val)[p] == 0.0;
    if (ES == 4) return reinterpret_cast<const float *>(val)[p] == 0.0f;
    return (reinterpret_cast<const uint16_t *>(val)[p] & 0x7fffu) == 0;
}

__device__ __forceinline__ bool is_zero(const void *val, int es, int64_t p) {
    return es == 8 ? is_zero<8>(val, p) : es == 4 ? is_zero<4>(val, p) : is_zero<2>(val, p);
}

template <int ES>
__device__ __forceinline__ void copy_val(void *dst, int64_t q, const void *src, int64_t p) {
    if (ES == 8) reinterpret_cast<uint64_t *>(dst)[q] = reinterpret_cast<const uint64_t *>(src)[p];
    else if (ES == 4) reinterpret_cast<uint32_t *>(dst)[q] = reinterpret_cast<const uint32_t *>(src)[p];
    else reinterpret_cast<uint16_t *>(dst)[q] = reinterpret_cast<const uint16_t *>(src)[p];
}

// Zero-fills bytes [b0, b1) of `dst` with the CTA, 16-byte stores where aligned.
__device__ void zero_bytes(char *dst, int64_t b0, int64_t b1) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(dst + b0);
    int64_t head = (int64_t)((16 - (a0 & 15)) & 15);
    if (head > b1 - b0) head = b1 - b0;
    for (int64_t i = b0 + threadIdx.x; i < b0 + head; i += blockDim.x) dst[i] = 0;
    const int64_t vb = b0 + head;
    const int64_t nv = (b1 - vb) / 16;
    uint4 *v = reinterpret_cast<uint4 *>(dst + vb);
    for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) v[i] = make_uint4(0, 0, 0, 0);
    for (int64_t i = vb + nv * 16 + threadIdx.x; i < b1; i += blockDim.x) dst[i] = 0;
}

// Entry source of one block row: CSR rows or a COO bucket.
struct Src {
    const int32_t *rowptr;   // CSR: row pointer (null for COO)
    const int32_t *rows;     // COO: row coordinates
    const int32_t *cols;
    const void *val;
    const int32_t *boffs;    // COO: bucket offsets (mb+1), base 0
    const int32_t *bent;     // COO: bucketed storage indices
    int64_t m, n;
    int b1, b2, base, es;
    int sh1, sh2;            // log2(b1), log2(b2) when a power of two, else -1

    __device__ __forceinline__ int64_t blk_col(int64_t j) const { return sh2 >= 0 ? j >> sh2 : j / b2; }
    __device__ __forceinline__ int64_t in_col(int64_t j) const { return sh2 >= 0 ? j & (b2 - 1) : j % b2; }
    __device__ __forceinline__ int64_t in_row(int64_t i) const { return sh1 >= 0 ? i & (b1 - 1) : i % b1; }
    // 32-bit forms for CSR columns (Int32 coordinates)
    __device__ __forceinline__ int blk_col32(int j) const { return sh2 >= 0 ? j >> sh2 : j / b2; }
    __device__ __forceinline__ int in_col32(int j) const { return sh2 >= 0 ? j & (b2 - 1) : j % b2; }
};

inline int log2_exact(int b) {
    int k = 0;
    while ((1 << k) < b) ++k;
    return (1 << k) == b ? k : -1;
}

constexpr int kUnrollEntries = 4;   // entries per lane loaded before use

// CSR rows of block row I, warp-synchronously: every lane of the warp calls
// f(p, i, j, ok) for kUnrollEntries entries at a time (ok false for padding,
// explicit zeros and out-of-range columns), so f may use warp shuffles.  The
// loads of a batch are issued before any use.
// Entry indices and columns fit 32 bits (nnz < 2^31, Int32 coordinates).
template <int ES, typename F>
__device__ __forceinline__ void for_each_csr_row_sync(const Src &s, int64_t I, F f) {
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int64_t i0 = I * s.b1;
    const int n = (int)(s.n < INT32_MAX ? s.n : INT32_MAX);
    for (int r = warp; r < s.b1; r += kConvThreads / kWarp) {
        const int64_t i = i0 + r;
        if (i >= s.m) break;
        const int lo = s.rowptr[i] - s.base, hi = s.rowptr[i + 1] - s.base;
        for (int p0 = lo; p0 < hi; p0 += kWarp * kUnrollEntries) {
            int jj[kUnrollEntries];
            bool nz[kUnrollEntries];
#pragma unroll
            for (int u = 0; u < kUnrollEntries; ++u) {
                const int p = p0 + u * kWarp + lane;
                nz[u] = p < hi;
                jj[u] = nz[u] ? __ldg(s.cols + p) - s.base : -1;
                if (nz[u]) nz[u] = !is_zero<ES>(s.val, p);
            }
#pragma unroll
            for (int u = 0; u < kUnrollEntries; ++u) {
                const int p = p0 + u * kWarp + lane;
                bool ok = nz[u];
                if (ok && (jj[u] < 0 || jj[u] >= n)) {
                    dev_error(DEV_ERR_BOUNDS);
                    ok = false;
                }
                f(p, i, jj[u], ok);
            }
        }
    }
}

// Calls f(p, i, j) for every nonzero entry of block row I (storage index p,
// 0-based row i and column j).  CSR: one warp per row, lanes over entries.
template <int ES, typename F>
__device__ __forceinline__ void for_each_entry(const Src &s, int64_t I, F f) {
    if (s.rowptr) {
        const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
        const int64_t i0 = I * s.b1;
        for (int r = warp; r < s.b1; r += kConvThreads / kWarp) {
            const int64_t i = i0 + r;
            if (i >= s.m) break;
            const int64_t lo = (int64_t)s.rowptr[i] - s.base, hi = (int64_t)s.rowptr[i + 1] - s.base;
            for (int64_t p = lo + lane; p < hi; p += kWarp) {
                if (is_zero<ES>(s.val, p)) continue;
                const int64_t j = (int64_t)s.cols[p] - s.base;
                if (j < 0 || j >= s.n) { dev_error(DEV_ERR_BOUNDS); continue; }
                f(p, i, j);
            }
        }
    } else {
        const int64_t e0 = s.boffs[I], e1 = s.boffs[I + 1];
        for (int64_t e = e0 + threadIdx.x; e < e1; e += kConvThreads) {
            const int64_t p = s.bent[e];
            const int64_t i = (int64_t)s.rows[p] - s.base, j = (int64_t)s.cols[p] - s.base;
            if (i < 0 || i >= s.m || j < 0 || j >= s.n) { dev_error(DEV_ERR_BOUNDS); continue; }
            f(p, i, j);
        }
    }
}

// Marks the block columns of window [w0, w0 + kWinBits) hit by block row I.
template <int ES>
__device__ __forceinline__ void mark_window(const Src &s, int64_t I, int64_t w0, uint32_t *bits) {
    if (s.rowptr) {
        // CSR: a row's columns ascend, so one atomic per run of equal block
        // columns across the lanes (compare with the previous lane; unsorted
        // rows stay correct, with more atomics)
        const int w0i = (int)w0;   // block columns fit 32 bits
        for_each_csr_row_sync<ES>(s, I, [&](int, int64_t, int j, bool ok) {
            const int J = ok ? s.blk_col32(j) - w0i : -1;
            const bool in = ok && J >= 0 && J < kWinBits;
            const int prev = __shfl_up_sync(0xffffffffu, in ? J : -1, 1);
            const bool lead = (threadIdx.x % kWarp) == 0 || prev != J;
            if (in && lead) atomicOr(&bits[J >> 5], 1u << (J & 31));
        });
        return;
    }
    for_each_entry<ES>(s, I, [&](int64_t p, int64_t i, int64_t j) {
        const int64_t J = s.blk_col(j) - w0;
        const bool in = J >= 0 && J < kWinBits;
        // one atomic per distinct J among the lanes that agree on it
        const unsigned act = __activemask();
        const unsigned peers = __match_any_sync(act, in ? (long long)J : -1ll);
        if (in && (__ffs(peers) - 1) == (int)(threadIdx.x % kWarp))
            atomicOr(&bits[J >> 5], 1u << (J & 31));
    });
}

__device__ __forceinline__ int64_t block_sum(int64_t v, int64_t *s_red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x % kWarp == 0) s_red[threadIdx.x / kWarp] = v;
    __syncthreads();
    int64_t t = 0;
    for (int w = 0; w < kConvThreads / kWarp; ++w) t += s_red[w];
    __syncthreads();
    return t;
}

// Block-column bitmaps handed from the count pass to the fill pass through the
// caller's workspace (one window only, i.e. at most kWinBits block columns):
// the fill pass then reads the CSR once instead of twice.  `stamp` holds a
// key of the count call's arguments; the fill pass uses the bitmaps only when
// its own key matches, and marks them again otherwise.
struct Carry {
    uint32_t *bits;      // mb x words, or null: no hand-over
    uint64_t *stamp;
    uint64_t key;
};

// Count pass: counts[I] (= browptr[I+1]) = number of distinct nonzero blocks.
template <int ES>
__global__ void __launch_bounds__(kConvThreads)
count_blocks(Src s, int64_t mb, int64_t nb, int32_t *__restrict__ counts, Carry carry) {
    __shared__ uint32_t bits[kWinWords];
    __shared__ int64_t s_red[kConvThreads / kWarp];
    for (int64_t I = blockIdx.x; I < mb; I += gridDim.x) {
        int64_t total = 0;
        for (int64_t w0 = 0; w0 < nb; w0 += kWinBits) {
            const int nw = (int)ceil_div((nb - w0) < kWinBits ? (nb - w0) : kWinBits, 32);
            for (int w = threadIdx.x; w < nw; w += kConvThreads) bits[w] = 0;
            __syncthreads();
            mark_window<ES>(s, I, w0, bits);
            __syncthreads();
            int64_t c = 0;
            for (int w = threadIdx.x; w < nw; w += kConvThreads) {
                c += __popc(bits[w]);
                if (carry.bits) carry.bits[I * nw + w] = bits[w];
            }
            total += block_sum(c, s_red);
        }
        if (threadIdx.x == 0) {
            if (total > INT32_MAX) dev_error(DEV_ERR_OVERFLOW);
            counts[I] = (int32_t)total;
        }
        __syncthreads();
    }
    if (carry.bits && blockIdx.x == 0 && threadIdx.x == 0) *carry.stamp = carry.key;
}

// Fill pass.  winner == nullptr means the source has unique coordinates.
template <int ES>
__global__ void __launch_bounds__(kConvThreads, 2)
fill_blocks(Src s, int64_t mb, int64_t nb, int64_t nnzb, const int32_t *__restrict__ browptr,
            int32_t *__restrict__ bcolind, void *__restrict__ bval, int32_t *__restrict__ winner,
            Carry carry) {
    const bool handed = carry.bits && *carry.stamp == carry.key;
    __shared__ uint32_t bits[kWinWords];
    __shared__ int32_t pref[kWinWords];
    __shared__ int64_t s_warp[kConvThreads / kWarp];
    const int64_t bsz = (int64_t)s.b1 * s.b2;
    for (int64_t I = blockIdx.x; I < mb; I += gridDim.x) {
        int64_t q0 = (int64_t)browptr[I] - s.base, q1 = (int64_t)browptr[I + 1] - s.base;
        if (q0 < 0 || q1 < q0 || q1 > nnzb) {
            if (threadIdx.x == 0) dev_error(DEV_ERR_BOUNDS);
            q0 = q1 = 0;  // write nothing for this block row
        }
        zero_bytes(reinterpret_cast<char *>(bval), q0 * bsz * s.es, q1 * bsz * s.es);
        if (winner)
            for (int64_t c = q0 * bsz + threadIdx.x; c < q1 * bsz; c += kConvThreads) winner[c] = INT32_MAX;
        __syncthreads();
        int64_t rank0 = 0;  // blocks in earlier windows
        for (int64_t w0 = 0; w0 < nb; w0 += kWinBits) {
            const int nw = (int)ceil_div((nb - w0) < kWinBits ? (nb - w0) : kWinBits, 32);
            if (handed) {
                for (int w = threadIdx.x; w < nw; w += kConvThreads) bits[w] = carry.bits[I * nw + w];
                __syncthreads();
            } else {
                for (int w = threadIdx.x; w < nw; w += kConvThreads) bits[w] = 0;
                __syncthreads();
                mark_window<ES>(s, I, w0, bits);
                __syncthreads();
            }
            // exclusive prefix of the word popcounts, kConvThreads words at a time
            int64_t carry = 0;
            for (int c0 = 0; c0 < nw; c0 += kConvThreads) {
                const int w = c0 + threadIdx.x;
                const int64_t v = w < nw ? __popc(bits[w]) : 0;
                int64_t tot;
                const int64_t ex = block_exclusive_scan<kConvThreads>(v, s_warp, tot);
                if (w < nw) pref[w] = (int32_t)(carry + ex);
                carry += tot;
            }
            __syncthreads();
            // block column array, ascending
            for (int w = threadIdx.x; w < nw; w += kConvThreads) {
                uint32_t word = bits[w];
                int r = pref[w];
                while (word) {
                    const int b = __ffs(word) - 1;
                    word &= word - 1;
                    if (q0 + rank0 + r < q1)
                        bcolind[q0 + rank0 + r] = (int32_t)(w0 + (int64_t)w * 32 + b) + s.base;
                    else
                        dev_error(DEV_ERR_BOUNDS);
                    ++r;
                }
            }
            auto cell_of = [&](int64_t i, int64_t j) -> int64_t {
                const int64_t J = s.blk_col(j) - w0;
                if (J < 0 || J >= kWinBits) return -1;
                const uint32_t word = bits[J >> 5];
                const int64_t rk = rank0 + pref[J >> 5] + __popc(word & ((1u << (J & 31)) - 1u));
                if (q0 + rk >= q1) { dev_error(DEV_ERR_BOUNDS); return -1; }
                return (q0 + rk) * bsz + s.in_row(i) * s.b2 + s.in_col(j);
            };
            if (winner) {
                for_each_entry<ES>(s, I, [&](int64_t p, int64_t i, int64_t j) {
                    const int64_t c = cell_of(i, j);
                    if (c >= 0) atomicMin(&winner[c], (int32_t)p);
                });
                __syncthreads();
                for_each_entry<ES>(s, I, [&](int64_t p, int64_t i, int64_t j) {
                    const int64_t c = cell_of(i, j);
                    if (c >= 0 && winner[c] == (int32_t)p) copy_val<ES>(bval, c, s.val, p);
                });
            } else if (s.rowptr) {
                // CSR: the same cell in 32-bit arithmetic (block ranks < nnzb < 2^31)
                const int w0i = (int)w0, rank0i = (int)rank0;
                for_each_csr_row_sync<ES>(s, I, [&](int p, int64_t i, int j, bool ok) {
                    if (!ok) return;
                    const int J = s.blk_col32(j) - w0i;
                    if ((unsigned)J >= (unsigned)kWinBits) return;
                    const uint32_t word = bits[J >> 5];
                    const int rk = rank0i + pref[J >> 5] + __popc(word & ((1u << (J & 31)) - 1u));
                    if (q0 + rk >= q1) { dev_error(DEV_ERR_BOUNDS); return; }
                    copy_val<ES>(bval, (q0 + rk) * bsz + s.in_row(i) * s.b2 + s.in_col32(j), s.val, p);
                });
            } else {
                for_each_entry<ES>(s, I, [&](int64_t p, int64_t i, int64_t j) {
                    const int64_t c = cell_of(i, j);
                    if (c >= 0) copy_val<ES>(bval, c, s.val, p);
                });
            }
            rank0 += carry;
            __syncthreads();
        }
    }
}

// COO bucketing by block row.
__global__ void coo_bucket_count(int64_t nnz, const int32_t *__restrict__ rows,
                                 const void *__restrict__ val, int es, int b1, int base,
                                 int64_t m, int32_t *__restrict__ cnt) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < nnz; p += stride) {
        if (is_zero(val, es, p)) continue;
        const int64_t i = (int64_t)rows[p] - base;
        if (i < 0 || i >= m) { dev_error(DEV_ERR_BOUNDS); continue; }
        atomicAdd(&cnt[i / b1], 1);
    }
}

__global__ void coo_bucket_scatter(int64_t nnz, const int32_t *__restrict__ rows,
                                   const void *__restrict__ val, int es, int b1, int base,
                                   int64_t m, int32_t *__restrict__ cursor,
                                   int32_t *__restrict__ bent) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < nnz; p += stride) {
        if (is_zero(val, es, p)) continue;
        const int64_t i = (int64_t)rows[p] - base;
        if (i < 0 || i >= m) continue;
        bent[atomicAdd(&cursor[i / b1], 1)] = (int32_t)p;
    }
}

__global__ void check_cols(int64_t nnz, const int32_t *__restrict__ cols, int base, int64_t n) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < nnz; p += stride) {
        const int64_t j = (int64_t)cols[p] - base;
        if (j < 0 || j >= n) dev_error(DEV_ERR_BOUNDS);
    }
}

inline unsigned grid_for(int64_t items, int per = 256) {
    const int64_t g = ceil_div(items > 0 ? items : 1, per);
    return (unsigned)(g < 148 * 32 ? g : 148 * 32);
}

// Instantiates a conversion kernel for the value size of `es`.
#define JLB_CONV_LAUNCH(kernel, es, grid, st, ...)                                      \
    do {                                                                                 \
        if ((es) == 8) conv::kernel<8><<<(grid), conv::kConvThreads, 0, (st)>>>(__VA_ARGS__); \
        else if ((es) == 4) conv::kernel<4><<<(grid), conv::kConvThreads, 0, (st)>>>(__VA_ARGS__); \
        else conv::kernel<2><<<(grid), conv::kConvThreads, 0, (st)>>>(__VA_ARGS__);      \
    } while (0)

inline unsigned grid_rows(int64_t mb) { return (unsigned)(mb < 148 * 64 ? (mb > 0 ? mb : 1) : 148 * 64); }

}  // namespace conv

// Workspace carving helper: 256-byte aligned sub-buffers.
struct Carve {
    char *base;
    size_t off = 0;
    template <typename T>
    T *take(size_t count) {
        off = (off + 255) & ~(size_t)255;
        T *p = reinterpret_cast<T *>(base ? base + off : nullptr);
        off += count * sizeof(T);
        return p;
    }
};

}  // namespace jlb

using namespace jlb;

static int conv_args(int dtype, int idx_base, int64_t m, int64_t n, int64_t nnz, int b1, int b2) {
    if (dtype_size(dtype) == 0) return fail(JLB_ERR_UNSUPPORTED_VALUE_TYPE, "bad dtype %d", dtype);
    if (idx_base != 0 && idx_base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (m < 0 || n < 0 || nnz < 0) return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "negative extent");
    if (b1 <= 0 || b2 <= 0) return fail(JLB_ERR_UNSUPPORTED_FORMAT, "block size must be positive");
    if (nnz > INT32_MAX - 1) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "nnz exceeds Int32 positions");
    if (ceil_div(n, b2) > INT32_MAX - 1) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "block columns exceed Int32");
    return JLB_OK;
}

extern "C" JLB_API size_t jlb_scan_workspace_size(int64_t n) { return conv::scan_ws(n); }

extern "C" JLB_API int jlb_exclusive_scan_i32(void *stream, int64_t n, const int32_t *counts,
                                              int32_t *out, int idx_base, void *workspace,
                                              size_t workspace_bytes) {
    if (n < 0) return fail(JLB_ERR_INVALID_ARGUMENT, "negative length");
    if (!out || (n > 0 && !counts)) return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    return conv::scan(as_stream(stream), n, counts, out, idx_base, workspace, workspace_bytes);
}

// ------------------------------------------------------------------ CSR -> BSR
// Workspace: [scan scratch | stamp | block-column bitmaps (when handed over)].
constexpr size_t kMaxCarryBytes = (size_t)256 << 20;

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

static size_t carry_bytes(int64_t m, int64_t n, int b1, int b2) {
    const int64_t mb = ceil_div(m, b1), nb = ceil_div(n, b2);
    if (nb > conv::kWinBits || mb <= 0) return 0;
    const size_t bytes = (size_t)mb * (size_t)ceil_div(nb, 32) * 4;
    return bytes <= kMaxCarryBytes ? bytes : 0;
}

static size_t csr_scan_ws(int64_t m, int b1) { return align256(conv::scan_ws(ceil_div(m, b1)) + 256); }

static size_t csr_ws(int64_t m, int64_t n, int b1, int b2) {
    const size_t cb = carry_bytes(m, n, b1, b2);
    return cb ? csr_scan_ws(m, b1) + 256 + cb : csr_scan_ws(m, b1);
}

static uint64_t carry_key(int64_t m, int64_t n, int64_t nnz, int b1, int b2, int base, int dtype,
                          const void *rowptr, const void *colind, const void *val) {
    uint64_t h = 0x9e3779b97f4a7c15ull;
    const uint64_t parts[10] = {(uint64_t)m, (uint64_t)n, (uint64_t)nnz, (uint64_t)b1,
                                (uint64_t)b2, (uint64_t)base, (uint64_t)dtype,
                                (uint64_t)(uintptr_t)rowptr, (uint64_t)(uintptr_t)colind,
                                (uint64_t)(uintptr_t)val};
    for (uint64_t v : parts) {
        h ^= v + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
        h *= 0xbf58476d1ce4e5b9ull;
    }
    return h | 1ull;   // never 0: a zeroed workspace never matches
}

// The hand-over region of a CSR workspace, or {null} when it is too small or
// the matrix needs more than one bitmap window.
static conv::Carry csr_carry(void *ws, size_t wsb, int64_t m, int64_t n, int64_t nnz, int b1,
                             int b2, int base, int dtype, const void *rowptr, const void *colind,
                             const void *val) {
    conv::Carry c{nullptr, nullptr, 0};
    const size_t cb = carry_bytes(m, n, b1, b2);
    const size_t scan = csr_scan_ws(m, b1);
    if (!cb || !ws || wsb < scan + 256 + cb) return c;
    char *p = reinterpret_cast<char *>(ws);
    c.stamp = reinterpret_cast<uint64_t *>(p + scan);
    c.bits = reinterpret_cast<uint32_t *>(p + scan + 256);
    c.key = carry_key(m, n, nnz, b1, b2, base, dtype, rowptr, colind, val);
    return c;
}

extern "C" JLB_API size_t jlb_csr_to_bsr_workspace_size(int64_t m, int64_t n, int64_t nnz, int b1,
                                                        int b2) {
    return b1 > 0 && b2 > 0 ? csr_ws(m, n, b1, b2) : 0;
}

static conv::Src csr_src(int dtype, int idx_base, int64_t m, int64_t n, const int32_t *rowptr,
                         const int32_t *colind, const void *val, int b1, int b2) {
    conv::Src s{};
    s.rowptr = rowptr; s.rows = nullptr; s.cols = colind; s.val = val;
    s.boffs = nullptr; s.bent = nullptr; s.m = m; s.n = n;
    s.b1 = b1; s.b2 = b2; s.base = idx_base; s.es = (int)dtype_size(dtype);
    s.sh1 = conv::log2_exact(b1); s.sh2 = conv::log2_exact(b2);
    return s;
}

static int finish_count(cudaStream_t st, int64_t mb, int idx_base, int32_t *browptr,
                        int64_t *nnzb, void *ws, size_t wsb, int *dev_bits) {
    // browptr[1..mb] holds the counts: scan in place.
    int r = conv::scan(st, mb, browptr + 1, browptr, idx_base, ws, wsb);
    if (r) return r;
    int32_t last = 0;
    JLB_CUDA(cudaMemcpyAsync(&last, browptr + mb, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    JLB_CUDA(cudaStreamSynchronize(st));
    const int bits = take_dev_error_convert();
    if (dev_bits) *dev_bits = bits;
    if (bits < 0) return fail(JLB_ERR_CUDA, "reading the device error word failed");
    if (bits & DEV_ERR_BOUNDS)
        return fail(JLB_ERR_NONCANONICAL_STORAGE, "coordinate outside the matrix extents");
    if (bits & DEV_ERR_OVERFLOW)
        return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "block count overflows Int32 positions");
    *nnzb = (int64_t)last - idx_base;
    return ok();
}

extern "C" JLB_API int jlb_csr_to_bsr_count(void *stream, int dtype, int idx_base, int64_t m,
                                            int64_t n, int64_t nnz, const int32_t *rowptr,
                                            const int32_t *colind, const void *val, int b1,
                                            int b2, int32_t *browptr, int64_t *nnzb,
                                            void *workspace, size_t workspace_bytes) {
    int r = conv_args(dtype, idx_base, m, n, nnz, b1, b2);
    if (r) return r;
    if (!browptr || !nnzb || !rowptr || (nnz > 0 && (!colind || !val)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    if (workspace_bytes < csr_scan_ws(m, b1)) return fail(JLB_ERR_WORKSPACE, "workspace too small");
    cudaStream_t st = as_stream(stream);
    const int64_t mb = ceil_div(m, b1), nb = ceil_div(n, b2);
    if (mb > 0) {
        JLB_CONV_LAUNCH(count_blocks, dtype_size(dtype), conv::grid_rows(mb), st,
                        csr_src(dtype, idx_base, m, n, rowptr, colind, val, b1, b2), mb, nb,
                        browptr + 1,
                        csr_carry(workspace, workspace_bytes, m, n, nnz, b1, b2, idx_base, dtype,
                                  rowptr, colind, val));
        JLB_LAUNCH_CHECK("count_blocks");
    }
    return finish_count(st, mb, idx_base, browptr, nnzb, workspace, workspace_bytes, nullptr);
}

extern "C" JLB_API int jlb_csr_to_bsr_fill(void *stream, int dtype, int idx_base, int64_t m,
                                           int64_t n, int64_t nnz, const int32_t *rowptr,
                                           const int32_t *colind, const void *val, int b1, int b2,
                                           const int32_t *browptr, int64_t nnzb, int32_t *bcolind,
                                           void *bval, void *workspace, size_t workspace_bytes) {
    int r = conv_args(dtype, idx_base, m, n, nnz, b1, b2);
    if (r) return r;
    if (!browptr || !rowptr || (nnz > 0 && (!colind || !val)) || (nnzb > 0 && (!bcolind || !bval)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    if (nnzb < 0) return fail(JLB_ERR_INVALID_ARGUMENT, "negative nnzb");
    const int64_t mb = ceil_div(m, b1), nb = ceil_div(n, b2);
    if (mb == 0) return ok();
    cudaStream_t st = as_stream(stream);
    JLB_CONV_LAUNCH(fill_blocks, dtype_size(dtype), conv::grid_rows(mb), st,
                    csr_src(dtype, idx_base, m, n, rowptr, colind, val, b1, b2), mb, nb, nnzb,
                    browptr, bcolind, bval, nullptr,
                    csr_carry(workspace, workspace_bytes, m, n, nnz, b1, b2, idx_base, dtype,
                              rowptr, colind, val));
    JLB_LAUNCH_CHECK("fill_blocks");
    return ok();
}

// ------------------------------------------------------------------ COO -> BSR
static size_t coo_ws(int64_t m, int64_t nnz, int b1, int b2, int64_t nnzb, Carve *c) {
    const int64_t mb = ceil_div(m, b1);
    Carve k = c ? *c : Carve{nullptr};
    k.take<int32_t>((size_t)mb + 1);          // bucket offsets
    k.take<int32_t>((size_t)(mb > 0 ? mb : 1));  // cursors
    k.take<int32_t>((size_t)(nnz > 0 ? nnz : 1));  // bucketed entries
    k.take<char>(conv::scan_ws(mb > 0 ? mb : 1));
    k.take<int32_t>((size_t)(nnzb > 0 ? nnzb : 0) * (size_t)b1 * (size_t)b2);  // winners
    return k.off + 256;
}

extern "C" JLB_API size_t jlb_coo_to_bsr_workspace_size(int64_t m, int64_t n, int64_t nnz, int b1,
                                                        int b2, int64_t nnzb) {
    if (b1 <= 0 || b2 <= 0) return 0;
    return coo_ws(m, nnz, b1, b2, nnzb, nullptr);
}

// Buckets the nonzero COO entries by block row; returns the bucket arrays.
static int coo_bucket(cudaStream_t st, int dtype, int idx_base, int64_t m, int64_t n, int64_t nnz,
                      const int32_t *rows, const int32_t *cols, const void *val, int b1,
                      void *ws, int32_t **boffs, int32_t **bent) {
    const int64_t mb = ceil_div(m, b1);
    const int es = (int)dtype_size(dtype);
    Carve k{reinterpret_cast<char *>(ws)};
    int32_t *offs = k.take<int32_t>((size_t)mb + 1);
    int32_t *cur = k.take<int32_t>((size_t)(mb > 0 ? mb : 1));
    int32_t *ent = k.take<int32_t>((size_t)(nnz > 0 ? nnz : 1));
    const size_t sws = conv::scan_ws(mb > 0 ? mb : 1);
    char *scan_ws = k.take<char>(sws);
    JLB_CUDA(cudaMemsetAsync(offs, 0, sizeof(int32_t) * ((size_t)mb + 1), st));
    if (nnz > 0) {
        conv::check_cols<<<conv::grid_for(nnz), 256, 0, st>>>(nnz, cols, idx_base, n);
        conv::coo_bucket_count<<<conv::grid_for(nnz), 256, 0, st>>>(nnz, rows, val, es, b1,
                                                                     idx_base, m, offs + 1);
        JLB_LAUNCH_CHECK("coo_bucket_count");
    }
    int r = conv::scan(st, mb, offs + 1, offs, 0, scan_ws, sws);
    if (r) return r;
    if (mb > 0) JLB_CUDA(cudaMemcpyAsync(cur, offs, sizeof(int32_t) * (size_t)mb, cudaMemcpyDeviceToDevice, st));
    if (nnz > 0) {
        conv::coo_bucket_scatter<<<conv::grid_for(nnz), 256, 0, st>>>(nnz, rows, val, es, b1,
                                                                       idx_base, m, cur, ent);
        JLB_LAUNCH_CHECK("coo_bucket_scatter");
    }
    *boffs = offs;
    *bent = ent;
    return ok();
}

static conv::Src coo_src(int dtype, int idx_base, int64_t m, int64_t n, const int32_t *rows,
                         const int32_t *cols, const void *val, int b1, int b2,
                         const int32_t *boffs, const int32_t *bent) {
    conv::Src s{};
    s.rowptr = nullptr; s.rows = rows; s.cols = cols; s.val = val;
    s.boffs = boffs; s.bent = bent; s.m = m; s.n = n;
    s.b1 = b1; s.b2 = b2; s.base = idx_base; s.es = (int)dtype_size(dtype);
    s.sh1 = conv::log2_exact(b1); s.sh2 = conv::log2_exact(b2);
    return s;
}

extern "C" JLB_API int jlb_coo_to_bsr_count(void *stream, int dtype, int idx_base, int64_t m,
                                            int64_t n, int64_t nnz, const int32_t *rows,
                                            const int32_t *cols, const void *val, int b1, int b2,
                                            int32_t *browptr, int64_t *nnzb, void *workspace,
                                            size_t workspace_bytes) {
    int r = conv_args(dtype, idx_base, m, n, nnz, b1, b2);
    if (r) return r;
    if (!browptr || !nnzb || (nnz > 0 && (!rows || !cols || !val)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    if (!workspace || workspace_bytes < coo_ws(m, nnz, b1, b2, 0, nullptr))
        return fail(JLB_ERR_WORKSPACE, "workspace too small for the count phase");
    cudaStream_t st = as_stream(stream);
    const int64_t mb = ceil_div(m, b1), nb = ceil_div(n, b2);
    int32_t *boffs, *bent;
    r = coo_bucket(st, dtype, idx_base, m, n, nnz, rows, cols, val, b1, workspace, &boffs, &bent);
    if (r) return r;
    if (mb > 0) {
        JLB_CONV_LAUNCH(count_blocks, dtype_size(dtype), conv::grid_rows(mb), st,
                        coo_src(dtype, idx_base, m, n, rows, cols, val, b1, b2, boffs, bent), mb,
                        nb, browptr + 1, conv::Carry{nullptr, nullptr, 0});
        JLB_LAUNCH_CHECK("count_blocks");
    }
    // The bucket scan already used the scan workspace; reuse it for browptr.
    Carve k{reinterpret_cast<char *>(workspace)};
    k.take<int32_t>((size_t)mb + 1);
    k.take<int32_t>((size_t)(mb > 0 ? mb : 1));
    k.take<int32_t>((size_t)(nnz > 0 ? nnz : 1));
    const size_t sws = conv::scan_ws(mb > 0 ? mb : 1);
    char *scan_ws = k.take<char>(sws);
    return finish_count(st, mb, idx_base, browptr, nnzb, scan_ws, sws, nullptr);
}

extern "C" JLB_API int jlb_coo_to_bsr_fill(void *stream, int dtype, int idx_base, int64_t m,
                                           int64_t n, int64_t nnz, const int32_t *rows,
                                           const int32_t *cols, const void *val, int b1, int b2,
                                           const int32_t *browptr, int64_t nnzb, int32_t *bcolind,
                                           void *bval, void *workspace, size_t workspace_bytes) {
    int r = conv_args(dtype, idx_base, m, n, nnz, b1, b2);
    if (r) return r;
    if (!browptr || (nnz > 0 && (!rows || !cols || !val)) || (nnzb > 0 && (!bcolind || !bval)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    if (nnzb < 0) return fail(JLB_ERR_INVALID_ARGUMENT, "negative nnzb");
    if (!workspace || workspace_bytes < coo_ws(m, nnz, b1, b2, nnzb, nullptr))
        return fail(JLB_ERR_WORKSPACE, "workspace too small for the fill phase");
    cudaStream_t st = as_stream(stream);
    const int64_t mb = ceil_div(m, b1), nb = ceil_div(n, b2);
    if (mb == 0) return ok();
    int32_t *boffs, *bent;
    r = coo_bucket(st, dtype, idx_base, m, n, nnz, rows, cols, val, b1, workspace, &boffs, &bent);
    if (r) return r;
    Carve k{reinterpret_cast<char *>(workspace)};
    k.take<int32_t>((size_t)mb + 1);
    k.take<int32_t>((size_t)mb);
    k.take<int32_t>((size_t)(nnz > 0 ? nnz : 1));
    k.take<char>(conv::scan_ws(mb));
    int32_t *winner = k.take<int32_t>((size_t)nnzb * (size_t)b1 * (size_t)b2);
    JLB_CONV_LAUNCH(fill_blocks, dtype_size(dtype), conv::grid_rows(mb), st,
                    coo_src(dtype, idx_base, m, n, rows, cols, val, b1, b2, boffs, bent), mb, nb,
                    nnzb, browptr, bcolind, bval, winner, conv::Carry{nullptr, nullptr, 0});
    JLB_LAUNCH_CHECK("fill_blocks");
    return ok();
}

// ------------------------------------------------- allocation-free scan
// A variant of jlb_exclusive_scan_i32 for callers that cannot allocate device
// memory: its scratch (one int64 partial sum per 2048 counts) lives in this
// file-scope device array instead of a caller workspace.  The array exists on
// every GPU that loads the library, for the life of the process.
namespace jlb {
namespace conv {

constexpr int64_t kNoAllocTiles = 16384;                    // 128 KB of scratch
constexpr int64_t kNoAllocMaxN = kNoAllocTiles * kScanTile; // 33,554,432 counts

static __device__ __align__(256) int64_t g_scan_noalloc_sums[kNoAllocTiles];

// Device address of g_scan_noalloc_sums on the current device.  The name of
// the array is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
static int noalloc_scratch(void **ptr) {
    constexpr int kMaxDevices = 64;
    static void *cache[kMaxDevices] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    JLB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(JLB_ERR_DEVICE_MISMATCH, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_scan_noalloc_sums);
        if (e != cudaSuccess) return cuda_check(e, "cudaGetSymbolAddress(g_scan_noalloc_sums)");
        cache[dev] = p;
    }
    *ptr = cache[dev];
    return JLB_OK;
}

}  // namespace conv
}  // namespace jlb

extern "C" JLB_API int jlb_exclusive_scan_i32_noalloc(void *stream, int64_t n,
                                                      const int32_t *counts, int32_t *out,
                                                      int idx_base) {
    if (n < 0) return fail(JLB_ERR_INVALID_ARGUMENT, "negative length");
    if (n > conv::kNoAllocMaxN)
        return fail(JLB_ERR_INVALID_ARGUMENT,
                    "jlb_exclusive_scan_i32_noalloc: n = %lld exceeds the static scratch limit of "
                    "%lld counts; use jlb_exclusive_scan_i32 with a workspace",
                    (long long)n, (long long)conv::kNoAllocMaxN);
    if (!out || (n > 0 && !counts)) return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    void *scratch = nullptr;
    int r = conv::noalloc_scratch(&scratch);
    if (r) return r;
    // Every partial sum the kernels read is written earlier in the same call,
    // so the scratch needs no clearing between calls.
    return conv::scan(as_stream(stream), n, counts, out, idx_base, scratch,
                      (size_t)conv::kNoAllocTiles * sizeof(int64_t));
}
