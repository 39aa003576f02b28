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

}  // namespace jlb

#include "sort.cuh"

namespace jlb {

namespace conv {

constexpr int kThreads = 256;
constexpr int kConvThreads = 1024;   // threads of the CSR/COO -> BSR kernels (one CTA per block row)
constexpr int kScanItems = 16;
constexpr int kScanTile = kThreads * kScanItems;   // 4096 counts per tile
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

// Reduce-then-scan over tiles of kScanTile counts, three launches and no
// waits between CTAs.  Counts are read in striped order (coalesced); the final
// pass stages its tile in shared memory so that each thread scans kScanItems
// consecutive counts, and stores the tile back striped.
constexpr int kScanSumThreads = 1024;

__device__ __forceinline__ int scan_pad(int i) { return i + (i >> 5); }   // one word per 32: no bank conflicts

// Programmatic dependent launch between the three scan kernels: each lets
// the next grid be scheduled once all its CTAs have started, and the next
// waits for this grid's completion (griddepcontrol.wait, a no-op when
// launched normally) before it reads what this one wrote.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads)
scan_tile_sums(int64_t n, const int32_t *__restrict__ counts, int64_t *__restrict__ sums) {
    __shared__ int64_t s_warp[kThreads / kWarp];
    pdl_trigger();
    const int64_t t0 = (int64_t)blockIdx.x * kScanTile;
    int64_t v = 0;
    if (t0 + kScanTile <= n && (reinterpret_cast<uintptr_t>(counts) & 15) == 0) {
        // four 16-byte loads a thread, striped
        const int4 *c4 = reinterpret_cast<const int4 *>(counts + t0);
#pragma unroll
        for (int j = 0; j < kScanItems / 4; ++j) {
            const int4 q = __ldg(c4 + j * kThreads + threadIdx.x);
            v += (int64_t)q.x + q.y + q.z + q.w;
        }
    } else if (t0 + kScanTile <= n) {
#pragma unroll
        for (int j = 0; j < kScanItems; ++j) v += ldg(counts + t0 + j * kThreads + threadIdx.x);
    } else {
#pragma unroll
        for (int j = 0; j < kScanItems; ++j) {
            const int64_t i = t0 + j * kThreads + threadIdx.x;
            if (i < n) v += ldg(counts + i);
        }
    }
    int64_t total;
    block_exclusive_scan(v, s_warp, total);
    if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// Exclusive scan of the tile sums in place by one CTA: each thread adds a
// contiguous chunk, one block scan of the chunk totals, then each thread
// rewrites its chunk.
__global__ void __launch_bounds__(kScanSumThreads)
scan_sums_single(int64_t ntiles, int64_t *__restrict__ sums) {
    __shared__ int64_t s_warp[kScanSumThreads / kWarp];
    pdl_trigger();
    pdl_wait();
    const int64_t per = (ntiles + kScanSumThreads - 1) / kScanSumThreads;
    const int64_t c0 = threadIdx.x * per, c1 = c0 + per < ntiles ? c0 + per : ntiles;
    int64_t v = 0;
    int64_t i = c0;
    for (; i + 4 <= c1; i += 4) {   // four loads in flight
        const int64_t a = sums[i], b = sums[i + 1], c = sums[i + 2], d = sums[i + 3];
        v += a + b + c + d;
    }
    for (; i < c1; ++i) v += sums[i];
    int64_t total;
    int64_t run = block_exclusive_scan<kScanSumThreads>(v, s_warp, total);
    for (int64_t i = c0; i < c1; ++i) {
        const int64_t x = sums[i];
        sums[i] = run;
        run += x;
    }
}

__global__ void __launch_bounds__(kThreads, 6)
scan_tiles_final(int64_t n, const int32_t *counts, int32_t *out, const int64_t *__restrict__ sums,
                 int base) {
    __shared__ int64_t s_warp[kThreads / kWarp];
    __shared__ int32_t s_tile[kScanTile + kScanTile / 32];
    const int64_t t0 = (int64_t)blockIdx.x * kScanTile;
    const bool full = t0 + kScanTile <= n;
    // `out` may alias `counts + 1`: this CTA reads exactly the counts whose
    // outputs it writes, all before the barrier below.  The counts are the
    // caller's input: they are read before waiting for the tile sums.
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const int k = j * kThreads + threadIdx.x;
        s_tile[scan_pad(k)] = (full || t0 + k < n) ? counts[t0 + k] : 0;
    }
    pdl_wait();
    const int64_t offset = sums[blockIdx.x] + base;
    __syncthreads();
    // the thread's counts are read from shared memory twice rather than held
    // in registers: at most 40 registers a thread, six CTAs an SM
    int64_t v = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) v += s_tile[scan_pad(threadIdx.x * kScanItems + j)];
    int64_t total;
    int64_t run = block_exclusive_scan(v, s_warp, total) + offset;
    bool over = false;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const int q = scan_pad(threadIdx.x * kScanItems + j);
        run += s_tile[q];
        over |= run > INT32_MAX;
        s_tile[q] = (int32_t)run;   // inclusive: out[i + 1]
    }
    if (over) dev_error(DEV_ERR_OVERFLOW);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const int k = j * kThreads + threadIdx.x;
        if (full || t0 + k < n) out[t0 + k + 1] = s_tile[scan_pad(k)];
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) out[0] = base;
}

// The final pass when `out` does not overlap `counts` and both are 16-byte
// aligned: tile t writes out[t0 .. t0 + kScanTile) (the exclusive values of
// its own counts; out[t0] is the tile's offset) with 16-byte stores, the
// last tile also out[n].  Loads and stores are 16-byte vectors, striped.
__global__ void __launch_bounds__(kThreads, 6)
scan_tiles_final_aligned(int64_t n, const int32_t *__restrict__ counts, int32_t *__restrict__ out,
                         const int64_t *__restrict__ sums, int base) {
    __shared__ int64_t s_warp[kThreads / kWarp];
    __shared__ int32_t s_tile[kScanTile + kScanTile / 32];
    const int64_t t0 = (int64_t)blockIdx.x * kScanTile;
    const bool full = t0 + kScanTile <= n;
    if (full) {
        const int4 *c4 = reinterpret_cast<const int4 *>(counts + t0);
#pragma unroll
        for (int j = 0; j < kScanItems / 4; ++j) {
            const int k = 4 * (j * kThreads + threadIdx.x);
            const int4 q = __ldg(c4 + j * kThreads + threadIdx.x);
            s_tile[scan_pad(k)] = q.x;
            s_tile[scan_pad(k + 1)] = q.y;
            s_tile[scan_pad(k + 2)] = q.z;
            s_tile[scan_pad(k + 3)] = q.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < kScanItems; ++j) {
            const int k = j * kThreads + threadIdx.x;
            s_tile[scan_pad(k)] = t0 + k < n ? __ldg(counts + t0 + k) : 0;
        }
    }
    pdl_wait();
    const int64_t offset = sums[blockIdx.x] + base;
    __syncthreads();
    int64_t v = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) v += s_tile[scan_pad(threadIdx.x * kScanItems + j)];
    int64_t total;
    int64_t run = block_exclusive_scan(v, s_warp, total) + offset;
    bool over = false;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const int q = scan_pad(threadIdx.x * kScanItems + j);
        const int32_t c = s_tile[q];
        over |= run > INT32_MAX;
        s_tile[q] = (int32_t)run;   // exclusive: out[t0 + k]
        run += c;
    }
    if (over) dev_error(DEV_ERR_OVERFLOW);
    if (!full && threadIdx.x == kThreads - 1) {
        if (run > INT32_MAX) dev_error(DEV_ERR_OVERFLOW);
        out[n] = (int32_t)run;   // the last tile: the total
    } else if (full && t0 + kScanTile == n && threadIdx.x == kThreads - 1) {
        if (run > INT32_MAX) dev_error(DEV_ERR_OVERFLOW);
        out[n] = (int32_t)run;
    }
    __syncthreads();
    if (full) {
        int4 *o4 = reinterpret_cast<int4 *>(out + t0);
#pragma unroll
        for (int j = 0; j < kScanItems / 4; ++j) {
            const int k = 4 * (j * kThreads + threadIdx.x);
            o4[j * kThreads + threadIdx.x] = make_int4(s_tile[scan_pad(k)], s_tile[scan_pad(k + 1)],
                                                       s_tile[scan_pad(k + 2)], s_tile[scan_pad(k + 3)]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < kScanItems; ++j) {
            const int k = j * kThreads + threadIdx.x;
            if (t0 + k < n) out[t0 + k] = s_tile[scan_pad(k)];
        }
    }
}

__global__ void scan_write_base(int32_t *out, int base) { out[0] = base; }

size_t scan_ws(int64_t n) { return (size_t)(ceil_div(n > 0 ? n : 1, kScanTile) * sizeof(int64_t)); }

int scan(cudaStream_t st, int64_t n, const int32_t *counts, int32_t *out, int base, void *ws,
         size_t ws_bytes) {
    if (ws_bytes < scan_ws(n) || (!ws && n > 0))
        return fail(JLB_ERR_WORKSPACE, "scan workspace %zu < %zu bytes", ws_bytes, scan_ws(n));
    if (n == 0) {
        // out[0] = base by a kernel on the stream: no host buffer to outlive
        // an async copy, no synchronisation, and capturable in a graph.
        scan_write_base<<<1, 1, 0, st>>>(out, base);
        JLB_LAUNCH_CHECK("exclusive_scan (empty)");
        return ok();
    }
    const int64_t ntiles = ceil_div(n, kScanTile);
    int64_t *sums = (int64_t *)ws;
    scan_tile_sums<<<(unsigned)ntiles, kThreads, 0, st>>>(n, counts, sums);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kScanSumThreads);
    JLB_CUDA(cudaLaunchKernelEx(&cfg, scan_sums_single, ntiles, sums));
    cfg.gridDim = dim3((unsigned)ntiles);
    cfg.blockDim = dim3(kThreads);
    // out[0 .. n] and counts[0 .. n) apart: aligned 16-byte stores of the
    // exclusive values; otherwise (in place, out == counts - 1, or unaligned)
    // each tile writes the inclusive values of its own counts
    const char *cb = reinterpret_cast<const char *>(counts), *ob = reinterpret_cast<const char *>(out);
    const bool apart = ob + (size_t)(n + 1) * 4 <= cb || cb + (size_t)n * 4 <= ob;
    if (apart && aligned16(counts) && aligned16(out))
        JLB_CUDA(cudaLaunchKernelEx(&cfg, scan_tiles_final_aligned, n, counts, out,
                                    (const int64_t *)sums, base));
    else
        JLB_CUDA(cudaLaunchKernelEx(&cfg, scan_tiles_final, n, counts, out, (const int64_t *)sums,
                                    base));
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

template <int ES>
__device__ __forceinline__ void store_zero(void *dst, int64_t q) {
    if (ES == 8) reinterpret_cast<uint64_t *>(dst)[q] = 0;
    else if (ES == 4) reinterpret_cast<uint32_t *>(dst)[q] = 0;
    else reinterpret_cast<uint16_t *>(dst)[q] = 0;
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
    int64_t nnz;             // CSR: entries in cols / val
    int b1, b2, base, es;
    int sh1, sh2;            // log2(b1), log2(b2) when a power of two, else -1
    int vec;                 // CSR: cols 16-byte aligned (four columns per load)

    __device__ __forceinline__ int64_t blk_col(int64_t j) const { return sh2 >= 0 ? j >> sh2 : j / b2; }
    __device__ __forceinline__ int64_t in_col(int64_t j) const { return sh2 >= 0 ? j & (b2 - 1) : j % b2; }
    __device__ __forceinline__ int64_t in_row(int64_t i) const { return sh1 >= 0 ? i & (b1 - 1) : i % b1; }
    // 32-bit forms for CSR columns (Int32 coordinates)
    __device__ __forceinline__ int blk_col32(int j) const { return sh2 >= 0 ? j >> sh2 : j / b2; }
    __device__ __forceinline__ int in_col32(int j) const { return sh2 >= 0 ? j & (b2 - 1) : j % b2; }
};

// Block column of column j: a shift when the block width is a power of two
// (P2), else a division.
template <bool P2>
__device__ __forceinline__ int blk32(const Src &s, int j) {
    if constexpr (P2) return j >> s.sh2;
    else return j / s.b2;
}

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

// Entries [E0, E1) of a CSR (the rows of one block row, contiguous), marking
// the block columns of window [w0i, w0i + kWinBits) that hold a nonzero
// entry.  The CTA's warps take chunks of kWarp * K entries round robin, K (a
// multiple of 4) consecutive entries a lane (16-byte loads of columns
// when aligned), so every warp has the same share whatever the row lengths.
// A lead is an entry whose block column differs from the entry before it in
// the chunk (the chunk's first entry always leads).  Only leads' values are
// read: when every lead of a chunk is nonzero, every block column of the
// chunk holds a nonzero entry and the leads mark them all (one atomic per run
// of a block column); when some lead is zero the chunk reads all its values
// and marks per nonzero entry.  With desc non-null, adds the number of
// entries whose column is not above the previous entry's (first entry
// excluded) -- row starts included, which the caller accounts for.
template <int ES, int K>
__device__ __forceinline__ void mark_csr_flat(const Src &s, int E0, int E1, int w0i,
                                              uint32_t *bits, int *desc) {
    constexpr int kChunk = kWarp * K;
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int nwarps = blockDim.x / kWarp;
    const unsigned n = (unsigned)(s.n < INT32_MAX ? s.n : INT32_MAX);
    int d = 0;
    auto mark = [&](int J) {
        const int Jw = J - w0i;
        if (Jw >= 0 && Jw < kWinBits) atomicOr(&bits[Jw >> 5], 1u << (Jw & 31));
    };
    for (int g0 = (E0 & ~3) + warp * kChunk; g0 < E1; g0 += nwarps * kChunk) {
        const int g = g0 + K * lane;
        int c[K];
        bool v[K];
#pragma unroll
        for (int u = 0; u < K; ++u) v[u] = g + u >= E0 && g + u < E1;
        if (s.vec && (int64_t)g + K <= s.nnz) {
#pragma unroll
            for (int h = 0; h < K; h += 4) {
                const int4 q = __ldg(reinterpret_cast<const int4 *>(s.cols + g + h));
                c[h] = q.x; c[h + 1] = q.y; c[h + 2] = q.z; c[h + 3] = q.w;
            }
        } else {
#pragma unroll
            for (int u = 0; u < K; ++u) c[u] = v[u] ? __ldg(s.cols + g + u) : 0;
        }
        // the entry before this lane's first: the previous lane's last, or
        // (lane 0) a load
        int prev = __shfl_up_sync(0xffffffffu, c[K - 1], 1);
        const bool has_prev = g - 1 >= E0 && g - 1 < E1;
        if (lane == 0) prev = has_prev ? __ldg(s.cols + g - 1) : 0;
        prev -= s.base;
        int J[K];
#pragma unroll
        for (int u = 0; u < K; ++u) {
            c[u] -= s.base;
            if (v[u] && (unsigned)c[u] >= n) {
                dev_error(DEV_ERR_BOUNDS);
                v[u] = false;
            }
            J[u] = s.blk_col32(c[u]);
        }
        if (desc) {
            if (v[0] && has_prev && c[0] <= prev) ++d;
#pragma unroll
            for (int u = 1; u < K; ++u)
                if (v[u] && v[u - 1] && c[u] <= c[u - 1]) ++d;
        }
        bool lead[K], zero_lead = false;
#pragma unroll
        for (int u = 0; u < K; ++u) {
            const int pj = u > 0 ? (v[u - 1] ? J[u - 1] : -1)
                                 : (lane > 0 && has_prev ? s.blk_col32(prev) : -1);
            lead[u] = v[u] && J[u] != pj;
            if (lead[u] && is_zero<ES>(s.val, g + u)) zero_lead = true;
        }
        if (__any_sync(0xffffffffu, zero_lead)) {
            int pj = -1;
#pragma unroll
            for (int u = 0; u < K; ++u)
                if (v[u] && !is_zero<ES>(s.val, g + u)) {
                    if (J[u] != pj) mark(J[u]);
                    pj = J[u];
                }
        } else {
#pragma unroll
            for (int u = 0; u < K; ++u)
                if (lead[u]) mark(J[u]);
        }
    }
    if (desc) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (lane == 0 && d) atomicAdd(desc, d);
    }
}

// Entry range of block row I of a CSR: [E0, E1).
__device__ __forceinline__ void csr_block_range(const Src &s, int64_t I, int &E0, int &E1) {
    const int64_t i0 = I * s.b1, i1 = i0 + s.b1 < s.m ? i0 + s.b1 : s.m;
    E0 = s.rowptr[i0] - s.base;
    E1 = s.rowptr[i1] - s.base;
}

// Marks the block columns of window [w0, w0 + kWinBits) hit by block row I.
template <int ES>
__device__ __forceinline__ void mark_window(const Src &s, int64_t I, int64_t w0, uint32_t *bits) {
    if (s.rowptr) {
        int E0, E1;
        csr_block_range(s, I, E0, E1);
        mark_csr_flat<ES, 4>(s, E0, E1, (int)w0, bits, nullptr);   // block columns fit 32 bits
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

template <int NT = kConvThreads>
__device__ __forceinline__ int64_t block_sum(int64_t v, int64_t *s_red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x % kWarp == 0) s_red[threadIdx.x / kWarp] = v;
    __syncthreads();
    int64_t t = 0;
    for (int w = 0; w < NT / kWarp; ++w) t += s_red[w];
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
    uint8_t *asc;        // mb flags: every row of the block row strictly ascending
    uint8_t *row_done;   // mb * b1 flags of the fill's tile-row path
    int32_t *row_runs;   // mb * b1: the row's runs of block columns, -1 unknown (count pass)
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

// Nonzero flags of entries g .. g+7 (v: in range), from one, two or four
// 16-byte loads of values when `vec`.
template <int ES>
__device__ __forceinline__ void nonzero8(const Src &s, int g, bool vec, const bool (&v)[8],
                                         bool (&nz)[8]) {
    if (vec) {
        const int4 *q = reinterpret_cast<const int4 *>(static_cast<const char *>(s.val) + (size_t)g * ES);
        if constexpr (ES == 2) {
            const int4 a = __ldg(q);
            const uint32_t w[4] = {(uint32_t)a.x, (uint32_t)a.y, (uint32_t)a.z, (uint32_t)a.w};
#pragma unroll
            for (int u = 0; u < 8; ++u) nz[u] = v[u] && ((w[u >> 1] >> ((u & 1) * 16)) & 0x7fffu) != 0;
        } else if constexpr (ES == 4) {
            const int4 a = __ldg(q), b = __ldg(q + 1);
            const uint32_t w[8] = {(uint32_t)a.x, (uint32_t)a.y, (uint32_t)a.z, (uint32_t)a.w,
                                   (uint32_t)b.x, (uint32_t)b.y, (uint32_t)b.z, (uint32_t)b.w};
#pragma unroll
            for (int u = 0; u < 8; ++u) nz[u] = v[u] && (w[u] & 0x7fffffffu) != 0;
        } else {
            uint32_t w[16];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const int4 a = __ldg(q + h);
                w[4 * h] = a.x; w[4 * h + 1] = a.y; w[4 * h + 2] = a.z; w[4 * h + 3] = a.w;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) nz[u] = v[u] && (w[2 * u] | (w[2 * u + 1] & 0x7fffffffu)) != 0;
        }
    } else {
#pragma unroll
        for (int u = 0; u < 8; ++u) nz[u] = v[u] && !is_zero<ES>(s.val, g + u);
    }
}

// Columns and values of eight consecutive entries g .. g+7 as loaded (16-byte
// loads when aligned and inside the arrays, else the in-range ones singly).
template <int ES>
struct Raw8 {
    int c[8];
    uint32_t w[2 * ES];   // the eight values' bits (vector loads)
    uint32_t nzm;         // nonzero mask (single loads)
    bool vec;

    __device__ __forceinline__ void load(const Src &s, int g, int E0, int E1) {
        vec = s.vec && (int64_t)g + 8 <= s.nnz;
        if (vec) {
            const int4 p0 = __ldg(reinterpret_cast<const int4 *>(s.cols + g));
            const int4 p1 = __ldg(reinterpret_cast<const int4 *>(s.cols + g + 4));
            c[0] = p0.x; c[1] = p0.y; c[2] = p0.z; c[3] = p0.w;
            c[4] = p1.x; c[5] = p1.y; c[6] = p1.z; c[7] = p1.w;
            const int4 *q = reinterpret_cast<const int4 *>(static_cast<const char *>(s.val) + (size_t)g * ES);
#pragma unroll
            for (int h = 0; h < ES / 2; ++h) {
                const int4 a = __ldg(q + h);
                w[4 * h] = a.x; w[4 * h + 1] = a.y; w[4 * h + 2] = a.z; w[4 * h + 3] = a.w;
            }
        } else {
            nzm = 0;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const bool in = g + u >= E0 && g + u < E1;
                c[u] = in ? __ldg(s.cols + g + u) : 0;
                if (in && !is_zero<ES>(s.val, g + u)) nzm |= 1u << u;
            }
        }
    }
    __device__ __forceinline__ void nonzero(const bool (&v)[8], bool (&nz)[8]) const {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            bool z;
            if (!vec) z = !((nzm >> u) & 1u);
            else if (ES == 2) z = ((w[u >> 1] >> ((u & 1) * 16)) & 0x7fffu) == 0;
            else if (ES == 4) z = (w[u] & 0x7fffffffu) == 0;
            else z = (w[2 * u] | (w[2 * u + 1] & 0x7fffffffu)) == 0;
            nz[u] = v[u] && !z;
        }
    }
};

// Entries [E0, E1) of a CSR (the rows of one block row, contiguous), marking
// the block columns of window [w0i, w0i + kWinBits) that hold a nonzero
// entry, for the count pass.  The CTA's warps take chunks of 256 entries
// round robin (chunks aligned to 8 entries), eight consecutive entries a
// lane.
//   Lean chunks -- inside [E0, E1), 16-byte loads, every entry nonzero and in
//   range -- mark only where the block column changes: a lane marks its first
//   entry's block column unless the lane before ended in it, and each entry
//   whose block column differs from the entry before it in the lane (a bit
//   mask; usually empty).
//   Other chunks go entry by entry: an entry marks its block column when it
//   is nonzero and the previous nonzero entry (in the lane, or the lane
//   before) had another one.
// Adds to *desc the number of entries whose column is not above the previous
// entry's (first entry excluded) -- row starts included, which the caller
// accounts for.  With jc non-null, sets bit e - E0 of jc for every entry e
// whose block column differs from the entry before's, and sets *zero_run when
// such an entry is zero.
template <int ES, bool P2>
__device__ __forceinline__ void mark_csr_count(const Src &s, int E0, int E1, int w0i, uint32_t *bits,
                                               int *desc, uint32_t *jc, int *zero_run) {
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int nwarps = blockDim.x / kWarp;
    const unsigned n = (unsigned)(s.n < INT32_MAX ? s.n : INT32_MAX);
    int d = 0;
    auto mark = [&](int J) {
        const int Jw = J - w0i;
        if (Jw >= 0 && Jw < kWinBits) atomicOr(&bits[Jw >> 5], 1u << (Jw & 31));
    };
    auto change_at = [&](int e) { atomicOr(&jc[(e - E0) >> 5], 1u << ((e - E0) & 31)); };
    for (int g0 = (E0 & ~7) + warp * 8 * kWarp; g0 < E1; g0 += nwarps * 8 * kWarp) {
        const int g = g0 + 8 * lane;
        const bool interior = s.vec && g0 >= E0 && g0 + 8 * kWarp <= E1;   // warp-uniform
        {
            // this warp's next chunk into L2 while this one is worked on
            const int64_t gn = (int64_t)g + nwarps * 8 * kWarp;
            if (gn + 8 <= E1) {
                asm volatile("prefetch.global.L2 [%0];" ::"l"(s.cols + gn));
                asm volatile("prefetch.global.L2 [%0];" ::"l"(static_cast<const char *>(s.val) + gn * ES));
            }
        }
        if (interior) {
            const int4 p0 = __ldg(reinterpret_cast<const int4 *>(s.cols + g));
            const int4 p1 = __ldg(reinterpret_cast<const int4 *>(s.cols + g + 4));
            const int4 *q = reinterpret_cast<const int4 *>(static_cast<const char *>(s.val) + (size_t)g * ES);
            bool f = true;
            if constexpr (ES == 2) {
                // a 16-bit half that is +-0: (t - 0x00010001) & ~t & 0x80008000 != 0
                // for t = w & 0x7fff7fff when some half of t is zero (a borrow
                // may flag its neighbour too, which only sends the chunk to the
                // entry-by-entry path)
                const int4 a = __ldg(q);
                const uint32_t w[4] = {(uint32_t)a.x, (uint32_t)a.y, (uint32_t)a.z, (uint32_t)a.w};
                uint32_t z = 0;
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const uint32_t t = w[h] & 0x7fff7fffu;
                    z |= (t - 0x00010001u) & ~t & 0x80008000u;
                }
                f = z == 0;
            } else if constexpr (ES == 4) {
                const int4 a = __ldg(q), b = __ldg(q + 1);
                f = (a.x & 0x7fffffff) && (a.y & 0x7fffffff) && (a.z & 0x7fffffff) &&
                    (a.w & 0x7fffffff) && (b.x & 0x7fffffff) && (b.y & 0x7fffffff) &&
                    (b.z & 0x7fffffff) && (b.w & 0x7fffffff);
            } else {
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const int4 a = __ldg(q + h);
                    f = f && (a.x | (a.y & 0x7fffffff)) && (a.z | (a.w & 0x7fffffff));
                }
            }
            const int cr[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
            int c[8], J[8];
            uint32_t chg = 0;   // bit u: entry u's block column differs from entry u-1's
            int dsc = 0;        // entries not above the one before, inside the lane
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                c[u] = cr[u] - s.base;
                f = f && (unsigned)c[u] < n;
                J[u] = blk32<P2>(s, c[u]);
            }
#pragma unroll
            for (int u = 1; u < 8; ++u) {
                dsc += c[u] <= c[u - 1];
                chg |= (uint32_t)(J[u] != J[u - 1]) << u;
            }
            int prev = __shfl_up_sync(0xffffffffu, p1.w, 1);
            const int upJ = __shfl_up_sync(0xffffffffu, J[7], 1);
            if (__all_sync(0xffffffffu, f)) {
                const bool has_prev = g > E0;
                if (lane == 0 && has_prev) prev = __ldg(s.cols + g - 1);
                d += dsc + (has_prev && p0.x <= prev);   // descents: not above the entry before
                if (lane == 0 || J[0] != upJ) mark(J[0]);
                if (jc && has_prev && J[0] != blk32<P2>(s, prev - s.base)) change_at(g);
                while (chg) {   // usually no bit, at most a few
                    const int u = __ffs(chg) - 1;
                    chg &= chg - 1;
                    const int Ju = u == 1 ? J[1] : u == 2 ? J[2] : u == 3 ? J[3] : u == 4 ? J[4]
                                 : u == 5 ? J[5] : u == 6 ? J[6] : J[7];
                    mark(Ju);
                    if (jc) change_at(g + u);
                }
                continue;
            }
        }
        // entry by entry
        Raw8<ES> cur;
        cur.load(s, g, E0, E1);
        bool v[8], nz[8];
        int c[8], J[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            v[u] = g + u >= E0 && g + u < E1;
            c[u] = cur.c[u];
        }
        cur.nonzero(v, nz);
        const bool has_prev = g - 1 >= E0 && g - 1 < E1;
        int prevc = __shfl_up_sync(0xffffffffu, c[7], 1);
        if (lane == 0) prevc = has_prev ? __ldg(s.cols + g - 1) : 0;
        prevc -= s.base;
        int last_nz = -1;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            c[u] -= s.base;
            if (v[u] && (unsigned)c[u] >= n) {
                dev_error(DEV_ERR_BOUNDS);
                v[u] = nz[u] = false;
            }
            J[u] = blk32<P2>(s, c[u]);
            if (nz[u]) last_nz = J[u];
        }
        const int up_nz = __shfl_up_sync(0xffffffffu, last_nz, 1);
        int pnz = lane == 0 ? -1 : up_nz;
        if (v[0] && has_prev && c[0] <= prevc) ++d;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (u > 0 && v[u] && v[u - 1] && c[u] <= c[u - 1]) ++d;
            if (nz[u] && J[u] != pnz) mark(J[u]);
            if (nz[u]) pnz = J[u];
            if (jc && v[u] && (u > 0 ? v[u - 1] && J[u] != J[u - 1] : has_prev && J[0] != blk32<P2>(s, prevc))) {
                change_at(g + u);
                if (!nz[u]) *zero_run = 1;
            }
        }
    }
    if (desc) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (lane == 0 && d) atomicAdd(desc, d);
    }
}

// Count pass of a CSR source, one block row per CTA of kCsrThreads threads
// (two CTAs an SM): the block row's entries are marked as one flat range
// (mark_csr_count).  With a hand-over it also records what the fill pass's
// tile-row path relies on:
//   * per block row, whether every row's columns strictly ascend: the
//     entries not above their predecessor (counted while marking) must all
//     be row starts, i.e. their number must equal the number of nonempty rows
//     whose first column is not above the last column before it;
//   * per row, its number of runs of block columns -- 1 + the block-column
//     changes after its first entry (the jc bits) -- or -1 when some run
//     starts with a zero (or the block row has too many entries to track).
// Shared memory (dynamic): the block-column bitmap, then the jc bits.
constexpr int kCsrThreads = 512;
constexpr int kJcWords = 8192;     // entries of a block row the change bits cover: 262,144
constexpr size_t kCountSmem = (size_t)(kWinWords + kJcWords) * 4;

template <int ES, bool P2>
__global__ void __launch_bounds__(kCsrThreads, 2)
count_csr(Src s, int64_t mb, int64_t nb, int32_t *__restrict__ counts, Carry carry) {
    extern __shared__ uint32_t dyn_smem[];
    uint32_t *bits = dyn_smem;
    uint32_t *jc = dyn_smem + kWinWords;
    __shared__ int64_t s_red[kCsrThreads / kWarp];
    __shared__ int s_desc, s_zero;
    for (int64_t I = blockIdx.x; I < mb; I += gridDim.x) {
        int E0, E1;
        csr_block_range(s, I, E0, E1);
        const int64_t i0 = I * s.b1;
        const int rows = (int)(s.m - i0 < s.b1 ? s.m - i0 : s.b1);
        const bool runs = carry.bits && E1 - E0 <= kJcWords * 32;
        if (threadIdx.x == 0) s_desc = s_zero = 0;
        if (runs)
            for (int w = threadIdx.x; w < (int)ceil_div(E1 - E0, 32); w += kCsrThreads) jc[w] = 0;
        int64_t total = 0;
        for (int64_t w0 = 0; w0 < nb; w0 += kWinBits) {
            const int nw = (int)ceil_div((nb - w0) < kWinBits ? (nb - w0) : kWinBits, 32);
            for (int w = threadIdx.x; w < nw; w += kCsrThreads) bits[w] = 0;
            __syncthreads();
            mark_csr_count<ES, P2>(s, E0, E1, (int)w0, bits, w0 == 0 ? &s_desc : nullptr,
                                   runs && w0 == 0 ? jc : nullptr, &s_zero);
            __syncthreads();
            int64_t c = 0;
            for (int w = threadIdx.x; w < nw; w += kCsrThreads) {
                c += __popc(bits[w]);
                if (carry.bits) carry.bits[I * nw + w] = bits[w];
            }
            total += block_sum<kCsrThreads>(c, s_red);
        }
        // per row: descent at its start; its runs
        int64_t at_starts = 0;
        for (int r = threadIdx.x; r < rows; r += kCsrThreads) {
            const int lo = s.rowptr[i0 + r] - s.base, hi = s.rowptr[i0 + r + 1] - s.base;
            int nr = 0;
            bool zr = !runs || s_zero;
            if (hi > lo) {
                if (lo > E0 && __ldg(s.cols + lo) <= __ldg(s.cols + lo - 1)) ++at_starts;
                if (runs) {
                    zr = zr || is_zero<ES>(s.val, lo);
                    nr = 1;
                    for (int b = lo - E0 + 1; b < hi - E0;) {   // change bits in (lo, hi)
                        const int w = b >> 5, sh = b & 31;
                        const int take = min(32 - sh, hi - E0 - b);
                        const uint32_t m = take == 32 ? 0xffffffffu : ((1u << take) - 1u) << sh;
                        nr += __popc(jc[w] & m);
                        b += take;
                    }
                }
            }
            if (carry.bits) carry.row_runs[i0 + r] = zr ? -1 : nr;
        }
        at_starts = block_sum<kCsrThreads>(at_starts, s_red);
        if (threadIdx.x == 0) {
            if (total > INT32_MAX) dev_error(DEV_ERR_OVERFLOW);
            counts[I] = (int32_t)total;
            if (carry.bits) carry.asc[I] = (uint8_t)(s_desc == at_starts);
        }
        __syncthreads();
    }
    if (carry.bits && blockIdx.x == 0 && threadIdx.x == 0) *carry.stamp = carry.key;
}

// ---------------------------------------------------------- fill, fast rows
// Value copy with explicit zeros (either sign) written as +0, as the tiles'
// zero padding: U-byte units of ES-byte values.
template <int ES, typename UT>
__device__ __forceinline__ UT plus_zero(UT w);
template <>
__device__ __forceinline__ uint16_t plus_zero<2, uint16_t>(uint16_t w) { return (w & 0x7fffu) ? w : 0; }
__device__ __forceinline__ uint32_t pz2(uint32_t w) {
    uint32_t keep = 0;
    if (w & 0x00007fffu) keep |= 0x0000ffffu;
    if (w & 0x7fff0000u) keep |= 0xffff0000u;
    return w & keep;
}
__device__ __forceinline__ uint32_t pz4(uint32_t w) { return (w & 0x7fffffffu) ? w : 0u; }
__device__ __forceinline__ uint2 pz8(uint2 w) {
    return ((w.x | (w.y & 0x7fffffffu)) != 0) ? w : make_uint2(0u, 0u);
}
template <>
__device__ __forceinline__ uint32_t plus_zero<2, uint32_t>(uint32_t w) { return pz2(w); }
template <>
__device__ __forceinline__ uint32_t plus_zero<4, uint32_t>(uint32_t w) { return pz4(w); }
template <>
__device__ __forceinline__ uint2 plus_zero<2, uint2>(uint2 w) { return make_uint2(pz2(w.x), pz2(w.y)); }
template <>
__device__ __forceinline__ uint2 plus_zero<4, uint2>(uint2 w) { return make_uint2(pz4(w.x), pz4(w.y)); }
template <>
__device__ __forceinline__ uint2 plus_zero<8, uint2>(uint2 w) { return pz8(w); }
template <>
__device__ __forceinline__ uint4 plus_zero<2, uint4>(uint4 w) {
    return make_uint4(pz2(w.x), pz2(w.y), pz2(w.z), pz2(w.w));
}
template <>
__device__ __forceinline__ uint4 plus_zero<4, uint4>(uint4 w) {
    return make_uint4(pz4(w.x), pz4(w.y), pz4(w.z), pz4(w.w));
}
template <>
__device__ __forceinline__ uint4 plus_zero<8, uint4>(uint4 w) {
    const uint2 a = pz8(make_uint2(w.x, w.y)), b = pz8(make_uint2(w.z, w.w));
    return make_uint4(a.x, a.y, b.x, b.y);
}

// Copies `run` consecutive full tile rows: values [p, p + run * b2) of the
// CSR (contiguous) to tile row r of tiles k .. k + run - 1 (dst = tile k's
// row r, tiles tile_bytes apart), in UT units spread over the warp's lanes.
constexpr int kCopyUnroll = 8;   // units a lane loads before storing

template <int ES, typename UT>
__device__ __forceinline__ void copy_tile_rows(char *dst, int64_t tile_bytes, const char *src,
                                               int upr, int upr_sh, int run, int lane) {
    const UT *s = reinterpret_cast<const UT *>(src);
    const int total = run * upr;
    for (int x0 = 0; x0 < total; x0 += kCopyUnroll * kWarp) {
        UT w[kCopyUnroll];
#pragma unroll
        for (int j = 0; j < kCopyUnroll; ++j) {
            const int x = x0 + j * kWarp + lane;
            if (x < total) w[j] = s[x];
        }
#pragma unroll
        for (int j = 0; j < kCopyUnroll; ++j) {
            const int x = x0 + j * kWarp + lane;
            if (x < total) {
                const int t = upr_sh >= 0 ? x >> upr_sh : x / upr;
                const int u = x - t * upr;
                reinterpret_cast<UT *>(dst + (int64_t)t * tile_bytes)[u] = plus_zero<ES, UT>(w[j]);
            }
        }
    }
}

// Zero-fills `bytes` bytes at dst with the warp (UT-aligned dst and size).
template <typename UT>
__device__ __forceinline__ void zero_units(char *dst, int bytes, int lane) {
    UT z;
    memset(&z, 0, sizeof(UT));
    for (int x = lane; x < bytes / (int)sizeof(UT); x += kWarp) reinterpret_cast<UT *>(dst)[x] = z;
}

__device__ __forceinline__ void zero_row(char *dst, int bytes, int lane) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(dst) | (uintptr_t)bytes;
    if ((a & 15) == 0) zero_units<uint4>(dst, bytes, lane);
    else if ((a & 7) == 0) zero_units<uint2>(dst, bytes, lane);
    else if ((a & 3) == 0) zero_units<uint32_t>(dst, bytes, lane);
    else if ((a & 1) == 0) zero_units<uint16_t>(dst, bytes, lane);
    else zero_units<uint8_t>(dst, bytes, lane);
}

// Copies `run` full runs of a row starting at entry p (values [p, p + run *
// b2), contiguous) to tile row r of `run` consecutive tiles (dst = the first
// one's row), in the widest unit the addresses allow.
template <int ES>
__device__ __forceinline__ void copy_row_any(const char *src, char *dst, int64_t tile_bytes, int total,
                                             int upr_sh, int lane);

template <int ES>
__device__ __forceinline__ void copy_runs(const Src &s, int64_t p, char *dst, int64_t tile_bytes,
                                          int run, int lane) {
    const int b2 = s.b2, row_bytes = b2 * ES;
    const char *src = reinterpret_cast<const char *>(s.val) + p * ES;
    const uintptr_t dal = reinterpret_cast<uintptr_t>(dst) | (uintptr_t)row_bytes | (uintptr_t)tile_bytes;
    const uintptr_t al = reinterpret_cast<uintptr_t>(src) | dal;
    auto sh = [](int upr) { return (upr & (upr - 1)) ? -1 : __ffs(upr) - 1; };
    if ((dal & 15) == 0 && sh(row_bytes / 16) >= 0) {
        // 16-byte units on the tile side, any source offset
        copy_row_any<ES>(src, dst, tile_bytes, run * (row_bytes / 16), sh(row_bytes / 16), lane);
    } else if ((al & 15) == 0) {
        copy_tile_rows<ES, uint4>(dst, tile_bytes, src, row_bytes / 16, sh(row_bytes / 16), run, lane);
    } else if ((al & 7) == 0) {
        copy_tile_rows<ES, uint2>(dst, tile_bytes, src, row_bytes / 8, sh(row_bytes / 8), run, lane);
    } else if (ES <= 4 && (al & 3) == 0) {
        if constexpr (ES <= 4)
            copy_tile_rows<ES, uint32_t>(dst, tile_bytes, src, row_bytes / 4, sh(row_bytes / 4), run, lane);
    } else {
        // 2-byte values at odd positions: one value at a time
        for (int t = 0; t < run; ++t)
            for (int c = lane; c < b2; c += kWarp) {
                const int64_t e = p + (int64_t)t * b2 + c;
                if (is_zero<ES>(s.val, e)) store_zero<ES>(dst + (int64_t)t * tile_bytes, c);
                else copy_val<ES>(dst + (int64_t)t * tile_bytes, c, s.val, e);
            }
    }
}

// One row of block row I by runs (the row is ascending): for the block row's
// blocks k (block columns bcol[k], ascending) a tile row is a full run when
// the row's entries from the cursor p are exactly the block's b2 columns --
// with ascending columns that holds iff the first is the block's first
// column and the entry b2 - 1 further is its last.  The 32 lanes test blocks
// k .. k+31 at once, assuming each earlier one a full run, and the warp
// copies the leading full runs as one contiguous stretch of values; a block
// that is not a full run is zeroed and its entries scattered (entries before
// it belong to blocks with only explicit zeros and are skipped).
template <int ES>
__device__ __noinline__ void fill_row_runs(const Src &s, int64_t i, char *row0, int nblk, const int32_t *bcol,
                              int64_t tile_bytes, int lane) {
    const int b2 = s.b2, row_bytes = b2 * ES;
    if (i >= s.m) {   // rows past the matrix: padding
        for (int k = 0; k < nblk; ++k) zero_row(row0 + (int64_t)k * tile_bytes, row_bytes, lane);
        return;
    }
    int64_t p = s.rowptr[i] - s.base;
    const int64_t hi = s.rowptr[i + 1] - s.base;
    int k = 0;
    while (k < nblk) {
        const int kk = k + lane;
        bool full = false;
        if (kk < nblk) {
            const int64_t c0 = (int64_t)(__ldcg(bcol + kk) - s.base) * b2;
            const int64_t ph = p + (int64_t)lane * b2;
            if (ph + b2 <= hi)
                full = (int64_t)(__ldg(s.cols + ph) - s.base) == c0 &&
                       (int64_t)(__ldg(s.cols + ph + b2 - 1) - s.base) == c0 + b2 - 1;
        }
        const unsigned fm = __ballot_sync(0xffffffffu, full);
        const int run = fm == 0xffffffffu ? kWarp : __ffs(~fm) - 1;
        if (run > 0) {
            copy_runs<ES>(s, p, row0 + (int64_t)k * tile_bytes, tile_bytes, run, lane);
            p += (int64_t)run * b2;
            k += run;
        }
        if (run < kWarp && k < nblk) {
            // block k is not a full run of this row: zero its tile row, then
            // scatter the row's entries that fall in it
            const int64_t c0 = (int64_t)(__ldcg(bcol + k) - s.base) * b2;
            char *dst = row0 + (int64_t)k * tile_bytes;
            zero_row(dst, row_bytes, lane);
            __syncwarp();
            for (;;) {
                const int64_t e = p + lane;
                const int64_t c = e < hi ? (int64_t)(__ldg(s.cols + e) - s.base) : INT64_MAX;
                const bool in = c < c0 + b2;   // ascending: a prefix of the lanes
                const int cnt = __popc(__ballot_sync(0xffffffffu, in));
                if (in && c >= c0 && !is_zero<ES>(s.val, e)) copy_val<ES>(dst, c - c0, s.val, e);
                p += cnt;
                if (cnt < kWarp) break;
            }
            __syncwarp();
            ++k;
        }
    }
}

// A CSR block row that the tile-row fill (fill_ascending) takes: the count
// pass handed its bitmap over and found all its rows ascending.
__device__ __forceinline__ bool fast_block_row(const Src &s, const Carry &carry, bool handed,
                                               int64_t I) {
    return handed && s.rowptr && carry.asc[I];
}

// Fill pass.  winner == nullptr means the source has unique coordinates.
// The block rows that fast_block_row() picks are left to fill_ascending.
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
        if (!winner && fast_block_row(s, carry, handed, I)) continue;
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

// Fill of the block rows that fast_block_row() picks, in three launches:
// fill_asc_columns writes their block columns (from the handed-over bitmap:
// one window, as the hand-over implies), fill_whole_rows copies every row
// that is whole -- nblk * b2 entries forming a full run in each of the block
// row's blocks -- and fill_other_rows writes the rest run by run.  Every byte
// of these tiles is written once (no zero fill).  A per-row flag in the
// workspace tells the third launch which rows the second did.
constexpr int kAscThreads = 512;

template <int ES>
__global__ void __launch_bounds__(kAscThreads)
fill_asc_columns(Src s, int64_t mb, int64_t nb, int64_t nnzb, const int32_t *__restrict__ browptr,
                 int32_t *__restrict__ bcolind, Carry carry) {
    const bool handed = carry.bits && *carry.stamp == carry.key;
    if (!handed) return;
    __shared__ uint32_t bits[kWinWords];
    __shared__ int32_t pref[kWinWords];
    __shared__ int64_t s_warp[kAscThreads / kWarp];
    const int nw = (int)ceil_div(nb, 32);
    for (int64_t I = blockIdx.x; I < mb; I += gridDim.x) {
        if (!fast_block_row(s, carry, handed, I)) continue;
        const int64_t q0 = (int64_t)browptr[I] - s.base, q1 = (int64_t)browptr[I + 1] - s.base;
        if (q0 < 0 || q1 < q0 || q1 > nnzb) {
            if (threadIdx.x == 0) dev_error(DEV_ERR_BOUNDS);
            continue;   // write nothing for this block row
        }
        for (int w = threadIdx.x; w < nw; w += kAscThreads) bits[w] = carry.bits[I * nw + w];
        __syncthreads();
        int64_t run = 0;
        for (int c0 = 0; c0 < nw; c0 += kAscThreads) {
            const int w = c0 + threadIdx.x;
            const int64_t v = w < nw ? __popc(bits[w]) : 0;
            int64_t tot;
            const int64_t ex = block_exclusive_scan<kAscThreads>(v, s_warp, tot);
            if (w < nw) pref[w] = (int32_t)(run + ex);
            run += tot;
        }
        __syncthreads();
        if (run != q1 - q0) {   // block row pointer and bitmap disagree
            if (threadIdx.x == 0) dev_error(DEV_ERR_BOUNDS);
            continue;
        }
        for (int w = threadIdx.x; w < nw; w += kAscThreads) {
            uint32_t word = bits[w];
            int r = pref[w];
            while (word) {
                const int b = __ffs(word) - 1;
                word &= word - 1;
                bcolind[q0 + r] = w * 32 + b + s.base;
                ++r;
            }
        }
        __syncthreads();
    }
}

// The block row of row i when fast_block_row() picks it and its block row
// pointer is sane: q0 and nblk; false otherwise.
__device__ __forceinline__ bool asc_row(const Src &s, const Carry &carry, bool handed,
                                        const int32_t *__restrict__ browptr, int64_t nnzb,
                                        int64_t I, int64_t &q0, int &nblk) {
    if (!fast_block_row(s, carry, handed, I)) return false;
    q0 = (int64_t)browptr[I] - s.base;
    const int64_t q1 = (int64_t)browptr[I + 1] - s.base;
    if (q0 < 0 || q1 < q0 || q1 > nnzb) return false;   // reported by fill_asc_columns
    nblk = (int)(q1 - q0);
    return true;
}

// One warp per row (rows of all block rows, padding rows included).  A whole
// row's values are contiguous and its tile rows are nblk * b2 * ES bytes of
// them in order, so the copy is a stream of 16-, 8- or 4-byte units, four in
// flight per lane.  Marks row_done[i] for the rows it wrote.
constexpr int kRowThreads = 256;

template <int ES, typename UT>
__device__ __forceinline__ void copy_row_units(const char *src, char *dst, int64_t tile_bytes,
                                               int total, int upr_sh, int lane) {
    const UT *sp = reinterpret_cast<const UT *>(src);
    const int mask = (1 << upr_sh) - 1;
    for (int x0 = 0; x0 < total; x0 += 4 * kWarp) {
        UT w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int x = x0 + j * kWarp + lane;
            if (x < total) w[j] = __ldcs(sp + x);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int x = x0 + j * kWarp + lane;
            if (x < total)
                reinterpret_cast<UT *>(dst + (int64_t)(x >> upr_sh) * tile_bytes)[x & mask] =
                    plus_zero<ES, UT>(w[j]);
        }
    }
}

// The same stream when the source starts `off` bytes (0 < off < 16, a
// multiple of ES) past a 16-byte boundary: each lane loads the aligned unit
// holding its first bytes, takes the next one from the lane after it (lane 31
// loads it), and funnel-shifts the pair into place.  The aligned units read
// stay inside the 16-byte blocks that hold the row's own bytes.
template <int ES, int WS>
__device__ __forceinline__ uint4 realign(uint4 a, uint4 b, int bs) {
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    return make_uint4(__funnelshift_r(w[WS], w[WS + 1], bs), __funnelshift_r(w[WS + 1], w[WS + 2], bs),
                      __funnelshift_r(w[WS + 2], w[WS + 3], bs), __funnelshift_r(w[WS + 3], w[WS + 4], bs));
}

template <int ES, int WS>
__device__ __forceinline__ void copy_row_shifted(const uint4 *sp, int bs, char *dst, int64_t tile_bytes,
                                                 int total, int upr_sh, int lane) {
    // destination units x < total read aligned source units x and x + 1
    // (unit `total` holds the row's last bytes)
    const int mask = (1 << upr_sh) - 1;
    for (int x0 = 0; x0 < total; x0 += 4 * kWarp) {
        uint4 a[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int x = x0 + j * kWarp + lane;
            a[j] = x <= total ? __ldcs(sp + x) : make_uint4(0, 0, 0, 0);
        }
        const uint4 tail = lane == kWarp - 1 && x0 + 4 * kWarp <= total ? __ldcs(sp + x0 + 4 * kWarp)
                                                                        : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            // unit x + 1: the next lane's, for lane 31 lane 0's of the next j
            const uint4 &up = j < 3 ? a[j + 1] : a[j];
            uint4 nx, wrap;
            nx.x = __shfl_down_sync(0xffffffffu, a[j].x, 1);
            nx.y = __shfl_down_sync(0xffffffffu, a[j].y, 1);
            nx.z = __shfl_down_sync(0xffffffffu, a[j].z, 1);
            nx.w = __shfl_down_sync(0xffffffffu, a[j].w, 1);
            wrap.x = __shfl_sync(0xffffffffu, up.x, 0);
            wrap.y = __shfl_sync(0xffffffffu, up.y, 0);
            wrap.z = __shfl_sync(0xffffffffu, up.z, 0);
            wrap.w = __shfl_sync(0xffffffffu, up.w, 0);
            if (lane == kWarp - 1) nx = j < 3 ? wrap : tail;
            const int x = x0 + j * kWarp + lane;
            if (x < total)
                reinterpret_cast<uint4 *>(dst + (int64_t)(x >> upr_sh) * tile_bytes)[x & mask] =
                    plus_zero<ES, uint4>(realign<ES, WS>(a[j], nx, bs));
        }
    }
}

template <int ES>
__device__ __forceinline__ void copy_row_any(const char *src, char *dst, int64_t tile_bytes, int total,
                                             int upr_sh, int lane) {
    const int off = (int)(reinterpret_cast<uintptr_t>(src) & 15);
    if (off == 0) {
        copy_row_units<ES, uint4>(src, dst, tile_bytes, total, upr_sh, lane);
        return;
    }
    const uint4 *sp = reinterpret_cast<const uint4 *>(src - off);
    const int bs = (off & 3) * 8;
    switch (off >> 2) {
        case 0: copy_row_shifted<ES, 0>(sp, bs, dst, tile_bytes, total, upr_sh, lane); break;
        case 1: copy_row_shifted<ES, 1>(sp, bs, dst, tile_bytes, total, upr_sh, lane); break;
        case 2: copy_row_shifted<ES, 2>(sp, bs, dst, tile_bytes, total, upr_sh, lane); break;
        default: copy_row_shifted<ES, 3>(sp, bs, dst, tile_bytes, total, upr_sh, lane); break;
    }
}

template <int ES>
__global__ void __launch_bounds__(kRowThreads, 3)
fill_whole_rows(Src s, int64_t mb, int64_t nnzb, const int32_t *__restrict__ browptr,
                const int32_t *__restrict__ bcolind, char *__restrict__ bval, Carry carry) {
    const bool handed = carry.bits && *carry.stamp == carry.key;
    if (!handed) return;
    const int lane = threadIdx.x % kWarp;
    const int b1 = s.b1, b2 = s.b2, row_bytes = b2 * ES;
    const int64_t tile_bytes = (int64_t)b1 * row_bytes;
    const int64_t nrows = mb * b1;
    const int64_t warps = (int64_t)gridDim.x * (kRowThreads / kWarp);
    for (int64_t i = (int64_t)blockIdx.x * (kRowThreads / kWarp) + threadIdx.x / kWarp; i < nrows;
         i += warps) {
        const int64_t I = i / b1;
        const int r = (int)(i - I * b1);
        int64_t q0;
        int nblk;
        if (!asc_row(s, carry, handed, browptr, nnzb, I, q0, nblk)) continue;
        char *row0 = bval + q0 * tile_bytes + (int64_t)r * row_bytes;
        bool done = false;
        if (i >= s.m) {   // rows past the matrix: padding
            for (int k = 0; k < nblk; ++k) zero_row(row0 + (int64_t)k * tile_bytes, row_bytes, lane);
            done = true;
        } else if (nblk == 0) {
            done = true;
        } else {
            const int64_t lo = s.rowptr[i] - s.base, hi = s.rowptr[i + 1] - s.base;
            // ascending, nblk runs (block columns) each starting nonzero -- so
            // each is one of the block row's nblk blocks -- and nblk * b2
            // entries: at most b2 a block, so exactly b2, every run full
            const bool whole = carry.row_runs[i] == nblk && hi - lo == (int64_t)nblk * b2;
            const char *src = reinterpret_cast<const char *>(s.val) + lo * ES;
            const uintptr_t dal = reinterpret_cast<uintptr_t>(row0) | (uintptr_t)row_bytes |
                                  (uintptr_t)tile_bytes;
            const uintptr_t al = reinterpret_cast<uintptr_t>(src) | dal;
            const int ub = (al & 15) == 0 ? 16 : (al & 7) == 0 ? 8 : (al & 3) == 0 ? 4 : 0;
            const int upr = ub ? row_bytes / ub : 0;
            const int upr16 = row_bytes / 16;
            if (whole && (dal & 15) == 0 && (upr16 & (upr16 - 1)) == 0) {
                // 16-byte units on the tile side, any source offset
                copy_row_any<ES>(src, row0, tile_bytes, nblk * upr16, __ffs(upr16) - 1, lane);
                done = true;
            } else if (whole && ub && (upr & (upr - 1)) == 0) {
                const int sh = __ffs(upr) - 1, total = nblk * upr;
                if (ub == 16) copy_row_units<ES, uint4>(src, row0, tile_bytes, total, sh, lane);
                else if (ub == 8) copy_row_units<ES, uint2>(src, row0, tile_bytes, total, sh, lane);
                else if constexpr (ES <= 4)
                    copy_row_units<ES, uint32_t>(src, row0, tile_bytes, total, sh, lane);
                done = true;
            }
        }
        if (lane == 0) carry.row_done[i] = done;
    }
}

// The rows fill_whole_rows left, run by run: a warp takes 32 rows, finds the
// ones to do with one flag load a lane, and does them one after another.
template <int ES>
__global__ void __launch_bounds__(kRowThreads)
fill_other_rows(Src s, int64_t mb, int64_t nnzb, const int32_t *__restrict__ browptr,
                const int32_t *__restrict__ bcolind, char *__restrict__ bval, Carry carry) {
    const bool handed = carry.bits && *carry.stamp == carry.key;
    if (!handed) return;
    const int lane = threadIdx.x % kWarp;
    const int b1 = s.b1, row_bytes = s.b2 * ES;
    const int64_t tile_bytes = (int64_t)b1 * row_bytes;
    const int64_t nrows = mb * b1;
    const int64_t warps = (int64_t)gridDim.x * (kRowThreads / kWarp);
    for (int64_t i0 = ((int64_t)blockIdx.x * (kRowThreads / kWarp) + threadIdx.x / kWarp) * kWarp;
         i0 < nrows; i0 += warps * kWarp) {
        const int64_t i = i0 + lane;
        bool todo = false;
        if (i < nrows) {
            const int64_t I = i / b1;
            int64_t q0;
            int nblk;
            todo = asc_row(s, carry, handed, browptr, nnzb, I, q0, nblk) && !carry.row_done[i];
        }
        unsigned pend = __ballot_sync(0xffffffffu, todo);
        while (pend) {
            const int l = __ffs(pend) - 1;
            pend &= pend - 1;
            const int64_t ir = i0 + l, I = ir / b1;
            int64_t q0;
            int nblk;
            asc_row(s, carry, handed, browptr, nnzb, I, q0, nblk);
            fill_row_runs<ES>(s, ir, bval + q0 * tile_bytes + (ir - I * b1) * row_bytes, nblk,
                              bcolind + q0, tile_bytes, lane);
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

// ------------------------------------------------- sorted compression
// COO-style (outer, inner) coordinate pairs compressed along the outer
// coordinate, the composer's path when the target's level order differs from
// the source's (CSC targets, CSC -> CSR): the nonzero entries are bucketed by
// outer coordinate (coo_bucket with one bucket per outer index), each bucket
// is sorted by (inner coordinate, storage index) with the sorts of sort.cuh --
// the order of the composer's stable lexsort (src/convert.jl:334-345,
// 419-424) -- and the first entry of every run of equal inner coordinates is
// kept, as the composer keeps the first value of a run (src/convert.jl:
// 222-238).

// Writes the first entry of every run of equal columns of each sorted bucket
// to the CSR (one warp per row): its column (origin kept) and value.
template <int ES>
__global__ void __launch_bounds__(seg::kSortThreads)
emit_csr_rows(int64_t m, const int32_t *__restrict__ offs, const int32_t *__restrict__ ent,
              const int32_t *__restrict__ cols, const void *__restrict__ val, int base,
              const int32_t *__restrict__ rowptr, int64_t nnz_out, int32_t *__restrict__ colind,
              void *__restrict__ out_val) {
    const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
    const int64_t nwarps = (int64_t)gridDim.x * (seg::kSortThreads / kWarp);
    for (int64_t r = (int64_t)blockIdx.x * (seg::kSortThreads / kWarp) + warp; r < m; r += nwarps) {
        const int lo = ldg(offs + r), hi = ldg(offs + r + 1);
        const int64_t out = (int64_t)ldg(rowptr + r) - base, end = (int64_t)ldg(rowptr + r + 1) - base;
        int64_t run = 0;
        int32_t prev = 0;
        for (int i0 = lo; i0 < hi; i0 += kWarp) {
            const int i = i0 + lane;
            const bool in = i < hi;
            const int32_t e = in ? ent[i] : 0;
            const int32_t c = in ? ldg(cols + e) : 0;
            int32_t up = __shfl_up_sync(0xffffffffu, c, 1);
            if (lane == 0) up = prev;
            const bool first = in && (i == lo || c != up);
            const unsigned bal = __ballot_sync(0xffffffffu, first);
            if (first) {
                const int64_t q = out + run + __popc(bal & ((1u << lane) - 1u));
                if (q >= 0 && q < end && q < nnz_out) {
                    colind[q] = c;
                    copy_val<ES>(out_val, q, val, e);
                } else {
                    dev_error(DEV_ERR_OVERFLOW);
                }
            }
            run += __popc(bal);
            prev = __shfl_sync(0xffffffffu, c, kWarp - 1);
        }
    }
}

// ------------------------------------------------------------- COO -> CSR
// JLUST's COO format declares its levels ordered, so convert_format hands a
// COO source to the composer in storage order without sorting
// (src/convert.jl:346-355): rows must not decrease (the composer's dense row
// level asserts it, :246), entries keep their storage order within a row,
// explicit zeros are dropped (:316) and an entry whose coordinates equal
// those of the nonzero entry before it is merged into it, keeping the first
// value (the unique column level's run, :231-238).  So the CSR is a stable
// compaction of the COO: keep[p] marks the entries that stay, their ranks
// give their slots, and the first kept entry of row r writes rowptr for the
// rows since the previous kept entry's row.

// The last nonzero entry before p, or -1.  Every zero belongs to the run
// before exactly one nonzero entry, so these walks add up to at most nnz.
template <int ES>
__device__ __forceinline__ int64_t prev_nonzero(const void *__restrict__ val, int64_t p) {
    int64_t q = p - 1;
    while (q >= 0 && is_zero<ES>(val, q)) --q;
    return q;
}

// ---------------------------------------- COO -> CSR by tiles of entries
// The compaction works on tiles of kScanTile entries: the keep pass writes
// one byte per entry, each tile's kept count and (count phase) each row's
// kept count; the library scan turns the tile counts into tile offsets and
// the row counts into the row pointer; the emit pass rebuilds each entry's
// slot from its tile's keep bytes with a block scan.  No per-entry slot
// array: each pass reads the COO arrays it needs once.

// keep[p] (one byte): nonzero, inside the extents and (merge) not on the
// coordinates of the nonzero entry before it; per tile the kept count; with
// row_counts (zeroed), each row's kept count: rows ascend, so a warp's 32
// consecutive entries fall in runs of equal rows; each run's first lane adds
// the run's kept count with one atomic (runs from a shuffle and two ballots:
// finding them with __match_any_sync took the kernel from 395 to 501 us on
// the cfg2 Laplacian).  The entry before, almost always the nonzero
// predecessor, is the lane before's entry and comes by shuffle (lane 0 loads
// it: 395 -> about 385 us); only past an explicit zero does a thread walk
// back.
template <int ES>
__global__ void __launch_bounds__(kThreads)
coo_keep_tiles(int64_t nnz, const int32_t *__restrict__ rows, const int32_t *__restrict__ cols,
               const void *__restrict__ val, int base, int64_t m, int64_t n, bool merge,
               uint8_t *__restrict__ keep, int32_t *__restrict__ tcount,
               int32_t *__restrict__ row_counts) {
    __shared__ int64_t s_warp[kThreads / kWarp];
    const int64_t t0 = (int64_t)blockIdx.x * kScanTile;
    const int lane = threadIdx.x % kWarp;
    int64_t cnt = 0;
#pragma unroll 4
    for (int i = 0; i < kScanItems; ++i) {
        const int64_t p = t0 + (int64_t)i * kThreads + threadIdx.x;
        if (p >= nnz) break;
        const bool has_prev = p > 0;
        const unsigned act = __activemask();
        const int32_t r = ldg(rows + p), c = ldg(cols + p);
        const bool zero = is_zero<ES>(val, p);
        // entry p - 1 is the lane before's entry (lane 0 loads it)
        int32_t r1 = __shfl_up_sync(act, r, 1), c1 = __shfl_up_sync(act, c, 1);
        bool zero1 = __shfl_up_sync(act, (int)zero, 1) != 0;
        if (lane == 0 || !((act >> (lane - 1)) & 1u)) {
            r1 = has_prev ? ldg(rows + p - 1) : 0;
            c1 = has_prev ? ldg(cols + p - 1) : 0;
            zero1 = !has_prev || is_zero<ES>(val, p - 1);
        }
        int k = 0;
        if (!zero) {
            if ((int64_t)r - base < 0 || (int64_t)r - base >= m || (int64_t)c - base < 0 ||
                (int64_t)c - base >= n) {
                dev_error(DEV_ERR_BOUNDS);
            } else {
                k = 1;
                if (merge) {
                    int64_t q = -1;
                    int32_t rq = 0, cq = 0;
                    if (!zero1) {
                        q = p - 1;
                        rq = r1;
                        cq = c1;
                    } else if (has_prev) {
                        q = prev_nonzero<ES>(val, p - 1);
                        if (q >= 0) {
                            rq = ldg(rows + q);
                            cq = ldg(cols + q);
                        }
                    }
                    if (q >= 0) {
                        if (rq > r) dev_error(DEV_ERR_ORDER);
                        k = (rq != r || cq != c);
                    }
                }
            }
        }
        keep[p] = (uint8_t)k;
        cnt += k;
        if (row_counts) {
            // a run starts where the row differs from the lane before's (or
            // that lane is not here: a split warp only adds more atomics); it
            // ends before the next run's first lane.  A run with a kept entry
            // is on that entry's row, checked in bounds above.
            const unsigned act = __activemask();
            const int32_t rb = __shfl_up_sync(act, r, 1);
            const bool head = lane == 0 || !((act >> (lane - 1)) & 1u) || rb != r;
            const unsigned heads = __ballot_sync(act, head), kept = __ballot_sync(act, k);
            if (head) {
                const unsigned above = heads & (0xfffffffeu << lane);
                const unsigned upto = above ? (above & (0u - above)) - 1u : 0xffffffffu;
                const int kc = __popc(kept & upto & (0xffffffffu << lane));
                if (kc) atomicAdd(&row_counts[r - base], kc);
            }
        }
    }
    int64_t tot;
    block_exclusive_scan<kThreads>(cnt, s_warp, tot);
    if (threadIdx.x == 0) tcount[blockIdx.x] = (int32_t)tot;
}

// Each entry's slot (its kept rank in storage order + the tile's first
// slot), or -1 when it is not kept, into s_slot[scan_pad(k)] for entry
// t0 + k: thread j ranks entries 16j .. 16j+15, whose keep bytes (0 or 1) it
// loads as one 16-byte vector when the tile is whole and aligned (padded
// indices: no bank conflicts).
__device__ __forceinline__ void coo_tile_slots(int64_t nnz, int64_t t0, const uint8_t *__restrict__ keep,
                                               int64_t first, int32_t *s_slot, int64_t *s_warp) {
    const int64_t e0 = t0 + (int64_t)threadIdx.x * kScanItems;
    uint32_t kb[kScanItems / 4];
    if (t0 + kScanTile <= nnz && (reinterpret_cast<uintptr_t>(keep + t0) & 15) == 0) {
        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(keep + e0));
        kb[0] = q.x; kb[1] = q.y; kb[2] = q.z; kb[3] = q.w;
    } else {
#pragma unroll
        for (int w = 0; w < kScanItems / 4; ++w) {
            kb[w] = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t e = e0 + 4 * w + j;
                if (e < nnz) kb[w] |= (uint32_t)keep[e] << (8 * j);
            }
        }
    }
    int64_t v = 0;
#pragma unroll
    for (int w = 0; w < kScanItems / 4; ++w) v += __popc(kb[w]);
    int64_t tot;
    int64_t run = block_exclusive_scan<kThreads>(v, s_warp, tot) + first;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const int kp = (kb[j / 4] >> (8 * (j % 4))) & 1;
        s_slot[scan_pad(threadIdx.x * kScanItems + j)] = kp ? (int32_t)run : -1;
        run += kp;
    }
    __syncthreads();
}

// colind / values (and rows_out) of the kept entries at their slots.  (A
// version that loaded the thread's columns and values before the block scan
// held 74 registers, three CTAs an SM, and took 598 us where this took 455
// on the cfg2 Laplacian; it now takes 355.)
template <int ES>
__global__ void __launch_bounds__(kThreads)
coo_emit_tiles(int64_t nnz, const int32_t *__restrict__ rows, const int32_t *__restrict__ cols,
               const void *__restrict__ val, const uint8_t *__restrict__ keep,
               const int32_t *__restrict__ tfirst, int64_t nnz_out, int32_t *__restrict__ rows_out,
               int32_t *__restrict__ colind, void *__restrict__ out_val) {
    __shared__ int64_t s_warp[kThreads / kWarp];
    __shared__ int32_t s_slot[kScanTile + kScanTile / 32];
    const int64_t t0 = (int64_t)blockIdx.x * kScanTile;
    coo_tile_slots(nnz, t0, keep, tfirst[blockIdx.x], s_slot, s_warp);
#pragma unroll 4
    for (int i = 0; i < kScanItems; ++i) {
        const int k = i * kThreads + threadIdx.x;
        const int64_t p = t0 + k;
        const int64_t q = s_slot[scan_pad(k)];
        if (p >= nnz || q < 0) continue;
        if (q >= nnz_out) {
            dev_error(DEV_ERR_OVERFLOW);
            continue;
        }
        if (rows_out) rows_out[q] = ldg(rows + p);
        colind[q] = ldg(cols + p);
        copy_val<ES>(out_val, q, val, p);
    }
}


// coordinates[k] = i + base for k in [ptr[i], ptr[i+1]) - base: the outer
// coordinate of every entry of a compressed level.  Each thread takes 16
// consecutive entries, finds the row of the first by binary search over ptr
// and walks on (balanced whatever the row lengths); it stores them as four
// 16-byte vectors when it can.  The same threads check every row's range.
constexpr int kExpandItems = 16;

__global__ void __launch_bounds__(kThreads)
expand_positions(int64_t n_outer, int64_t nnz, const int32_t *__restrict__ ptr, int base,
                 int32_t *__restrict__ coords) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (int64_t i = tid; i < n_outer; i += stride) {
        const int64_t lo = (int64_t)ldg(ptr + i) - base, hi = (int64_t)ldg(ptr + i + 1) - base;
        if (lo < 0 || hi > nnz || lo > hi) dev_error(DEV_ERR_BOUNDS);
    }
    const int64_t nchunks = (nnz + kExpandItems - 1) / kExpandItems;
    const bool vec = (reinterpret_cast<uintptr_t>(coords) & 15) == 0;
    for (int64_t c = tid; c < nchunks; c += stride) {
        const int64_t k0 = c * kExpandItems;
        const int64_t k1 = k0 + kExpandItems < nnz ? k0 + kExpandItems : nnz;
        // the last row r with ptr[r] - base <= k0
        int64_t a = 0, b = n_outer - 1;
        while (a < b) {
            const int64_t mid = (a + b + 1) >> 1;
            if ((int64_t)ldg(ptr + mid) - base <= k0) a = mid;
            else b = mid - 1;
        }
        int64_t r = a;
        int32_t v[kExpandItems];
#pragma unroll
        for (int u = 0; u < kExpandItems; ++u) {
            const int64_t k = k0 + u;
            while (r + 1 < n_outer && (int64_t)ldg(ptr + r + 1) - base <= k) ++r;
            v[u] = (int32_t)(r + base);
        }
        if (vec && k1 - k0 == kExpandItems) {
            int4 *dst = reinterpret_cast<int4 *>(coords + k0);
#pragma unroll
            for (int q = 0; q < kExpandItems / 4; ++q)
                dst[q] = make_int4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else {
            for (int64_t k = k0; k < k1; ++k) coords[k] = v[k - k0];
        }
    }
}

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

// bitmaps (mb x words) then one ascending-rows flag per block row
static size_t carry_bits_bytes(int64_t m, int64_t n, int b1, int b2) {
    const int64_t mb = ceil_div(m, b1), nb = ceil_div(n, b2);
    return align256((size_t)mb * (size_t)ceil_div(nb, 32) * 4);
}

static size_t carry_bytes(int64_t m, int64_t n, int b1, int b2) {
    const int64_t mb = ceil_div(m, b1), nb = ceil_div(n, b2);
    if (nb > conv::kWinBits || mb <= 0) return 0;
    const size_t bytes = carry_bits_bytes(m, n, b1, b2) + align256((size_t)mb) +
                         align256((size_t)mb * (size_t)b1) + align256((size_t)mb * (size_t)b1 * 4);
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
    conv::Carry c{nullptr, nullptr, nullptr, nullptr, nullptr, 0};
    const size_t cb = carry_bytes(m, n, b1, b2);
    const size_t scan = csr_scan_ws(m, b1);
    if (!cb || !ws || wsb < scan + 256 + cb) return c;
    char *p = reinterpret_cast<char *>(ws);
    c.stamp = reinterpret_cast<uint64_t *>(p + scan);
    c.bits = reinterpret_cast<uint32_t *>(p + scan + 256);
    c.asc = reinterpret_cast<uint8_t *>(p + scan + 256 + carry_bits_bytes(m, n, b1, b2));
    c.row_done = c.asc + align256((size_t)ceil_div(m, b1));
    c.row_runs = reinterpret_cast<int32_t *>(c.row_done + align256((size_t)ceil_div(m, b1) * (size_t)b1));
    c.key = carry_key(m, n, nnz, b1, b2, base, dtype, rowptr, colind, val);
    return c;
}

extern "C" JLB_API size_t jlb_csr_to_bsr_workspace_size(int64_t m, int64_t n, int64_t nnz, int b1,
                                                        int b2) {
    return b1 > 0 && b2 > 0 ? csr_ws(m, n, b1, b2) : 0;
}

static conv::Src csr_src(int dtype, int idx_base, int64_t m, int64_t n, int64_t nnz,
                         const int32_t *rowptr, const int32_t *colind, const void *val, int b1,
                         int b2) {
    conv::Src s{};
    s.rowptr = rowptr; s.rows = nullptr; s.cols = colind; s.val = val;
    s.boffs = nullptr; s.bent = nullptr; s.m = m; s.n = n;
    s.b1 = b1; s.b2 = b2; s.base = idx_base; s.es = (int)dtype_size(dtype);
    s.sh1 = conv::log2_exact(b1); s.sh2 = conv::log2_exact(b2);
    s.nnz = nnz; s.vec = aligned16(colind);
    return s;
}

static int finish_count(cudaStream_t st, int64_t mb, int idx_base, int32_t *browptr,
                        int64_t *nnzb, void *ws, size_t wsb, int *dev_bits,
                        const char *overflow_msg = "block count overflows Int32 positions") {
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
    if (bits & DEV_ERR_OVERFLOW) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "%s", overflow_msg);
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
        const conv::Src src = csr_src(dtype, idx_base, m, n, nnz, rowptr, colind, val, b1, b2);
        const conv::Carry cy = csr_carry(workspace, workspace_bytes, m, n, nnz, b1, b2, idx_base,
                                         dtype, rowptr, colind, val);
        const unsigned grid = conv::grid_rows(mb);
        const int es = (int)dtype_size(dtype);
#define JLB_COUNT_CSR(E)                                                                         \
    if (src.sh2 >= 0) {                                                                          \
        JLB_CUDA(cudaFuncSetAttribute(conv::count_csr<E, true>,                                  \
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,              \
                                      (int)conv::kCountSmem));                                   \
        conv::count_csr<E, true><<<grid, conv::kCsrThreads, conv::kCountSmem, st>>>(             \
            src, mb, nb, browptr + 1, cy);                                                       \
    } else {                                                                                     \
        JLB_CUDA(cudaFuncSetAttribute(conv::count_csr<E, false>,                                 \
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,              \
                                      (int)conv::kCountSmem));                                   \
        conv::count_csr<E, false><<<grid, conv::kCsrThreads, conv::kCountSmem, st>>>(            \
            src, mb, nb, browptr + 1, cy);                                                       \
    }
        if (es == 8) { JLB_COUNT_CSR(8); }
        else if (es == 4) { JLB_COUNT_CSR(4); }
        else { JLB_COUNT_CSR(2); }
#undef JLB_COUNT_CSR
        JLB_LAUNCH_CHECK("count_csr");
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
    const conv::Src src = csr_src(dtype, idx_base, m, n, nnz, rowptr, colind, val, b1, b2);
    const conv::Carry cy = csr_carry(workspace, workspace_bytes, m, n, nnz, b1, b2, idx_base, dtype,
                                     rowptr, colind, val);
    // block rows the count pass found ascending (hand-over present) take the
    // tile-row kernel; the entry-by-entry kernel does the others
    if (cy.bits) {
        const unsigned grid = conv::grid_rows(mb);
        const int64_t rows = mb * (int64_t)b1;
        const unsigned rgrid = (unsigned)std::min<int64_t>(ceil_div(rows, conv::kRowThreads / kWarp),
                                                           148 * 16);
        const unsigned ogrid = (unsigned)std::min<int64_t>(
            ceil_div(rows, (int64_t)conv::kRowThreads / kWarp * kWarp), 148 * 4);
        char *bv = static_cast<char *>(bval);
#define JLB_ASC_FILL(E)                                                                           \
    conv::fill_asc_columns<E><<<grid, conv::kAscThreads, 0, st>>>(src, mb, nb, nnzb, browptr,       \
                                                                  bcolind, cy);                    \
    conv::fill_whole_rows<E><<<rgrid, conv::kRowThreads, 0, st>>>(src, mb, nnzb, browptr, bcolind,  \
                                                                  bv, cy);                          \
    conv::fill_other_rows<E><<<ogrid, conv::kRowThreads, 0, st>>>(src, mb, nnzb, browptr, bcolind,  \
                                                                  bv, cy)
        const int es = (int)dtype_size(dtype);
        if (es == 8) { JLB_ASC_FILL(8); }
        else if (es == 4) { JLB_ASC_FILL(4); }
        else { JLB_ASC_FILL(2); }
#undef JLB_ASC_FILL
        JLB_LAUNCH_CHECK("fill_ascending");
    }
    JLB_CONV_LAUNCH(fill_blocks, dtype_size(dtype), conv::grid_rows(mb), st, src, mb, nb, nnzb,
                    browptr, bcolind, bval, nullptr, cy);
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
                    nnzb, browptr, bcolind, bval, winner, conv::Carry{nullptr, nullptr, nullptr, nullptr, nullptr, 0});
    JLB_LAUNCH_CHECK("fill_blocks");
    return ok();
}

// ------------------------------------------------- allocation-free scan
// A variant of jlb_exclusive_scan_i32 for callers that cannot allocate device
// memory: its scratch (one int64 partial sum per tile of kScanTile = 4096
// counts) lives in this
// file-scope device array instead of a caller workspace.  The array exists on
// every GPU that loads the library, for the life of the process.
namespace jlb {
namespace conv {

constexpr int64_t kNoAllocTiles = 8192;                     // 64 KB of scratch
constexpr int64_t kNoAllocMaxN = kNoAllocTiles * kScanTile; // 33,554,432 counts
static_assert(kNoAllocMaxN == JLB_SCAN_NOALLOC_MAX_N, "header limit out of date");

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

// ------------------------------------------------- sorted compression
// Workspace: [buckets (as for COO -> BSR with b1 = 1) | stamp | long-bucket
// count | long-bucket list].  The count phase leaves the sorted buckets there
// for the fill phase.
namespace {
struct SortedWs {
    uint64_t *stamp;
    int32_t *n_long, *long_rows;
    int64_t long_cap;
    size_t bytes;
};

SortedWs sorted_ws(void *ws, int64_t n_outer, int64_t nnz) {
    SortedWs w{};
    Carve k{reinterpret_cast<char *>(ws)};
    k.off = coo_ws(n_outer, nnz, 1, 1, 0, nullptr);
    w.stamp = k.take<uint64_t>(1);
    w.n_long = k.take<int32_t>(1);
    w.long_cap = nnz / (seg::kWarpKeys + 1) + 1;
    w.long_rows = k.take<int32_t>((size_t)w.long_cap);
    w.bytes = k.off + 256;
    return w;
}

uint64_t sorted_key(int64_t n_outer, int64_t n_inner, int64_t nnz, int base, int dtype,
                    const void *outer, const void *inner, const void *val) {
    // b1 = b2 = -1 marks a sorted-compression workspace
    return carry_key(n_outer, n_inner, nnz, -1, -1, base, dtype, outer, inner, val);
}
}  // namespace

extern "C" JLB_API size_t jlb_sorted_compress_workspace_size(int64_t n_outer, int64_t nnz) {
    if (n_outer < 0 || nnz < 0) return 0;
    return sorted_ws(nullptr, n_outer, nnz).bytes;
}

extern "C" JLB_API int jlb_sorted_compress_count(void *stream, int dtype, int idx_base,
                                                 int64_t n_outer, int64_t n_inner, int64_t nnz,
                                                 const int32_t *outer, const int32_t *inner,
                                                 const void *val, int32_t *ptr, int64_t *nnz_out,
                                                 void *workspace, size_t workspace_bytes) {
    int r = conv_args(dtype, idx_base, n_outer, n_inner, nnz, 1, 1);
    if (r) return r;
    if (n_outer > INT32_MAX - 1) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "outer extent exceeds Int32");
    if (!ptr || !nnz_out || (nnz > 0 && (!outer || !inner || !val)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    const SortedWs w = sorted_ws(workspace, n_outer, nnz);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(JLB_ERR_WORKSPACE, "workspace too small");
    cudaStream_t st = as_stream(stream);
    int32_t *boffs, *bent;
    r = coo_bucket(st, dtype, idx_base, n_outer, n_inner, nnz, outer, inner, val, 1, workspace,
                   &boffs, &bent);
    if (r) return r;
    JLB_CUDA(cudaMemsetAsync(w.n_long, 0, sizeof(int32_t), st));
    if (n_outer > 0) {
        const int64_t g = ceil_div(n_outer, seg::kSortThreads / kWarp);
        seg::sort_short_rows<<<(unsigned)(g < 148 * 16 ? g : 148 * 16), seg::kSortThreads, 0, st>>>(
            n_outer, boffs, bent, inner, idx_base, ptr + 1, w.long_rows, w.n_long, w.long_cap);
        JLB_LAUNCH_CHECK("sort_short_rows");
        const int smem = seg::kCtaKeys * (int)sizeof(uint64_t);
        JLB_CUDA(cudaFuncSetAttribute(seg::sort_long_rows,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        seg::sort_long_rows<<<148, seg::kLongThreads, smem, st>>>(
            boffs, bent, inner, idx_base, ptr + 1, w.long_rows, w.n_long, w.long_cap);
        JLB_LAUNCH_CHECK("sort_long_rows");
    }
    const uint64_t key = sorted_key(n_outer, n_inner, nnz, idx_base, dtype, outer, inner, val);
    JLB_CUDA(cudaMemcpyAsync(w.stamp, &key, sizeof(key), cudaMemcpyHostToDevice, st));
    // The bucket scan is done with the scan workspace: reuse it for ptr.
    Carve k{reinterpret_cast<char *>(workspace)};
    k.take<int32_t>((size_t)n_outer + 1);
    k.take<int32_t>((size_t)(n_outer > 0 ? n_outer : 1));
    k.take<int32_t>((size_t)(nnz > 0 ? nnz : 1));
    const size_t sws = conv::scan_ws(n_outer > 0 ? n_outer : 1);
    char *scan_ws = k.take<char>(sws);
    return finish_count(st, n_outer, idx_base, ptr, nnz_out, scan_ws, sws, nullptr,
                        "an outer index holds more than 16,777,216 entries, the longest this "
                        "sort takes");
}

extern "C" JLB_API int jlb_sorted_compress_fill(void *stream, int dtype, int idx_base,
                                                int64_t n_outer, int64_t n_inner, int64_t nnz,
                                                const int32_t *outer, const int32_t *inner,
                                                const void *val, const int32_t *ptr,
                                                int64_t nnz_out, int32_t *inner_out,
                                                void *val_out, void *workspace,
                                                size_t workspace_bytes) {
    int r = conv_args(dtype, idx_base, n_outer, n_inner, nnz, 1, 1);
    if (r) return r;
    if (!ptr || (nnz > 0 && (!outer || !inner || !val)) || (nnz_out > 0 && (!inner_out || !val_out)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    if (nnz_out < 0 || nnz_out > nnz) return fail(JLB_ERR_INVALID_ARGUMENT, "bad nnz_out");
    const SortedWs w = sorted_ws(workspace, n_outer, nnz);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(JLB_ERR_WORKSPACE, "workspace too small");
    cudaStream_t st = as_stream(stream);
    uint64_t stamp = 0;
    JLB_CUDA(cudaMemcpyAsync(&stamp, w.stamp, sizeof(stamp), cudaMemcpyDeviceToHost, st));
    JLB_CUDA(cudaStreamSynchronize(st));
    if (stamp != sorted_key(n_outer, n_inner, nnz, idx_base, dtype, outer, inner, val))
        return fail(JLB_ERR_WORKSPACE,
                    "the fill phase needs the workspace its count phase filled, unchanged");
    if (n_outer == 0) return ok();
    Carve k{reinterpret_cast<char *>(workspace)};
    const int32_t *boffs = k.take<int32_t>((size_t)n_outer + 1);
    k.take<int32_t>((size_t)n_outer);
    const int32_t *bent = k.take<int32_t>((size_t)(nnz > 0 ? nnz : 1));
    const int64_t g64 = ceil_div(n_outer, seg::kSortThreads / kWarp);
    const unsigned g = (unsigned)(g64 < 148 * 16 ? g64 : 148 * 16);
    const size_t es = dtype_size(dtype);
    if (es == 8)
        conv::emit_csr_rows<8><<<g, seg::kSortThreads, 0, st>>>(n_outer, boffs, bent, inner, val,
                                                                 idx_base, ptr, nnz_out, inner_out, val_out);
    else if (es == 4)
        conv::emit_csr_rows<4><<<g, seg::kSortThreads, 0, st>>>(n_outer, boffs, bent, inner, val,
                                                                 idx_base, ptr, nnz_out, inner_out, val_out);
    else
        conv::emit_csr_rows<2><<<g, seg::kSortThreads, 0, st>>>(n_outer, boffs, bent, inner, val,
                                                                 idx_base, ptr, nnz_out, inner_out, val_out);
    JLB_LAUNCH_CHECK("emit_csr_rows");
    return ok();
}

extern "C" JLB_API int jlb_positions_to_coordinates(void *stream, int idx_base, int64_t n_outer,
                                                    int64_t nnz, const int32_t *ptr,
                                                    int32_t *coords) {
    if (idx_base != 0 && idx_base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (n_outer < 0 || nnz < 0) return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "negative extent");
    if (n_outer > INT32_MAX - 1) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "outer extent exceeds Int32");
    if (!ptr || (nnz > 0 && !coords)) return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    if (n_outer == 0) return ok();
    cudaStream_t st = as_stream(stream);
    const int64_t work = n_outer > ceil_div(nnz, conv::kExpandItems) ? n_outer
                                                                       : ceil_div(nnz, conv::kExpandItems);
    const int64_t g = ceil_div(work, conv::kThreads);
    conv::expand_positions<<<(unsigned)(g < 148 * 32 ? g : 148 * 32), conv::kThreads, 0, st>>>(
        n_outer, nnz, ptr, idx_base, coords);
    JLB_LAUNCH_CHECK("expand_positions");
    return ok();
}

// ------------------------------------------------------------- COO -> CSR
// Workspace: [stamp | keep bytes (nnz) | tile counts | tile first slots
// (+ the total) | row counts (m) | scan scratch].  The count phase stamps the
// keep bytes and tile slots it leaves; a fill phase given the same workspace
// for the same inputs uses them instead of recomputing.
namespace {
struct CooCsrWs {
    uint64_t *stamp;
    uint8_t *keep;
    int32_t *tcount, *tfirst, *rowcnt;
    char *scan;
    int64_t ntiles;
    size_t scan_bytes, bytes;
};

CooCsrWs coo_csr_ws(void *ws, int64_t nnz, int64_t m) {
    CooCsrWs w{};
    Carve k{reinterpret_cast<char *>(ws)};
    w.ntiles = ceil_div(nnz > 0 ? nnz : 1, conv::kScanTile);
    w.stamp = k.take<uint64_t>(1);
    w.keep = k.take<uint8_t>((size_t)(nnz > 0 ? nnz : 1));
    w.tcount = k.take<int32_t>((size_t)w.ntiles);
    w.tfirst = k.take<int32_t>((size_t)w.ntiles + 1);
    w.rowcnt = k.take<int32_t>((size_t)(m > 0 ? m : 1));
    const int64_t big = w.ntiles > m ? w.ntiles : m;
    w.scan_bytes = conv::scan_ws(big > 0 ? big : 1);
    w.scan = k.take<char>(w.scan_bytes);
    w.bytes = k.off + 256;
    return w;
}

#define JLB_ES_LAUNCH(kernel, es, grid, threads, st, ...)                                 \
    do {                                                                                   \
        if ((es) == 8) conv::kernel<8><<<(grid), (threads), 0, (st)>>>(__VA_ARGS__);      \
        else if ((es) == 4) conv::kernel<4><<<(grid), (threads), 0, (st)>>>(__VA_ARGS__); \
        else conv::kernel<2><<<(grid), (threads), 0, (st)>>>(__VA_ARGS__);                \
    } while (0)

// Keep bytes and tile first slots (tfirst[ntiles] = the kept total); with
// row_counts (zeroed), each row's kept count too.  merge: adjacent equal
// coordinates keep their first value (CSR targets), else only zeros go (COO
// targets).
int coo_csr_slots(cudaStream_t st, int dtype, int idx_base, int64_t m, int64_t n, int64_t nnz,
                  const int32_t *rows, const int32_t *cols, const void *val, const CooCsrWs &w,
                  bool merge = true, int32_t *row_counts = nullptr) {
    if (nnz > 0) {
        JLB_ES_LAUNCH(coo_keep_tiles, dtype_size(dtype), (unsigned)w.ntiles, conv::kThreads, st, nnz,
                      rows, cols, val, idx_base, m, n, merge, w.keep, w.tcount, row_counts);
        JLB_LAUNCH_CHECK("coo_keep_tiles");
        return conv::scan(st, w.ntiles, w.tcount, w.tfirst, 0, w.scan, w.scan_bytes);
    }
    JLB_CUDA(cudaMemsetAsync(w.tfirst, 0, (size_t)(w.ntiles + 1) * sizeof(int32_t), st));
    return ok();
}
}  // namespace

extern "C" JLB_API size_t jlb_coo_to_csr_workspace_size(int64_t m, int64_t n, int64_t nnz) {
    if (m < 0 || nnz < 0) return 0;
    return coo_csr_ws(nullptr, nnz, m).bytes;
}

extern "C" JLB_API int jlb_coo_to_csr_count(void *stream, int dtype, int idx_base, int64_t m,
                                            int64_t n, int64_t nnz, const int32_t *rows,
                                            const int32_t *cols, const void *val, int32_t *rowptr,
                                            int64_t *nnz_out, void *workspace,
                                            size_t workspace_bytes) {
    int r = conv_args(dtype, idx_base, m, n, nnz, 1, 1);
    if (r) return r;
    if (m > INT32_MAX - 1) return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "rows exceed Int32");
    if (!rowptr || !nnz_out || (nnz > 0 && (!rows || !cols || !val)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    const CooCsrWs w = coo_csr_ws(workspace, nnz, m);
    if (!workspace || workspace_bytes < w.bytes) return fail(JLB_ERR_WORKSPACE, "workspace too small");
    cudaStream_t st = as_stream(stream);
    if (m > 0) JLB_CUDA(cudaMemsetAsync(w.rowcnt, 0, (size_t)m * sizeof(int32_t), st));
    r = coo_csr_slots(st, dtype, idx_base, m, n, nnz, rows, cols, val, w, true, w.rowcnt);
    if (r) return r;
    // the row pointer: the exclusive scan of the rows' kept counts
    r = conv::scan(st, m, w.rowcnt, rowptr, idx_base, w.scan, w.scan_bytes);
    if (r) return r;
    // b1 = b2 = -2 marks a COO -> CSR workspace
    const uint64_t key = carry_key(m, n, nnz, -2, -2, idx_base, dtype, rows, cols, val);
    JLB_CUDA(cudaMemcpyAsync(w.stamp, &key, sizeof(key), cudaMemcpyHostToDevice, st));
    int32_t total = 0;
    JLB_CUDA(cudaMemcpyAsync(&total, w.tfirst + w.ntiles, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    JLB_CUDA(cudaStreamSynchronize(st));
    const int bits = take_dev_error_convert();
    if (bits < 0) return fail(JLB_ERR_CUDA, "reading the device error word failed");
    if (bits & DEV_ERR_BOUNDS)
        return fail(JLB_ERR_NONCANONICAL_STORAGE, "coordinate outside the matrix extents");
    if (bits & DEV_ERR_OVERFLOW)
        return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "kept entries overflow Int32 positions");
    if (bits & DEV_ERR_ORDER)
        return fail(JLB_ERR_NONCANONICAL_STORAGE,
                    "COO rows must not decrease (the COO format declares its rows ordered)");
    *nnz_out = total;
    return ok();
}

extern "C" JLB_API int jlb_coo_to_csr_fill(void *stream, int dtype, int idx_base, int64_t m,
                                           int64_t n, int64_t nnz, const int32_t *rows,
                                           const int32_t *cols, const void *val, int64_t nnz_out,
                                           int32_t *colind, void *csr_val, void *workspace,
                                           size_t workspace_bytes) {
    int r = conv_args(dtype, idx_base, m, n, nnz, 1, 1);
    if (r) return r;
    if ((nnz > 0 && (!rows || !cols || !val)) || (nnz_out > 0 && (!colind || !csr_val)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    if (nnz_out < 0 || nnz_out > nnz) return fail(JLB_ERR_INVALID_ARGUMENT, "bad nnz_out");
    const CooCsrWs w = coo_csr_ws(workspace, nnz, m);
    if (!workspace || workspace_bytes < w.bytes) return fail(JLB_ERR_WORKSPACE, "workspace too small");
    if (nnz == 0) return ok();
    cudaStream_t st = as_stream(stream);
    uint64_t stamp = 0;
    JLB_CUDA(cudaMemcpyAsync(&stamp, w.stamp, sizeof(stamp), cudaMemcpyDeviceToHost, st));
    JLB_CUDA(cudaStreamSynchronize(st));
    if (stamp != carry_key(m, n, nnz, -2, -2, idx_base, dtype, rows, cols, val)) {
        r = coo_csr_slots(st, dtype, idx_base, m, n, nnz, rows, cols, val, w);
        if (r) return r;
    }
    JLB_ES_LAUNCH(coo_emit_tiles, dtype_size(dtype), (unsigned)w.ntiles, conv::kThreads, st, nnz,
                  rows, cols, val, w.keep, w.tfirst, nnz_out, nullptr, colind, csr_val);
    JLB_LAUNCH_CHECK("coo_emit_tiles");
    return ok();
}

// ------------------------------------------------------------- COO -> COO
// A COO target's levels are not unique and the source is not sorted
// (src/convert.jl:346-355), so the composer only loses the explicit zeros:
// a stable compaction without merging (CSR -> COO after the rows are
// expanded, COO -> COO).  Workspace as for COO -> CSR; fill recomputes.
extern "C" JLB_API size_t jlb_coo_drop_zeros_workspace_size(int64_t nnz) {
    if (nnz < 0) return 0;
    return coo_csr_ws(nullptr, nnz, 0).bytes;
}

extern "C" JLB_API int jlb_coo_drop_zeros_count(void *stream, int dtype, int idx_base, int64_t m,
                                                int64_t n, int64_t nnz, const int32_t *rows,
                                                const int32_t *cols, const void *val,
                                                int64_t *nnz_out, void *workspace,
                                                size_t workspace_bytes) {
    int r = conv_args(dtype, idx_base, m, n, nnz, 1, 1);
    if (r) return r;
    if (!nnz_out || (nnz > 0 && (!rows || !cols || !val)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    const CooCsrWs w = coo_csr_ws(workspace, nnz, 0);
    if (!workspace || workspace_bytes < w.bytes) return fail(JLB_ERR_WORKSPACE, "workspace too small");
    cudaStream_t st = as_stream(stream);
    r = coo_csr_slots(st, dtype, idx_base, m, n, nnz, rows, cols, val, w, false);
    if (r) return r;
    int32_t total = 0;
    JLB_CUDA(cudaMemcpyAsync(&total, w.tfirst + w.ntiles, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    JLB_CUDA(cudaStreamSynchronize(st));
    const int bits = take_dev_error_convert();
    if (bits < 0) return fail(JLB_ERR_CUDA, "reading the device error word failed");
    if (bits & DEV_ERR_BOUNDS)
        return fail(JLB_ERR_NONCANONICAL_STORAGE, "coordinate outside the matrix extents");
    if (bits & DEV_ERR_OVERFLOW)
        return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "kept entries overflow Int32 positions");
    *nnz_out = total;
    return ok();
}

extern "C" JLB_API int jlb_coo_drop_zeros_fill(void *stream, int dtype, int idx_base, int64_t m,
                                               int64_t n, int64_t nnz, const int32_t *rows,
                                               const int32_t *cols, const void *val,
                                               int64_t nnz_out, int32_t *rows_out,
                                               int32_t *cols_out, void *val_out, void *workspace,
                                               size_t workspace_bytes) {
    int r = conv_args(dtype, idx_base, m, n, nnz, 1, 1);
    if (r) return r;
    if ((nnz > 0 && (!rows || !cols || !val)) ||
        (nnz_out > 0 && (!rows_out || !cols_out || !val_out)))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    if (nnz_out < 0 || nnz_out > nnz) return fail(JLB_ERR_INVALID_ARGUMENT, "bad nnz_out");
    const CooCsrWs w = coo_csr_ws(workspace, nnz, 0);
    if (!workspace || workspace_bytes < w.bytes) return fail(JLB_ERR_WORKSPACE, "workspace too small");
    if (nnz == 0) return ok();
    cudaStream_t st = as_stream(stream);
    r = coo_csr_slots(st, dtype, idx_base, m, n, nnz, rows, cols, val, w, false);
    if (r) return r;
    JLB_ES_LAUNCH(coo_emit_tiles, dtype_size(dtype), (unsigned)w.ntiles, conv::kThreads, st, nnz,
                  rows, cols, val, w.keep, w.tfirst, nnz_out, rows_out, cols_out, val_out);
    JLB_LAUNCH_CHECK("coo_emit_tiles");
    return ok();
}
