// spmm.cu -- CSR SpMM (C = alpha*A*B + beta*C) for sm_100a.
//
// Fast path (B and C row-major, 16-byte aligned rows).  The work is one
// gather of a B row per stored entry of A.  A group of 8 lanes works on a
// 256-byte column chunk of an output row (64 fp32 / 32 fp64 columns; lane l
// owns 16-byte vectors l and 8 + l).  Each lane copies its part of an entry's
// B-row chunk into one of the group's kDepth shared-memory slots with
// cp.async.cg (L2 only); the lanes add slot i while the copies for the next
// kDepth - 1 entries are in flight.  Holding the data in flight in shared
// memory instead of registers keeps registers at 64 and 32 warps resident per
// SM; measured on config 3 (power-law, k = 64), more resident warps with 3
// slots each beat deeper pipelines (1.37 ms per SpMM at depth 3, 4 CTAs/SM;
// 2.5 ms at depth 12, 2 CTAs/SM; 2.0 ms with registers as slots).  The
// untiled bulk copy (cp.async.bulk, one 256-byte copy per entry) was slower
// still (3.9 ms): per-copy cost dominates at this size.
//
// spmm_stream: each group owns a contiguous range of rows, balanced by rows +
// entries (each group finds its range with a 9-ary search of the row
// pointer), and streams through the range's entries in storage order across
// row boundaries; a row's chunk of C is stored when its last entry is in.
// Per output element the sum runs over the row's entries in storage order with
// separately rounded products and sums: the same operations as JLUST's Tiled
// SpMM body (ext/KernelAbstractionsExt/ops/spmm.jl:272-292), hence
// bit-identical.
//
// spmm_long_rows: rows longer than kLong entries, which the stream skips.  A
// CTA lists the long rows among kScanRows rows in ascending order and splits
// them into contiguous segments, each row getting groups in proportion to its
// length; the segments' partial sums are added in segment order
// (deterministic, within tolerance).  No atomics touch C.
//
// Generic path (any order / alignment): one thread per output element, the
// same storage-order sum.
#include "common.cuh"

#include <mutex>

namespace jlb {

JLB_DEFINE_DEV_ERROR(spmm)

namespace spmm {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

constexpr int kThreads = 256;
constexpr int kGroup = 8;                      // lanes per group
constexpr int kVec = 2;                        // 16-byte vectors per lane per B-row chunk
constexpr int kGroups = kThreads / kGroup;     // groups per CTA
constexpr int kChunkBytes = kGroup * kVec * 16;  // one B-row chunk (256 bytes)
constexpr int kLong = 256;                     // longer rows go to spmm_long_rows
constexpr int kDepth = 3;                      // B-row chunks in flight per group
constexpr int kMinWork = 64;                   // rows + entries per stream group, at least
constexpr int kScanRows = 256;                 // rows a long-row CTA inspects
constexpr int kSlotBytes = kGroups * kDepth * kChunkBytes;

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
// l sits at vector index w*kGroup + l (byte offset 16 * (w*kGroup + l) in the
// chunk), so each access of the group covers 128 contiguous bytes.
template <typename T>
struct Lanes {
    static constexpr int E = V16<T>::E;
    static constexpr int CW = kGroup * kVec * E;   // columns per chunk
    __device__ static int64_t col(int64_t c0, int lane, int w) { return c0 + ((int64_t)w * kGroup + lane) * E; }
};

// A group's slots: kDepth shared-memory chunks of 256 bytes.  Each lane
// copies its own two 16-byte vectors of an entry's B-row chunk with
// cp.async.cg (L2 only, no registers held while in flight) and commits one
// copy group per slot refill, empty when there is no entry left, so that
// `cp.async.wait_group kDepth-1` before reading slot u means slot u has
// landed.  A lane reads back only what it copied itself: no barrier.
template <typename T>
struct Slots {
    uint32_t buf;      // shared address of this lane's first vector in slot 0
    const unsigned char *data;   // generic pointer to the same
    int lane;
    bool ok[kVec];     // vector w of this lane lies inside the matrix

    __device__ void issue(int u, const T *row_c0) const {
#pragma unroll
        for (int w = 0; w < kVec; ++w)
            if (ok[w])
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                                 buf + (uint32_t)(u * kChunkBytes + w * kGroup * 16)),
                             "l"(row_c0 + (w * kGroup + lane) * V16<T>::E)
                             : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    __device__ void skip() const { asm volatile("cp.async.commit_group;" ::: "memory"); }
    // Waits for slot u (the oldest copy group in flight) and adds v * chunk.
    __device__ void add(int u, T v, T (&acc)[kVec][V16<T>::E]) const {
        using VT = typename V16<T>::type;
        asm volatile("cp.async.wait_group %0;" ::"n"(kDepth - 1) : "memory");
#pragma unroll
        for (int w = 0; w < kVec; ++w)
            if (ok[w]) {
                const VT b = *reinterpret_cast<const VT *>(data + u * kChunkBytes + w * kGroup * 16);
#pragma unroll
                for (int e = 0; e < V16<T>::E; ++e)
                    acc[w][e] = add_rn(acc[w][e], mul_rn(v, V16<T>::get(b, e)));
            }
    }
};

template <typename T>
__device__ __forceinline__ Slots<T> group_slots(unsigned char *smem, int group, int lane) {
    Slots<T> s;
    s.data = smem + (size_t)group * kDepth * kChunkBytes + lane * 16;
    s.buf = smem_u32(s.data);
    s.lane = lane;
    return s;
}

template <typename T>
__device__ __forceinline__ void set_chunk(Slots<T> &s, int64_t c0, int64_t k) {
#pragma unroll
    for (int w = 0; w < kVec; ++w) s.ok[w] = Lanes<T>::col(c0, s.lane, w) < k;
}

// Stores a row's chunk of C: 16-byte vectors into a row-major C, or scalars
// into a column-major C (element (row, col) at row + col*ldc, Julia's layout).
// A group walks consecutive rows, so the 32-byte sectors of a column-major C
// fill up in L2 before they are written back.
template <typename T, bool kBeta, bool kColC>
__device__ __forceinline__ void store_chunk(T *C, int64_t ldc, int64_t row, int64_t c0, int64_t k,
                                            const T (&acc)[kVec][V16<T>::E], T alpha, T beta,
                                            int lane) {
    using VT = typename V16<T>::type;
    constexpr int E = V16<T>::E;
#pragma unroll
    for (int w = 0; w < kVec; ++w) {
        const int64_t col = Lanes<T>::col(c0, lane, w);
        if (col >= k) continue;
        if (kColC) {
#pragma unroll
            for (int e = 0; e < E; ++e) {
                T *d = C + row + (col + e) * ldc;
                T o = mul_rn(alpha, acc[w][e]);
                if (kBeta) o = add_rn(o, mul_rn(beta, *d));
                *d = o;
            }
            continue;
        }
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
// both (kGroup+1)-ary searches run together, each lane of the group probing one point
// of each interval per step (about log9(m) dependent loads).
__device__ __forceinline__ void find_rows(int64_t m, const int32_t *__restrict__ rowptr, int base,
                                          int64_t t0, int64_t t1, int lane, unsigned gmask,
                                          int shift, int64_t &r0, int64_t &r1) {
    int64_t lo0 = 0, hi0 = m, lo1 = 0, hi1 = m;
    while (lo0 < hi0 || lo1 < hi1) {
        const int64_t p0 = lo0 + (hi0 - lo0) * (lane + 1) / (kGroup + 1);
        const int64_t p1 = lo1 + (hi1 - lo1) * (lane + 1) / (kGroup + 1);
        const bool q0 = lo0 < hi0 && p0 + (ldg(rowptr + p0) - base) >= t0;
        const bool q1 = lo1 < hi1 && p1 + (ldg(rowptr + p1) - base) >= t1;
        const unsigned b0 = (__ballot_sync(gmask, q0) >> shift) & ((1u << kGroup) - 1u);
        const unsigned b1 = (__ballot_sync(gmask, q1) >> shift) & ((1u << kGroup) - 1u);
        if (lo0 < hi0) {
            const int64_t span = hi0 - lo0;
            if (b0) {
                const int f = __ffs(b0) - 1;
                hi0 = lo0 + span * (f + 1) / (kGroup + 1);
                if (f > 0) lo0 = lo0 + span * f / (kGroup + 1) + 1;
            } else {
                lo0 = lo0 + span * kGroup / (kGroup + 1) + 1;
            }
        }
        if (lo1 < hi1) {
            const int64_t span = hi1 - lo1;
            if (b1) {
                const int f = __ffs(b1) - 1;
                hi1 = lo1 + span * (f + 1) / (kGroup + 1);
                if (f > 0) lo1 = lo1 + span * f / (kGroup + 1) + 1;
            } else {
                lo1 = lo1 + span * kGroup / (kGroup + 1) + 1;
            }
        }
    }
    r0 = lo0;
    r1 = lo1;
}

// Moves the issue cursor to the first entry of the next row in (r, re) that
// has entries and at most kLong of them; r == re when there is none.  e holds
// the end of row r on entry.
__device__ __forceinline__ void issue_seek(int &r, int &p, int &e, int re,
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
// longer than kLong excluded) with kDepth B-row chunks in flight, storing each
// row's chunk of C when its last entry is in, and the chunk of every empty row
// as alpha * 0 (+ beta * C).
template <typename T, bool kBeta, bool kColC>
__global__ void __launch_bounds__(kThreads, 4)
spmm_stream(int64_t m, int64_t k, const int32_t *__restrict__ rowptr,
            const int32_t *__restrict__ colind, const T *__restrict__ val,
            const T *__restrict__ B, int64_t ldb, T *__restrict__ C, int64_t ldc, T alpha, T beta,
            int base) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x;
    const int lane = tid % kGroup;
    const unsigned gmask = group_mask(tid);
    const int shift = (tid % kWarp) / kGroup * kGroup;
    const int64_t groups = (int64_t)gridDim.x * kGroups;
    const int64_t g = (int64_t)blockIdx.x * kGroups + tid / kGroup;
    const int64_t total = m + (int64_t)(ldg(rowptr + m) - base);
    int64_t rs64, re64;
    find_rows(m, rowptr, base, total * g / groups, total * (g + 1) / groups, lane, gmask, shift,
              rs64, re64);
    // row cursors in 32 bits (the launcher takes this path for m < 2^31 only)
    const int rs = (int)rs64, re = (int)re64;
    // no early exit: the whole warp stays in the loops below, which end when
    // every group of the warp is done, so its four groups reconverge every
    // iteration instead of running one after another
    const int first = ldg(rowptr + rs) - base;
    Slots<T> sl = group_slots<T>(smem, tid / kGroup, lane);

    for (int64_t c0 = 0; c0 < k; c0 += Lanes<T>::CW) {
        set_chunk(sl, c0, k);
        T acc[kVec][V16<T>::E];
        zero(acc);

        // consume cursor: row rc, next entry cp, row end ce.  Rows before the
        // first short non-empty one are stored now (empty) or skipped (long).
        int rc = rs - 1;
        int cp = first, ce = first;
        for (;;) {
            if (++rc >= re) break;
            const int lo = ce;
            ce = ldg(rowptr + rc + 1) - base;
            if (ce - lo > kLong || ce < lo) continue;
            if (ce == lo) {
                store_chunk<T, kBeta, kColC>(C, ldc, rc, c0, k, acc, alpha, beta, lane);
                continue;
            }
            cp = lo;
            break;
        }
        // issue cursor, kDepth entries ahead of the consume cursor
        int ri = rc;
        int ip = cp, ie = ce;
        T v[kDepth];
        uint32_t live = 0;   // bit u: slot u holds an entry
#pragma unroll
        for (int u = 0; u < kDepth; ++u) {
            if (ri < re) {
                live |= 1u << u;
                v[u] = ldg(val + ip);
                sl.issue(u, B + (int64_t)(ldg(colind + ip) - base) * ldb + c0);
                if (++ip >= ie) issue_seek(ri, ip, ie, re, rowptr, base);
            } else {
                sl.skip();
            }
        }
        while (__any_sync(0xffffffffu, live & 1u)) {
#pragma unroll
            for (int u = 0; u < kDepth; ++u) {
                if (!(live >> u & 1u)) continue;
                sl.add(u, v[u], acc);
                if (++cp >= ce) {
                    store_chunk<T, kBeta, kColC>(C, ldc, rc, c0, k, acc, alpha, beta, lane);
                    zero(acc);
                    for (;;) {
                        if (++rc >= re) break;
                        const int lo = ce;
                        ce = ldg(rowptr + rc + 1) - base;
                        if (ce - lo > kLong || ce < lo) continue;
                        if (ce == lo) {
                            store_chunk<T, kBeta, kColC>(C, ldc, rc, c0, k, acc, alpha, beta, lane);
                            continue;
                        }
                        cp = lo;
                        break;
                    }
                }
                if (ri < re) {
                    v[u] = ldg(val + ip);
                    sl.issue(u, B + (int64_t)(ldg(colind + ip) - base) * ldb + c0);
                    if (++ip >= ie) issue_seek(ri, ip, ie, re, rowptr, base);
                } else {
                    live &= ~(1u << u);
                    sl.skip();
                }
            }
        }
    }
}

// Adds entries [lo, hi) of one row, in storage order, into acc with kDepth
// chunks in flight.
template <typename T>
__device__ __forceinline__ void range_accumulate(const Slots<T> &sl, T (&acc)[kVec][V16<T>::E],
                                                 int lo, int hi,
                                                 const int32_t *__restrict__ colind,
                                                 const T *__restrict__ val,
                                                 const T *__restrict__ B, int64_t ldb, int64_t c0,
                                                 int base) {
    T v[kDepth];
#pragma unroll
    for (int u = 0; u < kDepth; ++u) {
        if (lo + u < hi) {
            v[u] = ldg(val + lo + u);
            sl.issue(u, B + (int64_t)(ldg(colind + lo + u) - base) * ldb + c0);
        } else {
            sl.skip();
        }
    }
    for (int p = lo; p < hi; p += kDepth) {
#pragma unroll
        for (int u = 0; u < kDepth; ++u) {
            if (p + u >= hi) break;
            sl.add(u, v[u], acc);
            const int q = p + u + kDepth;
            if (q < hi) {
                v[u] = ldg(val + q);
                sl.issue(u, B + (int64_t)(ldg(colind + q) - base) * ldb + c0);
            } else {
                sl.skip();
            }
        }
    }
}

// Long rows.  The CTA lists the rows longer than kLong among its kScanRows
// rows in ascending order (block scan of per-thread counts), then works
// through the list in rounds of up to kGroups rows.  In a round row i gets
// g_i = 1 + (kGroups - n) * L_i / E groups (n rows, L_i entries, E their sum),
// each taking one contiguous segment of ceil(L_i / g_i) entries; the first
// group of the row adds the g_i partial sums in segment order and stores the
// chunk.  Allocation and order depend only on the matrix: deterministic.
template <typename T, bool kBeta, bool kColC>
__global__ void __launch_bounds__(kThreads, 4)
spmm_long_rows(int64_t m, int64_t k, const int32_t *__restrict__ rowptr,
               const int32_t *__restrict__ colind, const T *__restrict__ val,
               const T *__restrict__ B, int64_t ldb, T *__restrict__ C, int64_t ldc, T alpha,
               T beta, int base) {
    constexpr int E = V16<T>::E;
    constexpr int kPer = kScanRows / kThreads;   // rows each thread inspects
    extern __shared__ __align__(128) unsigned char smem[];
    T(*s_part)[kVec * kGroup * E] = reinterpret_cast<T(*)[kVec * kGroup * E]>(smem + kSlotBytes);
    int *s_row = reinterpret_cast<int *>(smem + kSlotBytes + kGroups * kChunkBytes);
    int *s_len = s_row + kScanRows;
    __shared__ int s_warp[kThreads / kWarp];
    __shared__ int s_n;
    const int tid = threadIdx.x;
    const int gi = tid / kGroup, lane = tid % kGroup;
    const unsigned gmask = group_mask(tid);
    const int64_t r0 = (int64_t)blockIdx.x * kScanRows;

    // ascending list of long rows: per-thread counts, warp scan, block offsets
    int lens[kPer];
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int64_t r = r0 + (int64_t)tid * kPer + j;
        lens[j] = r < m ? ldg(rowptr + r + 1) - ldg(rowptr + r) : 0;
        cnt += lens[j] > kLong;
    }
    int incl = cnt;
#pragma unroll
    for (int d = 1; d < kWarp; d <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, d);
        if (tid % kWarp >= d) incl += t;
    }
    if (tid % kWarp == kWarp - 1) s_warp[tid / kWarp] = incl;
    __syncthreads();
    int off = incl - cnt;
    for (int w = 0; w < tid / kWarp; ++w) off += s_warp[w];
    if (tid == kThreads - 1) s_n = off + cnt;
#pragma unroll
    for (int j = 0; j < kPer; ++j)
        if (lens[j] > kLong) {
            s_row[off] = tid * kPer + j;
            s_len[off] = lens[j];
            ++off;
        }
    __syncthreads();
    const int n = s_n;
    if (n == 0) return;

    Slots<T> sl = group_slots<T>(smem, gi, lane);
    for (int i0 = 0; i0 < n; i0 += kGroups) {
        const int nr = n - i0 < kGroups ? n - i0 : kGroups;
        int64_t tot = 0;
        for (int i = 0; i < nr; ++i) tot += s_len[i0 + i];
        // this group's row, its first group and its group count
        int row = -1, first = 0, cnt_g = 0, acc_g = 0;
        for (int i = 0; i < nr; ++i) {
            const int gcount = 1 + (int)((int64_t)(kGroups - nr) * s_len[i0 + i] / tot);
            if (gi >= acc_g && gi < acc_g + gcount) {
                row = i0 + i;
                first = acc_g;
                cnt_g = gcount;
            }
            acc_g += gcount;
        }
        int slo = 0, shi = 0;
        int64_t r = 0;
        if (row >= 0) {
            r = r0 + s_row[row];
            const int lo = ldg(rowptr + r) - base, hi = ldg(rowptr + r + 1) - base;
            const int seg = (hi - lo + cnt_g - 1) / cnt_g;
            const int s = gi - first;
            slo = lo + s * seg < hi ? lo + s * seg : hi;
            shi = slo + seg < hi ? slo + seg : hi;
        }
        for (int64_t c0 = 0; c0 < k; c0 += Lanes<T>::CW) {
            set_chunk(sl, c0, k);
            T acc[kVec][E];
            zero(acc);
            if (row >= 0) range_accumulate<T>(sl, acc, slo, shi, colind, val, B, ldb, c0, base);
#pragma unroll
            for (int w = 0; w < kVec; ++w)
#pragma unroll
                for (int e = 0; e < E; ++e) s_part[gi][(w * kGroup + lane) * E + e] = acc[w][e];
            __syncthreads();
            if (row >= 0 && gi == first) {
                T sum[kVec][E];
#pragma unroll
                for (int w = 0; w < kVec; ++w)
#pragma unroll
                    for (int e = 0; e < E; ++e) {
                        const int idx = (w * kGroup + lane) * E + e;
                        sum[w][e] = s_part[first][idx];
                        for (int q = 1; q < cnt_g; ++q) sum[w][e] = add_rn(sum[w][e], s_part[first + q][idx]);
                    }
                store_chunk<T, kBeta, kColC>(C, ldc, r, c0, k, sum, alpha, beta, lane);
            }
            __syncthreads();
        }
    }
}

constexpr int kStreamSmem = kSlotBytes;
constexpr int kLongSmem = kSlotBytes + kGroups * kChunkBytes + 2 * kScanRows * 4;

// Opts the kernels into their dynamic shared memory once per device and
// returns the stream kernel's resident CTAs per SM times the SM count.
template <typename T, bool kBeta, bool kColC>
int prepare_kernels(int *grid_full) {
    // one grid size per device, filled under a lock: two host threads making
    // their first call at once both see either nothing or the whole entry
    static int grid[64] = {0};
    static std::mutex mu;
    int dev = 0;
    JLB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(JLB_ERR_DEVICE_MISMATCH, "device ordinal %d", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!grid[dev]) {
        JLB_CUDA(cudaFuncSetAttribute(spmm_stream<T, kBeta, kColC>, cudaFuncAttributeMaxDynamicSharedMemorySize, kStreamSmem));
        JLB_CUDA(cudaFuncSetAttribute(spmm_long_rows<T, kBeta, kColC>, cudaFuncAttributeMaxDynamicSharedMemorySize, kLongSmem));
        int sms = 0, p = 0;
        JLB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        JLB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&p, spmm_stream<T, kBeta, kColC>, kThreads, kStreamSmem));
        grid[dev] = (p < 1 ? 1 : p) * sms;
    }
    *grid_full = grid[dev];
    return JLB_OK;
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

template <typename T, bool kBeta, bool kColC>
int launch_fast(cudaStream_t st, int base, int64_t m, int64_t nnz, int64_t k,
                const int32_t *rowptr, const int32_t *colind, const T *val, const T *B,
                int64_t ldb, T *C, int64_t ldc, T a, T b) {
    int full = 0;
    const int rc = prepare_kernels<T, kBeta, kColC>(&full);
    if (rc != JLB_OK) return rc;
    const int64_t need = ceil_div(m + nnz, (int64_t)kGroups * kMinWork);
    const unsigned grid = (unsigned)(need < full ? need : full);
    spmm_stream<T, kBeta, kColC><<<grid, kThreads, kStreamSmem, st>>>(m, k, rowptr, colind, val, B,
                                                                      ldb, C, ldc, a, b, base);
    spmm_long_rows<T, kBeta, kColC><<<(unsigned)ceil_div(m, kScanRows), kThreads, kLongSmem, st>>>(
        m, k, rowptr, colind, val, B, ldb, C, ldc, a, b, base);
    JLB_LAUNCH_CHECK("spmm_stream");
    return ok();
}

template <typename T>
int launch_fast_any(cudaStream_t st, int base, int64_t m, int64_t nnz, int64_t k,
                    const int32_t *rowptr, const int32_t *colind, const T *val, const T *B,
                    int64_t ldb, T *C, int64_t ldc, bool col_c, T a, T b) {
    if (b == T(0))
        return col_c ? launch_fast<T, false, true>(st, base, m, nnz, k, rowptr, colind, val, B, ldb, C, ldc, a, b)
                     : launch_fast<T, false, false>(st, base, m, nnz, k, rowptr, colind, val, B, ldb, C, ldc, a, b);
    return col_c ? launch_fast<T, true, true>(st, base, m, nnz, k, rowptr, colind, val, B, ldb, C, ldc, a, b)
                 : launch_fast<T, true, false>(st, base, m, nnz, k, rowptr, colind, val, B, ldb, C, ldc, a, b);
}

// out (cols x rows, row-major, leading dim ldo) = in^T for in rows x cols
// row-major (leading dim ldi): 64 x 64 tiles through shared memory (padded a
// column, no bank conflicts either way), 16 loads in flight per thread, both
// sides in 128-byte warp accesses.  Turns a column-major n x k B (a row-major
// k x n array) into the row-major n x k copy the stream kernels gather rows
// from, and a row-major C back into a column-major one.
constexpr int kTile = 64;
template <typename T>
__global__ void __launch_bounds__(256, 4)
transpose_tiles(int64_t rows, int64_t cols, const T *__restrict__ in, int64_t ldi,
                T *__restrict__ out, int64_t ldo) {
    __shared__ T tile[kTile][kTile + 1];
    const int tx = threadIdx.x % kTile, ty = threadIdx.x / kTile;   // 64 x 4 threads
    const int64_t c0 = (int64_t)blockIdx.x * kTile;
    for (int64_t r0 = (int64_t)blockIdx.y * kTile; r0 < rows; r0 += (int64_t)gridDim.y * kTile) {
        const int64_t c = c0 + tx;
#pragma unroll
        for (int j = 0; j < kTile / 4; ++j) {
            const int64_t r = r0 + ty + 4 * j;
            if (r < rows && c < cols) tile[ty + 4 * j][tx] = __ldcs(in + r * ldi + c);
        }
        __syncthreads();
        const int64_t ocol = r0 + tx;
#pragma unroll
        for (int j = 0; j < kTile / 4; ++j) {
            const int64_t orow = c0 + ty + 4 * j;
            if (orow < cols && ocol < rows) __stcs(out + orow * ldo + ocol, tile[tx][ty + 4 * j]);
        }
        __syncthreads();
    }
}

inline size_t bt_bytes(int64_t n, int64_t k, size_t es) { return (size_t)n * (size_t)k * es + 256; }

// Workspace of a call with column-major operands: [row-major copy of B (n x k)
// when B is column-major | row-major C (m x k) when C is column-major], each
// part 256-byte aligned.
inline size_t ws_bytes_for(int64_t m, int64_t n, int64_t k, int b_order, int c_order, size_t es) {
    size_t b = 0;
    if (b_order == JLB_COL_MAJOR && n > 0 && k > 0) b += bt_bytes(n, k, es);
    if (c_order == JLB_COL_MAJOR && m > 0 && k > 0) b += bt_bytes(m, k, es);
    return b;
}

template <typename T>
void transpose(cudaStream_t st, int64_t rows, int64_t cols, const T *in, int64_t ldi, T *out,
               int64_t ldo) {
    const int64_t gx = ceil_div(cols, kTile);
    const int64_t gy = ceil_div(rows, kTile) < 65535 ? ceil_div(rows, kTile) : 65535;
    transpose_tiles<T><<<dim3((unsigned)gx, (unsigned)gy), 256, 0, st>>>(rows, cols, in, ldi, out,
                                                                       ldo);
}

template <typename T>
int launch(cudaStream_t st, int base, int64_t m, int64_t n, int64_t nnz, int64_t k,
           const int32_t *rowptr, const int32_t *colind, const void *val, const void *B,
           int64_t ldb, int b_order, void *C, int64_t ldc, int c_order, double alpha,
           double beta, void *ws, size_t ws_bytes) {
    if (m == 0 || k == 0) return ok();
    constexpr int E = V16<T>::E;
    const T a = (T)alpha, b = (T)beta;
    // C: row-major with 16-byte aligned rows, or column-major (scalar stores)
    const bool c_fast = (c_order == JLB_ROW_MAJOR && ldc % E == 0 && aligned16(C)) ||
                        c_order == JLB_COL_MAJOR;
    const bool shape_fast = m < INT32_MAX && k % E == 0 && c_fast;
    const bool col_c = c_order == JLB_COL_MAJOR;
    const bool b_fast = b_order == JLB_ROW_MAJOR && ldb % E == 0 && aligned16(B);
    // Column-major operands (Julia's layout).  A column-major B row is k
    // strided elements, each in its own sector, and a column-major C row is
    // k stores 4*m bytes apart (a different page each): with a workspace, B
    // is transposed once into a row-major copy whose rows are gathered, and
    // C is computed row-major in the workspace and transposed out (in first
    // as well when beta != 0).  The arithmetic is the row-major path's.
    const bool b_col = b_order == JLB_COL_MAJOR;
    if (m < INT32_MAX && k % E == 0 && (b_col || b_fast) && (b_col || col_c) && ws &&
        ws_bytes >= ws_bytes_for(m, n, k, b_order, c_order, sizeof(T))) {
        uintptr_t cur = (reinterpret_cast<uintptr_t>(ws) + 255) & ~(uintptr_t)255;
        const T *bsrc = (const T *)B;
        int64_t ldb_use = ldb;
        if (b_col && n > 0) {
            T *bt = reinterpret_cast<T *>(cur);
            cur = (cur + (size_t)n * (size_t)k * sizeof(T) + 255) & ~(uintptr_t)255;
            transpose<T>(st, k, n, (const T *)B, ldb, bt, k);
            JLB_LAUNCH_CHECK("transpose_tiles (B)");
            bsrc = bt;
            ldb_use = k;
        }
        T *cdst = (T *)C;
        int64_t ldc_use = ldc;
        if (col_c) {
            cdst = reinterpret_cast<T *>(cur);
            ldc_use = k;
            if (b != T(0)) {
                transpose<T>(st, k, m, (const T *)C, ldc, cdst, k);
                JLB_LAUNCH_CHECK("transpose_tiles (C in)");
            }
        }
        int rc = launch_fast_any<T>(st, base, m, nnz, k, rowptr, colind, (const T *)val, bsrc,
                                    ldb_use, cdst, ldc_use, false, a, b);
        if (rc != JLB_OK) return rc;
        if (col_c) {
            transpose<T>(st, m, k, cdst, k, (T *)C, ldc);
            JLB_LAUNCH_CHECK("transpose_tiles (C out)");
        }
        return ok();
    }
    // row-major B; C row-major, or column-major stored by scalars (no workspace)
    if (shape_fast && b_fast)
        return launch_fast_any<T>(st, base, m, nnz, k, rowptr, colind, (const T *)val,
                                  (const T *)B, ldb, (T *)C, ldc, col_c, a, b);
    const int64_t total = m * k;
    const unsigned grid = (unsigned)(ceil_div(total, 256) < 148 * 32 ? ceil_div(total, 256) : 148 * 32);
    spmm_generic<T><<<grid, 256, 0, st>>>(m, k, rowptr, colind, (const T *)val, (const T *)B,
                                          ldb, b_order, (T *)C, ldc, c_order, a, b, base,
                                          b != T(0));
    JLB_LAUNCH_CHECK("spmm_generic");
    return ok();
}

}  // namespace spmm
}  // namespace jlb

using namespace jlb;

static int csr_spmm(void *stream, int dtype, int idx_base, int64_t m, int64_t n, int64_t nnz,
                    const int32_t *rowptr, const int32_t *colind, const void *val, int64_t k,
                    const void *B, int64_t ldb, int b_order, void *C, int64_t ldc, int c_order,
                    double alpha, double beta, void *ws, size_t ws_bytes) {
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
        return spmm::launch<double>(as_stream(stream), idx_base, m, n, nnz, k, rowptr, colind, val, B,
                                    ldb, b_order, C, ldc, c_order, alpha, beta, ws, ws_bytes);
    return spmm::launch<float>(as_stream(stream), idx_base, m, n, nnz, k, rowptr, colind, val, B,
                               ldb, b_order, C, ldc, c_order, alpha, beta, ws, ws_bytes);
}

extern "C" JLB_API int jlb_csr_spmm(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                    int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                                    const void *val, int64_t k, const void *B, int64_t ldb,
                                    int b_order, void *C, int64_t ldc, int c_order, double alpha,
                                    double beta) {
    return csr_spmm(stream, dtype, idx_base, m, n, nnz, rowptr, colind, val, k, B, ldb, b_order, C,
                    ldc, c_order, alpha, beta, nullptr, 0);
}

extern "C" JLB_API size_t jlb_csr_spmm_workspace_size(int dtype, int64_t m, int64_t n, int64_t k,
                                                      int b_order, int c_order) {
    return spmm::ws_bytes_for(m, n, k, b_order, c_order, dtype == JLB_F64 ? 8 : 4);
}

extern "C" JLB_API int jlb_csr_spmm_ws(void *stream, int dtype, int idx_base, int64_t m, int64_t n,
                                       int64_t nnz, const int32_t *rowptr, const int32_t *colind,
                                       const void *val, int64_t k, const void *B, int64_t ldb,
                                       int b_order, void *C, int64_t ldc, int c_order,
                                       double alpha, double beta, void *workspace,
                                       size_t workspace_bytes) {
    return csr_spmm(stream, dtype, idx_base, m, n, nnz, rowptr, colind, val, k, B, ldb, b_order, C,
                    ldc, c_order, alpha, beta, workspace, workspace_bytes);
}
