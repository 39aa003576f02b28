// spgemm.cu -- sparse x sparse product C = alpha * A * B (CSR x CSR -> CSR)
// on sm_100a, with a prepared plan for repeated products of one structure.
//
// The plan's symbolic pass follows JLUST's scatter-sort-reduce SpGEMM
// (ext/KernelAbstractionsExt/ops/spgemm.jl:1-24, 330-438): every row i of C
// gets the products A[i,j] * B[j,c] of its A entries (storage order) times
// their B row's entries (storage order); the products of a row are sorted by
// (column, product order) -- the reference sorts (row, column) keys with a
// stable sort, so equal keys keep that order -- and each run of equal
// columns becomes one entry of C.  Here the products are laid out row by row
// (a scan of the per-row product counts), so the sort is per row, with the
// bucket sorts of sort.cuh, and the plan keeps, per product in sorted order,
// the A and B entry it multiplies and, per entry of C, where its run starts.
// The numeric pass (one thread per entry of C) sums its run from zero, left
// to right, of (A value * B value) [* alpha]: the reference's products and
// alpha scaling (:376-382), summed in the sorted order instead of by atomics,
// so the result is deterministic and matches the oracle bit for bit.
#include "common.cuh"

#include <new>

namespace jlb {
JLB_DEFINE_DEV_ERROR(spgemm)
}  // namespace jlb

#include "sort.cuh"

namespace jlb {
namespace spg {

constexpr int kThreads = 256;
constexpr int kWarpsPerBlock = kThreads / kWarp;

inline unsigned grid_warps(int64_t rows) {
    const int64_t g = ceil_div(rows > 0 ? rows : 1, kWarpsPerBlock);
    return (unsigned)(g < 148 * 16 ? g : 148 * 16);
}

inline unsigned grid_items(int64_t items) {
    const int64_t g = ceil_div(items > 0 ? items : 1, kThreads);
    return (unsigned)(g < 148 * 32 ? g : 148 * 32);
}

// Products of every row of C (one warp per row): the sum of the B row lengths
// over the row's A entries, into cnt[r] (clamped) and the 64-bit total.
__global__ void __launch_bounds__(kThreads)
count_products(int64_t m, int64_t k, int64_t nnz_a, int64_t nnz_b,
               const int32_t *__restrict__ a_rp, const int32_t *__restrict__ a_ci,
               const int32_t *__restrict__ b_rp, int base, int32_t *__restrict__ cnt,
               unsigned long long *__restrict__ total) {
    const int lane = threadIdx.x % kWarp;
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t r = (int64_t)blockIdx.x * kWarpsPerBlock + threadIdx.x / kWarp; r < m; r += nwarps) {
        const int64_t lo = (int64_t)ldg(a_rp + r) - base, hi = (int64_t)ldg(a_rp + r + 1) - base;
        long long s = 0;
        if (lo < 0 || hi > nnz_a || lo > hi) {
            if (lane == 0) dev_error(DEV_ERR_BOUNDS);
        } else {
            for (int64_t p = lo + lane; p < hi; p += kWarp) {
                const int64_t j = (int64_t)ldg(a_ci + p) - base;
                if (j < 0 || j >= k) {
                    dev_error(DEV_ERR_BOUNDS);
                    continue;
                }
                const int64_t blo = (int64_t)ldg(b_rp + j) - base, bhi = (int64_t)ldg(b_rp + j + 1) - base;
                if (blo < 0 || bhi > nnz_b || blo > bhi) {
                    dev_error(DEV_ERR_BOUNDS);
                    continue;
                }
                s += bhi - blo;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) {
            cnt[r] = (int32_t)(s < INT32_MAX - 1 ? s : INT32_MAX - 1);
            atomicAdd(total, (unsigned long long)s);
        }
    }
}

// Writes row r's products at its offset (one warp per row): column of C
// (0-based), the A and B entries multiplied, and the product's own index.
__global__ void __launch_bounds__(kThreads)
expand_products(int64_t m, int64_t k, int64_t n, int64_t nnz_a, int64_t nnz_b,
                const int32_t *__restrict__ a_rp, const int32_t *__restrict__ a_ci,
                const int32_t *__restrict__ b_rp, const int32_t *__restrict__ b_ci, int base,
                const int32_t *__restrict__ off, int32_t *__restrict__ col,
                int32_t *__restrict__ a_idx, int32_t *__restrict__ b_idx,
                int32_t *__restrict__ ent) {
    const int lane = threadIdx.x % kWarp;
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t r = (int64_t)blockIdx.x * kWarpsPerBlock + threadIdx.x / kWarp; r < m; r += nwarps) {
        const int64_t lo = (int64_t)ldg(a_rp + r) - base, hi = (int64_t)ldg(a_rp + r + 1) - base;
        if (lo < 0 || hi > nnz_a || lo > hi) continue;          // reported by count_products
        const int64_t o0 = ldg(off + r), o1 = ldg(off + r + 1);
        int64_t run = 0;
        for (int64_t p = lo; p < hi; ++p) {
            const int64_t j = (int64_t)ldg(a_ci + p) - base;
            if (j < 0 || j >= k) continue;
            const int64_t blo = (int64_t)ldg(b_rp + j) - base, bhi = (int64_t)ldg(b_rp + j + 1) - base;
            if (blo < 0 || bhi > nnz_b || blo > bhi) continue;
            for (int64_t q = blo + lane; q < bhi; q += kWarp) {
                const int64_t pos = o0 + run + (q - blo);
                if (pos >= o1) {
                    dev_error(DEV_ERR_OVERFLOW);
                    continue;
                }
                const int64_t c = (int64_t)ldg(b_ci + q) - base;
                if (c < 0 || c >= n) dev_error(DEV_ERR_BOUNDS);
                col[pos] = (int32_t)c;
                a_idx[pos] = (int32_t)p;
                b_idx[pos] = (int32_t)q;
                ent[pos] = (int32_t)pos;
            }
            run += bhi - blo;
        }
    }
}

// After the per-row sorts: the first product of every run of equal columns
// gives an entry of C (one warp per row): its column (with origin) and where
// its run starts in the sorted product order.
__global__ void __launch_bounds__(kThreads)
emit_structure(int64_t m, const int32_t *__restrict__ off, const int32_t *__restrict__ ent,
               const int32_t *__restrict__ col, const int32_t *__restrict__ c_rp, int base,
               int64_t nnz_c, int32_t *__restrict__ c_ci, int32_t *__restrict__ run_start) {
    const int lane = threadIdx.x % kWarp;
    const int64_t nwarps = (int64_t)gridDim.x * kWarpsPerBlock;
    for (int64_t r = (int64_t)blockIdx.x * kWarpsPerBlock + threadIdx.x / kWarp; r < m; r += nwarps) {
        const int lo = ldg(off + r), hi = ldg(off + r + 1);
        const int64_t out = (int64_t)ldg(c_rp + r) - base, end = (int64_t)ldg(c_rp + r + 1) - base;
        int64_t run = 0;
        int32_t prev = 0;
        for (int i0 = lo; i0 < hi; i0 += kWarp) {
            const int i = i0 + lane;
            const bool in = i < hi;
            const int32_t c = in ? ldg(col + ent[i]) : 0;
            int32_t up = __shfl_up_sync(0xffffffffu, c, 1);
            if (lane == 0) up = prev;
            const bool first = in && (i == lo || c != up);
            const unsigned bal = __ballot_sync(0xffffffffu, first);
            if (first) {
                const int64_t q = out + run + __popc(bal & ((1u << lane) - 1u));
                if (q >= 0 && q < end && q < nnz_c) {
                    c_ci[q] = c + base;
                    run_start[q] = i;
                } else {
                    dev_error(DEV_ERR_OVERFLOW);
                }
            }
            run += __popc(bal);
            prev = __shfl_sync(0xffffffffu, c, kWarp - 1);
        }
    }
}

// The A and B entries of every product in sorted order; run_start[nnz_c] = P.
__global__ void __launch_bounds__(kThreads)
gather_sorted(int64_t P, int64_t nnz_c, const int32_t *__restrict__ ent,
              const int32_t *__restrict__ a_idx, const int32_t *__restrict__ b_idx,
              int32_t *__restrict__ sa, int32_t *__restrict__ sb, int32_t *__restrict__ run_start) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < P; i += stride) {
        const int32_t e = ent[i];
        if (e < 0 || e >= P) {
            dev_error(DEV_ERR_BOUNDS);
            sa[i] = 0;
            sb[i] = 0;
            continue;
        }
        sa[i] = ldg(a_idx + e);
        sb[i] = ldg(b_idx + e);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) run_start[nnz_c] = (int32_t)P;
}

// One thread per entry of C: its run summed from zero in sorted order.
template <typename T>
__global__ void __launch_bounds__(kThreads)
numeric(int64_t nnz_c, const int32_t *__restrict__ run_start, const int32_t *__restrict__ sa,
        const int32_t *__restrict__ sb, const T *__restrict__ a_val, const T *__restrict__ b_val,
        T *__restrict__ c_val, T alpha, bool scale) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < nnz_c; q += stride) {
        const int s = ldg(run_start + q), e = ldg(run_start + q + 1);
        T acc = T(0);
        for (int i = s; i < e; ++i) {
            T t = mul_rn(ldg(a_val + ldg(sa + i)), ldg(b_val + ldg(sb + i)));
            if (scale) t = mul_rn(t, alpha);
            acc = add_rn(acc, t);
        }
        c_val[q] = acc;
    }
}

// Device buffer freed on the stream when it leaves scope.
struct Buf {
    void *p = nullptr;
    cudaStream_t st;
    explicit Buf(cudaStream_t s) : st(s) {}
    ~Buf() {
        if (p) cudaFreeAsync(p, st);
    }
    int alloc(size_t bytes) {
        cudaError_t e = cudaMallocAsync(&p, bytes ? bytes : 16, st);
        return e == cudaSuccess ? JLB_OK : cuda_check(e, "cudaMallocAsync");
    }
    template <typename T>
    T *as() const { return reinterpret_cast<T *>(p); }
};

int launch_check(const char *what) {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? JLB_OK : cuda_check(e, what);
}

int take_errors(const char *what) {
    const int bits = take_dev_error_spgemm();
    if (bits < 0) return fail(JLB_ERR_CUDA, "reading the device error word failed");
    if (bits & DEV_ERR_BOUNDS)
        return fail(JLB_ERR_NONCANONICAL_STORAGE, "%s: an index outside the extents", what);
    if (bits & DEV_ERR_OVERFLOW)
        return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE,
                    "%s: a row of C has more than 16,777,216 products, the longest the sort takes",
                    what);
    return JLB_OK;
}

}  // namespace spg
}  // namespace jlb

using namespace jlb;

struct jlb_spgemm_plan_s {
    int dtype, base, device;
    int64_t m, k, n, nnz_a, nnz_b, nnz_c, products;
    int32_t *c_rp = nullptr, *c_ci = nullptr, *run_start = nullptr, *sa = nullptr, *sb = nullptr;
};

static void plan_free(jlb_spgemm_plan p) {
    if (!p) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(p->device);
    for (int32_t *b : {p->c_rp, p->c_ci, p->run_start, p->sa, p->sb})
        if (b) cudaFree(b);
    cudaSetDevice(prev);
    delete p;
}

extern "C" JLB_API int jlb_spgemm_plan_create(jlb_spgemm_plan *plan, void *stream, int dtype,
                                              int idx_base, int64_t m, int64_t k, int64_t n,
                                              int64_t nnz_a, const int32_t *a_rowptr,
                                              const int32_t *a_colind, int64_t nnz_b,
                                              const int32_t *b_rowptr, const int32_t *b_colind,
                                              int64_t *nnz_c, int64_t *products) {
    if (!plan || !nnz_c) return fail(JLB_ERR_INVALID_ARGUMENT, "null out-pointer");
    *plan = nullptr;
    if (dtype != JLB_F32 && dtype != JLB_F64)
        return fail(JLB_ERR_UNSUPPORTED_VALUE_TYPE, "SpGEMM supports Float32 and Float64");
    if (idx_base != 0 && idx_base != 1) return fail(JLB_ERR_INVALID_ARGUMENT, "idx_base must be 0 or 1");
    if (m < 0 || k < 0 || n < 0 || nnz_a < 0 || nnz_b < 0)
        return fail(JLB_ERR_INCOMPATIBLE_EXTENTS, "negative extent");
    if (m > INT32_MAX - 1 || n > INT32_MAX - 1 || nnz_a > INT32_MAX - 1 || nnz_b > INT32_MAX - 1)
        return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "extents exceed Int32");
    if (!a_rowptr || !b_rowptr || (nnz_a > 0 && !a_colind) || (nnz_b > 0 && !b_colind))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    cudaStream_t st = as_stream(stream);
    jlb_spgemm_plan p = new (std::nothrow) jlb_spgemm_plan_s;
    if (!p) return fail(JLB_ERR_CUDA, "plan allocation failed");
    p->dtype = dtype;
    p->base = idx_base;
    p->m = m;
    p->k = k;
    p->n = n;
    p->nnz_a = nnz_a;
    p->nnz_b = nnz_b;
    cudaGetDevice(&p->device);
    int r = JLB_OK;
    // --- products per row and their offsets
    spg::Buf cnt(st), off(st), total(st), scan_ws(st), col(st), aidx(st), bidx(st), ent(st),
        long_n(st), long_rows(st);
    const size_t sws = conv::scan_ws(m > 0 ? m : 1);
    if ((r = cnt.alloc(sizeof(int32_t) * (size_t)(m > 0 ? m : 1))) ||
        (r = off.alloc(sizeof(int32_t) * (size_t)(m + 1))) ||
        (r = total.alloc(sizeof(unsigned long long))) || (r = scan_ws.alloc(sws)) ||
        (r = long_n.alloc(sizeof(int32_t)))) {
        plan_free(p);
        return r;
    }
    unsigned long long tot = 0;
    if (cudaMemsetAsync(total.p, 0, sizeof(unsigned long long), st) != cudaSuccess) {
        plan_free(p);
        return fail(JLB_ERR_CUDA, "cudaMemsetAsync failed");
    }
    if (m > 0) {
        spg::count_products<<<spg::grid_warps(m), spg::kThreads, 0, st>>>(
            m, k, nnz_a, nnz_b, a_rowptr, a_colind, b_rowptr, idx_base, cnt.as<int32_t>(),
            total.as<unsigned long long>());
        if ((r = spg::launch_check("count_products"))) {
            plan_free(p);
            return r;
        }
    }
    if (cudaMemcpyAsync(&tot, total.p, sizeof(tot), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
        plan_free(p);
        return fail(JLB_ERR_CUDA, "reading the product count failed");
    }
    if ((r = spg::take_errors("SpGEMM"))) {
        plan_free(p);
        return r;
    }
    if (tot > (unsigned long long)(INT32_MAX - 1)) {
        plan_free(p);
        return fail(JLB_ERR_UNSUPPORTED_INDEX_TYPE, "A*B has %llu products, more than Int32 positions",
                    tot);
    }
    const int64_t P = (int64_t)tot;
    p->products = P;
    if ((r = conv::scan(st, m, cnt.as<int32_t>(), off.as<int32_t>(), 0, scan_ws.p, sws))) {
        plan_free(p);
        return r;
    }
    // --- products, sorted per row
    const int64_t long_cap = P / (seg::kWarpKeys + 1) + 1;
    if ((r = col.alloc(sizeof(int32_t) * (size_t)P)) || (r = aidx.alloc(sizeof(int32_t) * (size_t)P)) ||
        (r = bidx.alloc(sizeof(int32_t) * (size_t)P)) || (r = ent.alloc(sizeof(int32_t) * (size_t)P)) ||
        (r = long_rows.alloc(sizeof(int32_t) * (size_t)long_cap))) {
        plan_free(p);
        return r;
    }
    if (cudaMalloc((void **)&p->c_rp, sizeof(int32_t) * (size_t)(m + 1)) != cudaSuccess) {
        plan_free(p);
        return fail(JLB_ERR_CUDA, "device allocation of the row pointer failed");
    }
    if (cudaMemsetAsync(long_n.p, 0, sizeof(int32_t), st) != cudaSuccess) {
        plan_free(p);
        return fail(JLB_ERR_CUDA, "cudaMemsetAsync failed");
    }
    if (m > 0) {
        spg::expand_products<<<spg::grid_warps(m), spg::kThreads, 0, st>>>(
            m, k, n, nnz_a, nnz_b, a_rowptr, a_colind, b_rowptr, b_colind, idx_base,
            off.as<int32_t>(), col.as<int32_t>(), aidx.as<int32_t>(), bidx.as<int32_t>(),
            ent.as<int32_t>());
        const int64_t g = ceil_div(m, seg::kSortThreads / kWarp);
        seg::sort_short_rows<<<(unsigned)(g < 148 * 16 ? g : 148 * 16), seg::kSortThreads, 0, st>>>(
            m, off.as<int32_t>(), ent.as<int32_t>(), col.as<int32_t>(), 0, p->c_rp + 1,
            long_rows.as<int32_t>(), long_n.as<int32_t>(), long_cap);
        const int smem = seg::kCtaKeys * (int)sizeof(uint64_t);
        cudaFuncSetAttribute(seg::sort_long_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        seg::sort_long_rows<<<148, seg::kLongThreads, smem, st>>>(
            off.as<int32_t>(), ent.as<int32_t>(), col.as<int32_t>(), 0, p->c_rp + 1,
            long_rows.as<int32_t>(), long_n.as<int32_t>(), long_cap);
        if ((r = spg::launch_check("SpGEMM symbolic pass"))) {
            plan_free(p);
            return r;
        }
    }
    // --- structure of C
    {
        spg::Buf cws(st);
        if ((r = cws.alloc(sws)) ||
            (r = conv::scan(st, m, p->c_rp + 1, p->c_rp, idx_base, cws.p, sws))) {
            plan_free(p);
            return r;
        }
    }
    int32_t last = 0;
    if (cudaMemcpyAsync(&last, p->c_rp + m, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess) {
        plan_free(p);
        return fail(JLB_ERR_CUDA, "reading nnz(C) failed");
    }
    if ((r = spg::take_errors("SpGEMM"))) {
        plan_free(p);
        return r;
    }
    p->nnz_c = (int64_t)last - idx_base;
    if (cudaMalloc((void **)&p->c_ci, sizeof(int32_t) * (size_t)(p->nnz_c > 0 ? p->nnz_c : 1)) != cudaSuccess ||
        cudaMalloc((void **)&p->run_start, sizeof(int32_t) * (size_t)(p->nnz_c + 1)) != cudaSuccess ||
        cudaMalloc((void **)&p->sa, sizeof(int32_t) * (size_t)(P > 0 ? P : 1)) != cudaSuccess ||
        cudaMalloc((void **)&p->sb, sizeof(int32_t) * (size_t)(P > 0 ? P : 1)) != cudaSuccess) {
        plan_free(p);
        return fail(JLB_ERR_CUDA, "device allocation of the plan failed");
    }
    if (m > 0) {
        spg::emit_structure<<<spg::grid_warps(m), spg::kThreads, 0, st>>>(
            m, off.as<int32_t>(), ent.as<int32_t>(), col.as<int32_t>(), p->c_rp, idx_base,
            p->nnz_c, p->c_ci, p->run_start);
    }
    spg::gather_sorted<<<spg::grid_items(P), spg::kThreads, 0, st>>>(
        P, p->nnz_c, ent.as<int32_t>(), aidx.as<int32_t>(), bidx.as<int32_t>(), p->sa, p->sb,
        p->run_start);
    if ((r = spg::launch_check("SpGEMM structure pass"))) {
        plan_free(p);
        return r;
    }
    if (cudaStreamSynchronize(st) != cudaSuccess) {
        plan_free(p);
        return fail(JLB_ERR_CUDA, "SpGEMM symbolic pass failed");
    }
    if ((r = spg::take_errors("SpGEMM"))) {
        plan_free(p);
        return r;
    }
    *nnz_c = p->nnz_c;
    if (products) *products = P;
    *plan = p;
    return ok();
}

extern "C" JLB_API int jlb_spgemm_plan_structure(jlb_spgemm_plan p, void *stream, int32_t *c_rowptr,
                                                 int32_t *c_colind) {
    if (!p) return fail(JLB_ERR_INVALID_ARGUMENT, "null plan");
    if (!c_rowptr || (p->nnz_c > 0 && !c_colind)) return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    cudaStream_t st = as_stream(stream);
    JLB_CUDA(cudaMemcpyAsync(c_rowptr, p->c_rp, sizeof(int32_t) * (size_t)(p->m + 1),
                             cudaMemcpyDeviceToDevice, st));
    if (p->nnz_c > 0)
        JLB_CUDA(cudaMemcpyAsync(c_colind, p->c_ci, sizeof(int32_t) * (size_t)p->nnz_c,
                                 cudaMemcpyDeviceToDevice, st));
    return ok();
}

extern "C" JLB_API int jlb_spgemm_plan_execute(jlb_spgemm_plan p, void *stream, const void *a_val,
                                               const void *b_val, void *c_val, double alpha) {
    if (!p) return fail(JLB_ERR_INVALID_ARGUMENT, "null plan");
    if ((p->nnz_a > 0 && !a_val) || (p->nnz_b > 0 && !b_val) || (p->nnz_c > 0 && !c_val))
        return fail(JLB_ERR_INVALID_ARGUMENT, "null buffer");
    if (p->nnz_c == 0) return ok();
    cudaStream_t st = as_stream(stream);
    const unsigned g = spg::grid_items(p->nnz_c);
    if (p->dtype == JLB_F64)
        spg::numeric<double><<<g, spg::kThreads, 0, st>>>(
            p->nnz_c, p->run_start, p->sa, p->sb, (const double *)a_val, (const double *)b_val,
            (double *)c_val, alpha, alpha != 1.0);
    else
        spg::numeric<float><<<g, spg::kThreads, 0, st>>>(
            p->nnz_c, p->run_start, p->sa, p->sb, (const float *)a_val, (const float *)b_val,
            (float *)c_val, (float)alpha, (float)alpha != 1.0f);
    JLB_LAUNCH_CHECK("spgemm numeric");
    return ok();
}

extern "C" JLB_API int jlb_spgemm_plan_destroy(jlb_spgemm_plan p) {
    plan_free(p);
    return ok();
}
