// api.cu -- runtime entry points of the C ABI: version, error reporting,
// device binding and the device error word.
#include "common.cuh"

#include <stdio.h>
#include <string.h>

namespace jlb {

namespace {
thread_local int t_status = JLB_OK;
thread_local char t_msg[512] = {0};
}  // namespace

int fail(int status, const char *fmt, ...) {
    t_status = status;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
    va_end(ap);
    return status;
}

int ok() {
    t_status = JLB_OK;
    t_msg[0] = 0;
    return JLB_OK;
}

int cuda_check(cudaError_t e, const char *what) {
    return fail(JLB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

}  // namespace jlb

using namespace jlb;

extern "C" JLB_API int jlb_version(void) { return 100; /* 0.1.0 */ }

extern "C" JLB_API const char *jlb_status_string(int status) {
    switch (status) {
        case JLB_OK: return "ok";
        case JLB_ERR_UNSUPPORTED_FORMAT: return "UnsupportedFormat";
        case JLB_ERR_UNSUPPORTED_INDEX_TYPE: return "UnsupportedIndexType";
        case JLB_ERR_UNSUPPORTED_VALUE_TYPE: return "UnsupportedValueType";
        case JLB_ERR_INDEX_ORIGIN_MISMATCH: return "IndexOriginMismatch";
        case JLB_ERR_DEVICE_MISMATCH: return "DeviceMismatch";
        case JLB_ERR_INCOMPATIBLE_EXTENTS: return "IncompatibleExtents";
        case JLB_ERR_NONCANONICAL_STORAGE: return "NonCanonicalStorage";
        case JLB_ERR_INVALID_ARGUMENT: return "InvalidArgument";
        case JLB_ERR_CUDA: return "CudaError";
        case JLB_ERR_DEVICE_TIMEOUT: return "DeviceTimeout";
        case JLB_ERR_WORKSPACE: return "WorkspaceTooSmall";
        default: return "UnknownStatus";
    }
}

extern "C" JLB_API int jlb_last_error(char *buf, size_t len) {
    if (buf && len > 0) {
        strncpy(buf, t_msg, len - 1);
        buf[len - 1] = 0;
    }
    return t_status;
}

extern "C" JLB_API int jlb_init(int device) {
    int count = 0;
    JLB_CUDA(cudaGetDeviceCount(&count));
    if (device < 0 || device >= count)
        return fail(JLB_ERR_DEVICE_MISMATCH, "device %d not present (%d devices)", device, count);
    JLB_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    JLB_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(JLB_ERR_DEVICE_MISMATCH,
                    "libjlust_b200 is built for sm_100a; device %d is sm_%d%d (%s)", device,
                    prop.major, prop.minor, prop.name);
    return ok();
}

extern "C" JLB_API int jlb_device_status(void *stream) {
    JLB_CUDA(cudaStreamSynchronize(as_stream(stream)));
    int bits = 0;
    const int parts[9] = {take_dev_error_spmv(), take_dev_error_spmm(), take_dev_error_sddmm(),
                          take_dev_error_bsr(), take_dev_error_convert(), take_dev_error_halo(),
                          take_dev_error_spmvfmt(), take_dev_error_bbm(),
                          take_dev_error_spgemm()};
    for (int v : parts) {
        if (v < 0) return fail(JLB_ERR_CUDA, "reading the device error word failed");
        bits |= v;
    }
    if (bits & DEV_ERR_TIMEOUT)
        return fail(JLB_ERR_DEVICE_TIMEOUT, "a bounded device wait gave up (error bits 0x%x)", bits);
    if (bits & (DEV_ERR_BOUNDS | DEV_ERR_OVERFLOW | DEV_ERR_ORDER))
        return fail(JLB_ERR_NONCANONICAL_STORAGE,
                    "a device bounds/overflow check failed (error bits 0x%x)", bits);
    return ok();
}

extern "C" JLB_API int jlb_l2_persist(void *stream, const void *base, size_t bytes,
                                      size_t *persisted_out) {
    cudaStream_t st = as_stream(stream);
    if (persisted_out) *persisted_out = 0;
    cudaStreamAttrValue v;
    memset(&v, 0, sizeof(v));
    if (bytes == 0 || base == nullptr) {
        v.accessPolicyWindow.num_bytes = 0;
        JLB_CUDA(cudaStreamSetAttribute(st, cudaStreamAttributeAccessPolicyWindow, &v));
        JLB_CUDA(cudaCtxResetPersistingL2Cache());
        JLB_CUDA(cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, 0));
        return ok();
    }
    int dev = 0, max_persist = 0, max_window = 0;
    JLB_CUDA(cudaGetDevice(&dev));
    JLB_CUDA(cudaDeviceGetAttribute(&max_persist, cudaDevAttrMaxPersistingL2CacheSize, dev));
    JLB_CUDA(cudaDeviceGetAttribute(&max_window, cudaDevAttrMaxAccessPolicyWindowSize, dev));
    if (max_persist <= 0 || max_window <= 0)
        return fail(JLB_ERR_CUDA, "device %d has no persisting L2 (set-aside %d, window %d)", dev,
                    max_persist, max_window);
    const size_t window = bytes < (size_t)max_window ? bytes : (size_t)max_window;
    const size_t setaside = window < (size_t)max_persist ? window : (size_t)max_persist;
    JLB_CUDA(cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, setaside));
    v.accessPolicyWindow.base_ptr = const_cast<void *>(base);
    v.accessPolicyWindow.num_bytes = window;
    v.accessPolicyWindow.hitRatio = (float)((double)setaside / (double)window);
    v.accessPolicyWindow.hitProp = cudaAccessPropertyPersisting;
    v.accessPolicyWindow.missProp = cudaAccessPropertyStreaming;
    JLB_CUDA(cudaStreamSetAttribute(st, cudaStreamAttributeAccessPolicyWindow, &v));
    if (persisted_out) *persisted_out = setaside;
    return ok();
}
