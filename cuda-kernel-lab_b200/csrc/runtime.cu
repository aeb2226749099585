// runtime.cu -- status/error reporting, the device-properties cache, the spin-wait
// limit, the device error word, tensor-map encoding, and the bandwidth probe.

#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>

#include "ckl_internal.h"
#include "ckl_ptx.cuh"

namespace ckl {

// Device-side error word (see DEVERR_* in ckl_ptx.cuh); kernels receive its address.
__device__ unsigned int g_device_error = 0;

namespace {
thread_local std::string t_last_error;

uint64_t initial_timeout() {
    const char* s = std::getenv("CKL_SPIN_TIMEOUT_NS");
    if (s && *s) return std::strtoull(s, nullptr, 10);
    return 1000000000ull;
}
uint64_t g_timeout_ns = initial_timeout();

constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
std::once_flag g_info_once[kMaxDevices];
}  // namespace

ckl_status fail(ckl_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return st;
}

ckl_status cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return CKL_OK;
    return fail(CKL_CUDA_ERROR, "%s: %s", what, cudaGetErrorString(e));
}

const DeviceInfo* device_info() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        cuda_status(e, "cudaGetDevice");
        return nullptr;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        fail(CKL_CUDA_ERROR, "device ordinal %d out of range", dev);
        return nullptr;
    }
    std::call_once(g_info_once[dev], [dev] {
        DeviceInfo& d = g_info[dev];
        d.device = dev;
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        cudaDeviceGetAttribute(&d.l2_bytes, cudaDevAttrL2CacheSize, dev);
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
        void* ew = nullptr;
        if (cudaGetSymbolAddress(&ew, g_device_error) == cudaSuccess)
            d.err_word = static_cast<unsigned*>(ew);
    });
    if (g_info[dev].sms <= 0 || !g_info[dev].err_word) {
        fail(CKL_CUDA_ERROR, "could not query device %d", dev);
        return nullptr;
    }
    if (g_info[dev].cc_major != 10) {
        fail(CKL_UNSUPPORTED_SHAPE, "device %d is sm_%d%d; this library is built for sm_100a only",
             dev, g_info[dev].cc_major, g_info[dev].cc_minor);
        return nullptr;
    }
    return &g_info[dev];
}

uint64_t spin_timeout_ns() { return g_timeout_ns; }

ckl_status encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* gaddr,
                        const uint64_t* dims, const uint64_t* strides_bytes,
                        const uint32_t* box, CUtensorMapSwizzle swizzle) {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    if (!fn) return fail(CKL_CUDA_ERROR, "cuTensorMapEncodeTiled entry point unavailable");
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(map, dtype, (cuuint32_t)rank, gaddr, (const cuuint64_t*)dims,
                    (const cuuint64_t*)strides_bytes, (const cuuint32_t*)box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CKL_INVALID_ARG, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CKL_OK;
}

// Achievable-bandwidth probe: every thread streams 16-byte loads and folds them into an
// XOR so the loads cannot be removed.
__global__ void stream_read_kernel(const uint4* p, size_t n, unsigned* sink) {
    unsigned acc = 0;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n; i += 4 * stride) {
        uint4 a = __ldcs(p + i), b = __ldcs(p + i + stride);
        uint4 c = __ldcs(p + i + 2 * stride), d = __ldcs(p + i + 3 * stride);
        acc ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w;
        acc ^= c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
    }
    for (; i < n; i += stride) {
        uint4 a = __ldcs(p + i);
        acc ^= a.x ^ a.y ^ a.z ^ a.w;
    }
    if (acc == 0x9e3779b9u) sink[0] = acc;
}

}  // namespace ckl

using namespace ckl;

extern "C" {

const char* ckl_last_error_string(void) { return t_last_error.c_str(); }

const char* ckl_version(void) { return "ckl-b200 0.1 (sm_100a)"; }

ckl_status ckl_check_device_error(void) {
    unsigned v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof v);
    if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyFromSymbol(g_device_error)");
    if (v) {
        e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof zero);
        if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyToSymbol(g_device_error)");
        if (v & DEVERR_TIMEOUT)
            return fail(CKL_TIMEOUT, "a kernel gave up on a bounded wait (device error 0x%x)", v);
        return fail(CKL_INVALID_ARG, "a device-side bound given by the caller was exceeded "
                    "(device error 0x%x)", v);
    }
    return CKL_OK;
}

void ckl_set_spin_timeout_ns(uint64_t ns) { g_timeout_ns = ns; }

ckl_status ckl_stream_read(const void* buf, size_t bytes, unsigned* sink, void* stream) {
    if (!buf || !sink || bytes % 16) return fail(CKL_INVALID_ARG, "stream_read: bad buffer/size");
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    stream_read_kernel<<<di->sms * 16, 256, 0, (cudaStream_t)stream>>>(
        (const uint4*)buf, bytes / 16, sink);
    CKL_CUDA_TRY(cudaGetLastError());
    return CKL_OK;
}

}  // extern "C"
