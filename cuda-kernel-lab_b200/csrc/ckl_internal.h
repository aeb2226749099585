// ckl_internal.h -- host-side helpers shared by the library's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>

#include "../../include/ckl.h"

namespace ckl {

// Records a formatted message as this thread's last error and returns `st`.
ckl_status fail(ckl_status st, const char* fmt, ...);
// Maps a CUDA runtime error (if any) to CKL_CUDA_ERROR with context.
ckl_status cuda_status(cudaError_t e, const char* what);
#define CKL_CUDA_TRY(call)                                              \
    do {                                                                \
        cudaError_t e_ = (call);                                        \
        if (e_ != cudaSuccess) return ::ckl::cuda_status(e_, #call);    \
    } while (0)

// Immutable per-device properties, queried once per device.
struct DeviceInfo {
    int device = 0;
    int sms = 0;
    int smem_optin = 0;   // max dynamic shared memory per block (opt-in)
    int l2_bytes = 0;
    int cc_major = 0, cc_minor = 0;
    unsigned* err_word = nullptr;   // device address of the device-side error word
};
const DeviceInfo* device_info();   // current device; nullptr (with error set) on failure

// Spin-wait limit passed to every kernel that waits on a barrier.
uint64_t spin_timeout_ns();

// Encodes a tiled tensor map through the driver entry point (no libcuda link needed).
ckl_status encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* gaddr,
                        const uint64_t* dims, const uint64_t* strides_bytes,
                        const uint32_t* box, CUtensorMapSwizzle swizzle);

// Launches `fn` on `stream`; with pdl = true the launch may begin while the previous kernel
// on the stream is still running (programmatic dependent launch): the kernel must call
// pdl_wait() before it reads anything that kernel writes.
inline cudaError_t launch(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          void** args, bool pdl) {
    if (!pdl) return cudaLaunchKernel(fn, grid, block, args, smem, stream);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace ckl
