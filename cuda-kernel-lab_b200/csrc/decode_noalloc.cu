// decode_noalloc.cu -- ckl_decode_attention for callers that cannot allocate device memory.
//
// Split-KV decode needs scratch for the per-chunk partial outputs. ckl_decode_attention
// takes that scratch from the caller, which assumes the caller can allocate. Some cannot:
// a host process whose memory pool has reserved the GPU's memory up front and hands out no
// raw device buffers, or a decode loop that must not call cudaMalloc/cudaFree because those
// calls can synchronise the device. For them this entry point uses a fixed scratch array
// compiled into the library instead (CKL_NOALLOC_SCRATCH_BYTES on every GPU that loads the
// library, held until the process exits) and runs the unchanged partial + merge kernels on
// it. No cudaMalloc, cudaFree or other allocating call is made.

#include <mutex>

#include "ckl_internal.h"

namespace ckl {
namespace {

// The scratch. In host code `g_noalloc_scratch` is only a host-side stand-in for the
// device array, never a device address: the device address is obtained per device with
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[CKL_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices];
bool g_scratch_valid[kMaxDevices];
std::mutex g_scratch_mu[kMaxDevices];

// Device address of the scratch on the current device. The lookup runs while that device is
// current and its result is kept only when it succeeds: a failed lookup (for example an
// error left behind by an earlier kernel) is retried by the next call instead of failing
// every later call on that device. The kept address belongs to the device's primary
// context; it does not survive cudaDeviceReset, after which this entry point must not be
// called again in the same process.
ckl_status scratch_on_current_device(void** out) {
    int dev = 0;
    CKL_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(CKL_CUDA_ERROR, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mu[dev]);
    if (!g_scratch_valid[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            (void)cudaGetLastError();   // do not leave the lookup's error for the next call
            return cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol,
                               "cudaGetSymbolAddress(noalloc scratch)");
        }
        g_scratch_ptr[dev] = p;
        g_scratch_valid[dev] = true;
    }
    *out = g_scratch_ptr[dev];
    return CKL_OK;
}

}  // namespace
}  // namespace ckl

using namespace ckl;

extern "C" ckl_status ckl_decode_attention_noalloc(const ckl_decode_params* p, void* out,
                                                   float* lse, void* stream) {
    if (!p) return fail(CKL_INVALID_ARG, "params is NULL");
    if (p->B > 0 && (p->chunk_base != 0 || p->part_stride != p->num_chunks))
        return fail(CKL_INVALID_ARG,
                    "decode_attention_noalloc: chunk_base must be 0 and part_stride == "
                    "num_chunks (every merged slot is written by the same call)");
    const size_t need = ckl_decode_workspace_size(p);
    if (need > (size_t)CKL_NOALLOC_SCRATCH_BYTES)
        return fail(CKL_WORKSPACE_TOO_SMALL,
                    "decode_attention_noalloc: this launch needs %zu bytes of scratch "
                    "(B*Hq*num_chunks = %lld partial rows); the built-in scratch holds %zu "
                    "bytes -- use ckl_decode_attention with a caller workspace",
                    need, (long long)p->B * p->Hq * p->num_chunks,
                    (size_t)CKL_NOALLOC_SCRATCH_BYTES);
    void* scratch = nullptr;
    if (need > 0) {
        ckl_status st = scratch_on_current_device(&scratch);
        if (st != CKL_OK) return st;
    }
    return ckl_decode_attention(p, out, lse, scratch, need > 0 ? (size_t)CKL_NOALLOC_SCRATCH_BYTES : 0,
                                stream);
}
