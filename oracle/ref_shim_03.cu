// ref_shim_03.cu -- C entry points into the reference's OWN MoE host and device code.
//
// TEST INFRASTRUCTURE ONLY (the checker, never the product). Compiled by oracle/Makefile
// together with the unmodified reference source 03_moe_wq_decode.cu (which includes
// common/moe.cuh), from where it lies in the reference tree, into oracle/_ref/libref03.so.
// Exposes make_logits (common/moe.cuh:142-151), host_weight (03_moe_wq_decode.cu:336-348),
// and -- for GPU-side pinning on a box with a GPU -- the reference's pack_weights kernel
// (03_moe_wq_decode.cu:49-87), router_topk kernel (common/moe.cuh:23-72) and QuantWeights
// (03:281-333) for the same-box GPU comparison. No reference code is copied into this
// repository.

#include <cstdint>
#include <cstring>

#define main ckl_ref03_main
#include "03_moe_wq_decode.cu"
#undef main

extern "C" {

void ref03_make_logits(int T, int E, unsigned seed, int disable, float* out) {
    std::vector<float> lg = make_logits(T, E, seed, disable);
    std::memcpy(out, lg.data(), lg.size() * 4);
}

// Dequantized weights of a reference-packed tensor, through the reference's host_weight.
// P: words as written by pack_weights<bits>; Sc: its fp16 scales (bit patterns).
void ref03_host_weight_all(int bits, const uint32_t* P, size_t nwords, const uint16_t* Sc,
                           size_t nscales, int E, int d, int f, float* out) {
    std::vector<uint32_t> pv(P, P + nwords);
    std::vector<half> sv(nscales);
    std::memcpy(sv.data(), Sc, nscales * 2);
    for (int e = 0; e < E; e++)
        for (int k = 0; k < d; k++)
            for (int c = 0; c < f; c++)
                out[((size_t)e * d + k) * f + c] = host_weight(bits, pv, sv, e, k, c, d, f);
}

// Launch the reference's pack_weights<bits> on device buffers (needs a GPU).
int ref03_pack_weights_device(int bits, const void* W, void* P, void* Sc, int E, int d,
                              int f) {
    if (bits == 16) pack_weights<16><<<1024, 256>>>((const half*)W, (uint32_t*)P, (half*)Sc, E, d, f);
    else if (bits == 8) pack_weights<8><<<1024, 256>>>((const half*)W, (uint32_t*)P, (half*)Sc, E, d, f);
    else pack_weights<4><<<1024, 256>>>((const half*)W, (uint32_t*)P, (half*)Sc, E, d, f);
    cudaError_t e = cudaDeviceSynchronize();
    return e == cudaSuccess ? 0 : (int)e;
}

// Launch the reference's router_topk on device buffers (needs a GPU).
int ref03_router_topk_device(const float* logits, int* ids, float* wts, int T, int E, int k) {
    router_topk<<<ceil_div(T * 32, 256), 256>>>(logits, ids, wts, T, E, k);
    cudaError_t e = cudaDeviceSynchronize();
    return e == cudaSuccess ? 0 : (int)e;
}

// The reference's QuantWeights (03:281-333) on a caller device W (packs with its own
// pack_weights<bits>), and QuantWeights::run on caller device Xp / Yp / offsets (needs a GPU).
void* ref03_quant_make(int bits, const void* W, int E, int d, int f) {
    QuantWeights* q = new QuantWeights(bits, (const half*)W, E, d, f);
    cudaDeviceSynchronize();
    return q;
}

void ref03_quant_run(void* qw, const void* Xp, void* Yp, const int* offsets, int A, int E, int d,
                     int f, int force_ksplit, void* stream) {
    static_cast<QuantWeights*>(qw)->run((const half*)Xp, (half*)Yp, offsets, A, E, d, f,
                                        force_ksplit, (cudaStream_t)stream);
}

void ref03_quant_free(void* qw) { delete static_cast<QuantWeights*>(qw); }

}  // extern "C"
