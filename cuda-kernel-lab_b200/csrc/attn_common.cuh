// attn_common.cuh -- pieces shared by the decode and cascade attention kernels: the page
// tile layout in shared memory, the KV-cache TMA descriptors, softmax constants, and the
// host-side helpers of decode_attention.cu that cascade.cu reuses.
#pragma once

#include "ckl_internal.h"
#include "ckl_ptx.cuh"

namespace ckl {
namespace attn {

constexpr int D = CKL_HEAD_DIM;
constexpr int PAGE = CKL_PAGE_SIZE;
constexpr int HALF_TILE = PAGE * 64 * 2;  // 16 keys x 64 dims fp16 = 2 KB, 128B-swizzled
constexpr int KV_TILE = 2 * HALF_TILE;    // one page of K (or V) for one head: 4 KB
constexpr int STAGE_BYTES = 2 * KV_TILE;  // K + V of one page
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr float RESCALE_THRESHOLD = 8.f;   // log2 units: p may grow to 2^8 before a rescale

// Byte offset of 16-byte chunk `cd` (0..15, dims 8cd..8cd+7) of key `key` inside a page
// tile: [half = cd/8][key][64 dims] with the TMA 128B swizzle (chunk ^= key%8 within each
// 128-byte row; the tile is 1024-byte aligned).
__device__ __forceinline__ uint32_t tile_off(int key, int cd) {
    const int c = cd & 7;
    return (uint32_t)((cd >> 3) * HALF_TILE + key * 128 + ((c ^ (key & 7)) << 4));
}

// Issues the four TMA loads of one page (K and V, dims 0-63 and 64-127) of kv head `kvh`
// into stage `st`, completing on `bar` (which must expect STAGE_BYTES).
__device__ __forceinline__ void load_page(uint8_t* st, const CUtensorMap* tmK,
                                          const CUtensorMap* tmV, int kvh, int page,
                                          uint64_t* bar, uint64_t pol) {
    tma_load_4d(st, tmK, 0, kvh, 0, page, bar, pol);
    tma_load_4d(st + HALF_TILE, tmK, 64, kvh, 0, page, bar, pol);
    tma_load_4d(st + KV_TILE, tmV, 0, kvh, 0, page, bar, pol);
    tma_load_4d(st + KV_TILE + HALF_TILE, tmV, 64, kvh, 0, page, bar, pol);
}

// 4-D maps [128 dims, Hkv, 16 tokens, num_pages] over the K and V caches, box 64x1x16x1,
// 128-byte swizzle.
inline ckl_status encode_kv_maps(const void* k_cache, const void* v_cache, int Hkv,
                                 int num_pages, CUtensorMap* tmK, CUtensorMap* tmV) {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)Hkv, (uint64_t)PAGE, (uint64_t)num_pages};
    const uint64_t strides[3] = {(uint64_t)D * 2, (uint64_t)Hkv * D * 2,
                                 (uint64_t)PAGE * Hkv * D * 2};
    const uint32_t box[4] = {64, 1, (uint32_t)PAGE, 1};
    ckl_status st = encode_tiled(tmK, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                                 const_cast<void*>(k_cache), dims, strides, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != CKL_OK) return st;
    return encode_tiled(tmV, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(v_cache),
                        dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// decode_attention.cu host helpers
ckl_status validate(const ckl_decode_params* p, int* G);
// out_heads / head_offset place direct-mode rows (b, h) at b*out_heads + head_offset + h
// (out_heads 0 = Hq).
ckl_status launch_partial(const ckl_decode_params* p, int G, bool direct, __half* out,
                          float* lse, float* part_o, float* part_lse, cudaStream_t stream,
                          int out_heads = 0, int head_offset = 0);
size_t part_o_bytes(const ckl_decode_params* p);

}  // namespace attn
}  // namespace ckl
