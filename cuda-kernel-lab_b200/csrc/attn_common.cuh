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
// tile as one page box writes it: 32 rows of 128 bytes, row 2*key + half (half = cd/8, the
// 64-dim half), with the TMA 128B swizzle (chunk ^= row%8; the tile is 1024-byte aligned).
__device__ __forceinline__ uint32_t tile_off(int key, int cd) {
    const int c = cd & 7, r = 2 * key + (cd >> 3);
    return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

// Issues the two TMA loads of one page (K and V, all 128 dims) of kv head `kvh` into stage
// `st`, completing on `bar` (which must expect STAGE_BYTES). Maps of encode_page_maps.
__device__ __forceinline__ void load_page(uint8_t* st, const CUtensorMap* tmK,
                                          const CUtensorMap* tmV, int kvh, int page,
                                          uint64_t* bar, uint64_t pol) {
    tma_load_5d(st, tmK, 0, 0, kvh, 0, page, bar, pol);
    tma_load_5d(st + KV_TILE, tmV, 0, 0, kvh, 0, page, bar, pol);
}

// The K and V caches as the packed 5-D tensors [num_pages][16 tokens][Hkv][2 halves][64 dims]
// (the 128 dims split in two 128-byte rows for the swizzle), box 64x2x1x16x1: one TMA load
// brings one head's page, both halves (4 KB), where two 2 KB boxes would take twice the TMA
// operations -- and TMA operations, not bytes in flight, bound a CTA's page rate.
inline ckl_status encode_page_maps(const void* k_cache, const void* v_cache, int Hkv,
                                   int num_pages, CUtensorMap* tmK, CUtensorMap* tmV) {
    const uint64_t dims[5] = {64, 2, (uint64_t)Hkv, (uint64_t)PAGE, (uint64_t)num_pages};
    const uint64_t strides[4] = {128, (uint64_t)D * 2, (uint64_t)Hkv * D * 2,
                                 (uint64_t)PAGE * Hkv * D * 2};
    const uint32_t box[5] = {64, 2, 1, (uint32_t)PAGE, 1};
    ckl_status st = encode_tiled(tmK, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
                                 const_cast<void*>(k_cache), dims, strides, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != CKL_OK) return st;
    return encode_tiled(tmV, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<void*>(v_cache), dims,
                        strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// 4-D maps [128 dims, Hkv, 16 tokens, num_pages] over the K and V caches, box 64x1x16x1,
// 128-byte swizzle: one 64-dim half of one head's page per load (the cascade prefix kernel,
// whose tensor-core operands want each half as its own swizzled tile).
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

// One warp's online-softmax attention state for the G query heads of one kv head (rows
// 0..G-1 of an m16n8k16 tile; rows 8..15 too when G = 16). Per 16-key page:
// S = Q K^T with mma.sync (K fragments by ldmatrix from the swizzled tile, q fragments in
// registers), scores scaled into the log2 domain and masked past `kend`, an online softmax
// whose running max only moves when a score exceeds it by 2^RESCALE_THRESHOLD, and
// O += P V (V fragments by ldmatrix.trans). Lane (g = lane/4, t = lane%4) holds rows g and
// g+8, dims 8j + 2t + {0,1} of o[j].
template <int G>
struct HeadState {
    static constexpr bool HI = G > 8;   // rows 8..15 of the MMA tile carry query heads too
    float o[16][4];
    float m_lo, m_hi, l_lo, l_hi;
    uint32_t qa0[8], qa1[8], qa2[8], qa3[8];

    __device__ __forceinline__ void reset() {
#pragma unroll
        for (int j = 0; j < 16; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        m_lo = m_hi = -INFINITY;
        l_lo = l_hi = 0.f;
    }
    // q rows of this kv head: q_head0 points at row 0 (of G) of [.., 128] fp16.
    __device__ __forceinline__ void load_q(const __half* q_head0, int lane) {
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) qa0[kk] = qa1[kk] = qa2[kk] = qa3[kk] = 0u;
        if (g < G) {
            const uint32_t* qrow = reinterpret_cast<const uint32_t*>(q_head0 + (size_t)g * D);
#pragma unroll
            for (int kk = 0; kk < 8; kk++) {
                qa0[kk] = __ldg(qrow + 8 * kk + t);
                qa2[kk] = __ldg(qrow + 8 * kk + 4 + t);
            }
            if (HI) {
                const uint32_t* qhi = qrow + 8 * D / 2;
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    qa1[kk] = __ldg(qhi + 8 * kk + t);
                    qa3[kk] = __ldg(qhi + 8 * kk + 4 + t);
                }
            }
        }
    }
    // Attend the page tile at shared address kb (K; V at kb + KV_TILE) holding keys
    // [kbase, kbase + 16); keys >= kend are masked.
    __device__ __forceinline__ void page(uint32_t kb, int kbase, int kend, float scale_log2, int lane) {
        const int t = lane & 3;
        // ldmatrix lane addressing (see tile_off): K as the B operand of Q K^T, non-trans:
        // lanes 0-7 keys 0-7 / dims 16kk..+7, 8-15 keys 0-7 / +8..15, 16-31 keys 8-15.
        const int k_key = (lane & 7) + ((lane >> 4) << 3), k_hi = (lane >> 3) & 1;
        // V as the B operand of P V, transposed: lanes 0-7 keys 0-7, 8-15 keys 8-15 of dim
        // chunk 2jj, lanes 16-31 the same for chunk 2jj+1.
        const int v_key = (lane & 7) + (((lane >> 3) & 1) << 3), v_hi = lane >> 4;
        const uint32_t vb = kb + KV_TILE;

        float sc[2][4];
#pragma unroll
        for (int n = 0; n < 2; n++) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
            uint32_t b00, b01, b10, b11;
            ldmatrix_x4(kb + tile_off(k_key, 2 * kk + k_hi), b00, b01, b10, b11);
            mma_16816(sc[0], qa0[kk], qa1[kk], qa2[kk], qa3[kk], b00, b01);
            mma_16816(sc[1], qa0[kk], qa1[kk], qa2[kk], qa3[kk], b10, b11);
        }
        // mask keys past the end (only a sequence's last page is partial)
        if (kbase + PAGE > kend) {
#pragma unroll
            for (int n = 0; n < 2; n++)
#pragma unroll
                for (int c = 0; c < 4; c++)
                    if (kbase + n * 8 + 2 * t + (c & 1) >= kend) sc[n][c] = -INFINITY;
        }
#pragma unroll
        for (int n = 0; n < 2; n++)
#pragma unroll
            for (int c = 0; c < 4; c++) sc[n][c] *= scale_log2;

        float mx_lo = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
        mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
        mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
        float mx_hi = -INFINITY;
        if (HI) {
            mx_hi = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
            mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
            mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
        }
        const bool need = mx_lo > m_lo + RESCALE_THRESHOLD || (HI && mx_hi > m_hi + RESCALE_THRESHOLD);
        if (__any_sync(0xffffffffu, need)) {
            const float mn_lo = fmaxf(m_lo, mx_lo);
            const float c_lo = ex2(m_lo - mn_lo);
            m_lo = mn_lo;
            l_lo *= c_lo;
#pragma unroll
            for (int j = 0; j < 16; j++) { o[j][0] *= c_lo; o[j][1] *= c_lo; }
            if (HI) {
                const float mn_hi = fmaxf(m_hi, mx_hi);
                const float c_hi = ex2(m_hi - mn_hi);
                m_hi = mn_hi;
                l_hi *= c_hi;
#pragma unroll
                for (int j = 0; j < 16; j++) { o[j][2] *= c_hi; o[j][3] *= c_hi; }
            }
        }
        const float p00 = ex2(sc[0][0] - m_lo), p01 = ex2(sc[0][1] - m_lo);
        const float p10 = ex2(sc[1][0] - m_lo), p11 = ex2(sc[1][1] - m_lo);
        l_lo += (p00 + p01) + (p10 + p11);
        const uint32_t pa0 = pack_half2(p00, p01), pa2 = pack_half2(p10, p11);
        uint32_t pa1 = 0u, pa3 = 0u;
        if (HI) {
            const float q00 = ex2(sc[0][2] - m_hi), q01 = ex2(sc[0][3] - m_hi);
            const float q10 = ex2(sc[1][2] - m_hi), q11 = ex2(sc[1][3] - m_hi);
            l_hi += (q00 + q01) + (q10 + q11);
            pa1 = pack_half2(q00, q01);
            pa3 = pack_half2(q10, q11);
        }
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
            uint32_t v0, v1, v2, v3;
            ldmatrix_x4_trans(vb + tile_off(v_key, 2 * jj + v_hi), v0, v1, v2, v3);
            mma_16816(o[2 * jj], pa0, pa1, pa2, pa3, v0, v1);
            mma_16816(o[2 * jj + 1], pa0, pa1, pa2, pa3, v2, v3);
        }
    }
    // Sum the row sums over the four lanes of a row (after the last page).
    __device__ __forceinline__ void reduce_l() {
        l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
        l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
        if (HI) {
            l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
            l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
        }
    }
};

// decode_attention.cu host helpers
ckl_status validate(const ckl_decode_params* p, int* G);
// out_heads / head_offset place direct-mode rows (b, h) at b*out_heads + head_offset + h
// (out_heads 0 = Hq). seq_tab (device, per sequence {kv_start, chunk_base}) overrides the
// uniform p->kv_start / p->chunk_base of partial-mode launches. pdl launches the kernel early
// behind the stream's previous kernel; wait_first 1 makes it wait for that kernel before it
// reads any input, 0 only before it completes, 2 before anything but the page table and the
// first pages that are not a sequence's last (the caller vouches those are older).
ckl_status launch_partial(const ckl_decode_params* p, int G, bool direct, __half* out,
                          float* lse, float* part_o, float* part_lse, cudaStream_t stream,
                          int out_heads = 0, int head_offset = 0, bool pdl = false,
                          const int2* seq_tab = nullptr, int wait_first = 0);
// merge_states_kernel launched with PDL (seq_tab NULL: every row merges `stride` slots)
ckl_status launch_merge(const float* part_o, const float* part_lse, __half* out, float* lse,
                        int rows, int stride, int Hq, int out_heads, int head_offset,
                        const int2* seq_tab, int tail, cudaStream_t stream);
size_t part_o_bytes(const ckl_decode_params* p);

}  // namespace attn
}  // namespace ckl
