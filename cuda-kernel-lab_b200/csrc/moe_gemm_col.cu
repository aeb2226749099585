// moe_gemm_col.cu -- int4 weight-only expert GEMM on the 5th-generation tensor cores with the
// weights' A operand in tensor memory: the path of ckl_moe_expert_gemm for weights packed in
// CKL_MOE_LAYOUT_COLUMN (int4, group 128, N % 128 == 0).
//
// Replaces moe_wq_gemv / decode_word / moe_splitk_reduce of the reference
// (03_moe_wq_decode.cu:100-333) for that layout: Y[r] = X[r] . dequant(W[e]) for the rows r of
// every expert e, with SwiGLU fused for the gate/up pair.
//
// Decode gives each expert a handful of rows, so the job streams packed weights. The
// weights are the M = 128 operand (output columns; "swap-AB") and the expert's rows the
// N = 16 operand. A decode thread owns one output column: it turns its column's 64 codes of a
// half group into fp16 offset codes -- ((w >> 4j) & 0x000F000F) | 0x64006400 is
// half2(1024 + q) of two consecutive k, seven integer instructions per 8 weights -- and
// writes them straight into its tensor-memory lane with one tcgen05.st, so the decoded
// weights never pass through shared memory; tcgen05.mma reads A from tensor memory and the
// rows from a 128-byte-swizzled shared tile. Every 128-k quantisation group accumulates in
// its own tensor-memory slot next to X_g[n] = the group's activation sum of row n (one more
// MMA against an all-ones A), and the epilogue folds the group in exactly:
//     y += s * (D_g - (1024 + z) X_g)
// so the zero point and the scale cost two fp32 FMAs per group, not work per weight.
//
// A persistent wave of CTAs (one per SM) loops over work items (128-column tile of the j-th
// active expert, K slice), 16 rows per pass. Warp roles, on rings of mbarriers that run on
// from one item to the next:
//   warp 0       producer: per 128-k group, one cp.async.bulk of the tile's block per matrix
//                (8 KB of codes + scales + zero points) and each row's 256-byte k slice into
//                the packed ring (no multicast)
//   warp 1       MMA issuer (lane 0; the warp walks the items): per 64-k half group, 4 k steps
//                x (gate, up, all-ones) tcgen05.mma; commits free the A slot and publish the
//                group's accumulators
//   warps 2-9    decode, 4 per matrix (warp w owns tensor-memory lanes 32 (w % 4)..+31):
//                codes -> offset codes -> tcgen05.st into an A slot; the rows' 64-k slice
//                into the swizzled B tile (matrix 0's warps); the group's scales and zero
//                points into a parameter slot
//   warps 10-13  epilogue: tcgen05.ld of the group's slot (lane = output column), the fold
//                above in fp32 registers; at the end of a pass SwiGLU (or not) and the rows'
//                stores (fp32 partials when K is split)
// The CTA's expert is found on the device from the expert offsets, so the launch needs no
// host sync (02_moe_grouped_gemm.cu:95, 234-235). Every mbarrier wait is bounded
// (globaltimer); on a timeout the roles leave their loops, the error word records it, and
// the CTA drains its copies and MMAs before it frees tensor memory.

#include <algorithm>
#include <mutex>

#include "ckl_internal.h"
#include "ckl_ptx.cuh"
#include "moe_common.cuh"
#include "moe_internal.h"

namespace ckl {
namespace moe {
namespace col {

constexpr int BM = COL_TILE;                 // output columns per item (the MMA's M)
constexpr int BN = 16;                       // rows per pass (the MMA's N)
constexpr int HK = 64;                       // k per A slot: half a group
constexpr int DEC_WARP0 = 2;                 // warps 2..9 decode (4 per matrix)
constexpr int EPI_WARP0 = 10;                // warps 10..13
constexpr int THREADS = 14 * 32;
constexpr int SA = 3;                        // A slots (half groups) in tensor memory
constexpr int SD = 4;                        // group accumulator slots
constexpr int ACOLS = 64;                    // columns per A slot: gate +0, up +32 (64 k as half2)
constexpr int ONES_COL = SA * ACOLS;         // 8 columns of all-ones A (k 16)
constexpr int D_COL0 = 256;                  // group slot d at D_COL0 + 64 d: gate +0, up +16, X_g +32
constexpr int DCOLS = 64;
constexpr uint32_t TMEM_COLS = 512;
constexpr int XROW = KGROUP_STAGE * 2;       // bytes of one row's 128-k slice
constexpr int B_TILE = BN * HK * 2;          // 2 KB: 16 rows x 64 k, 128-byte swizzle
static_assert(ONES_COL + 8 <= D_COL0 && D_COL0 + SD * DCOLS <= (int)TMEM_COLS, "tensor memory map");

template <bool SWIGLU>
struct Cfg {
    static constexpr int MATS = SWIGLU ? 2 : 1;
    static constexpr int DEC_WARPS = 4 * MATS;                    // decode warps that work
    static constexpr int P_W = MATS * COL_BLOCK;
    static constexpr int P_SLOT = P_W + BN * XROW;
    static constexpr int SP = SWIGLU ? 8 : 12;
    static constexpr int PRM = MATS * BM * 8;                     // float2 {s, 1024 + z} per column
    static constexpr int OFF_B = 0;
    static constexpr int OFF_P = OFF_B + SA * B_TILE;
    static constexpr int OFF_PRM = OFF_P + SP * P_SLOT;
    static constexpr int OFF_BAR = OFF_PRM + SD * PRM;
    static constexpr int NBAR = 2 * SP + 2 * SA + 3 * SD + 1;
    static constexpr int SMEM = 1024 + OFF_BAR + NBAR * 8 + 16;
    static_assert(B_TILE % 1024 == 0 && OFF_P % 16 == 0 && P_SLOT % 16 == 0, "alignment");
    static_assert(SMEM <= 227 * 1024 && SMEM > 114 * 1024, "one CTA per SM (it holds all of TMEM)");
};

struct Args {
    const __half* X;          // activation rows [*, K]
    const int* row_src;       // [A] X row of each expert-sorted row (nullptr: X is sorted)
    const int* offsets;       // [E+1]
    const uint8_t* W0;        // packed weights, column layout (the GEMM, or gate for SwiGLU)
    const uint8_t* W1;        // up projection (SwiGLU)
    void* Y;                  // [A, N] fp16 (or fp32 when y_f32), or fp32 split-K partials
    const int* row_dst;       // [A] Y row of each expert-sorted row (nullptr: kept)
    unsigned* err;
    unsigned long long timeout_ns;
    int E, K, N, ksplit, A, y_f32, mtiles, dep;
};

// The j-th expert (in id order) that has rows, or -1; and the number of such experts.
// Warp-collective (full mask): every lane calls it and gets the same value.
__device__ __forceinline__ int nth_active(const int* offsets, int E, int j) {
    const int lane = threadIdx.x & 31;
    int seen = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const bool act = e < E && __ldg(offsets + e + 1) > __ldg(offsets + e);
        const unsigned m = __ballot_sync(0xffffffffu, act);
        const int c = __popc(m);
        if (seen + c > j) {
            unsigned mm = m;
            for (int r = j - seen; r > 0; r--) mm &= mm - 1;
            return e0 + __ffs(mm) - 1;
        }
        seen += c;
    }
    return -1;
}
__device__ __forceinline__ int count_active(const int* offsets, int E) {
    const int lane = threadIdx.x & 31;
    int n = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const bool act = e < E && __ldg(offsets + e + 1) > __ldg(offsets + e);
        n += __popc(__ballot_sync(0xffffffffu, act));
    }
    return n;
}

// Work item it: 128-column tile mt of the j-th active expert over K slice z (tiles fastest,
// so the CTAs of one round share an expert's rows in L2). Warp-collective.
struct Item {
    int mt, z, e, row_beg, n_e, g_beg, g_end, npass;
};
__device__ __forceinline__ Item item_of(const Args& a, int it, int n_act) {
    Item w;
    w.mt = it % a.mtiles;
    const int rest = it / a.mtiles;
    w.z = rest / n_act;
    w.e = nth_active(a.offsets, a.E, rest % n_act);
    w.row_beg = __ldg(a.offsets + w.e);
    w.n_e = __ldg(a.offsets + w.e + 1) - w.row_beg;
    const int ngroups = a.K / KGROUP_STAGE;
    const int per = (ngroups + a.ksplit - 1) / a.ksplit;
    w.g_beg = min(ngroups, w.z * per);
    w.g_end = min(ngroups, w.g_beg + per);
    w.npass = (w.n_e + BN - 1) / BN;
    return w;
}

// half2(1024 + q) of k 2j, 2j+1 (j = 0..3) of one column-layout word.
__device__ __forceinline__ void dec_word(uint32_t w, uint32_t* o) {
    asm("{\n\t.reg .b32 w4, w8, w12;\n\t"
        "shr.b32 w4, %4, 4;\n\t"
        "shr.b32 w8, %4, 8;\n\t"
        "shr.b32 w12, %4, 12;\n\t"
        "lop3.b32 %0, %4, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 %1, w4, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 %2, w8, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 %3, w12, 0x000F000F, 0x64006400, 0xEA;\n\t}"
        : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
        : "r"(w));
}

// Byte offset of 16-byte chunk c (8 k) of row r in a K-major tile with 128-byte rows and the
// 128-byte swizzle (8-row groups 1 KB apart).
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

template <bool SWIGLU>
__global__ void __launch_bounds__(THREADS, 1)
moe_gemm_col_kernel(const Args a) {
    using C = Cfg<SWIGLU>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align_ptr<1024>(smem_raw);
    uint8_t* btiles = sm + C::OFF_B;
    uint8_t* pring = sm + C::OFF_P;
    float2* prm = reinterpret_cast<float2*>(sm + C::OFF_PRM);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
    uint64_t* p_full = bars;
    uint64_t* p_empty = p_full + C::SP;
    uint64_t* a_full = p_empty + C::SP;
    uint64_t* a_empty = a_full + SA;
    uint64_t* d_full = a_empty + SA;
    uint64_t* d_empty = d_full + SD;
    uint64_t* q_full = d_empty + SD;                      // parameters of a group slot written
    uint64_t* done = q_full + SD;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (a.dep == 1) pdl_wait();                           // offsets come from the previous kernel
    const int n_act = count_active(a.offsets, a.E);
    const int n_items = a.mtiles * n_act * a.ksplit;
    if ((int)blockIdx.x >= n_items) {                     // CTA past the items
        pdl_trigger();
        return;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::SP; s++) {
            mbar_init(&p_full[s], 1);
            mbar_init(&p_empty[s], C::DEC_WARPS);
        }
        for (int s = 0; s < SA; s++) {
            mbar_init(&a_full[s], C::DEC_WARPS);
            mbar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < SD; s++) {
            mbar_init(&d_full[s], 1);
            mbar_init(&d_empty[s], 4);
            mbar_init(&q_full[s], C::DEC_WARPS);
        }
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    if (warp >= EPI_WARP0) {                              // the all-ones A (8 columns, every lane)
        const uint32_t ones[8] = {0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u,
                                  0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u};
        tmem_st8(tmem + ((uint32_t)((warp & 3) * 32) << 16) + ONES_COL, ones);
        tmem_st_wait();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint64_t deadline = globaltimer() + a.timeout_ns;
    if (a.dep != 2) pdl_trigger();

    if (warp == 0) {
        // ------------------------------------------------------------------ producer
        const uint64_t wpol = policy_evict_first();       // weights: streamed once
        const uint64_t xpol = policy_evict_last();        // rows: re-read by the other tiles
        int ok = 1, pg = 0, npre = 0;
        if (a.dep == 2) {
            // the first groups' weights do not depend on the previous kernel: stream them,
            // then wait for it before any row is read
            const Item w = item_of(a, blockIdx.x, n_act);
            npre = min(C::SP, w.g_end - w.g_beg);
            if (lane == 0)
                for (int i = 0; i < npre; i++) {
                    uint8_t* st = pring + (size_t)i * C::P_SLOT;
                    mbar_expect_tx(&p_full[i], C::P_W);
                    for (int m = 0; m < C::MATS; m++)
                        bulk_load(st + (size_t)m * COL_BLOCK,
                                  (m ? a.W1 : a.W0) + col_block_offset(a.K, a.N, w.e, w.mt, w.g_beg + i),
                                  COL_BLOCK, &p_full[i], wpol);
                }
            pdl_wait();
            pdl_trigger();
        }
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const Item w = item_of(a, it, n_act);
            for (int p = 0; p < w.npass && ok; p++) {
                const int r0 = p * BN, nr = min(BN, w.n_e - r0);
                const int src = lane < nr ? (a.row_src ? __ldg(a.row_src + w.row_beg + r0 + lane)
                                                       : w.row_beg + r0 + lane) : 0;
                const __half* xrow = a.X + (size_t)src * a.K;
                for (int g = w.g_beg; g < w.g_end; g++, pg++) {
                    const int s = pg % C::SP;
                    if (lane == 0 && pg >= C::SP)
                        ok = mbar_wait(&p_empty[s], ((pg / C::SP) - 1) & 1, deadline, a.err);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    uint8_t* st = pring + (size_t)s * C::P_SLOT;
                    if (lane == 0) {
                        if (pg < npre) {
                            mbar_arrive_expect_tx(&p_full[s], nr * XROW);
                        } else {
                            mbar_arrive_expect_tx(&p_full[s], C::P_W + nr * XROW);
                            for (int m = 0; m < C::MATS; m++)
                                bulk_load(st + (size_t)m * COL_BLOCK,
                                          (m ? a.W1 : a.W0) + col_block_offset(a.K, a.N, w.e, w.mt, g), COL_BLOCK,
                                          &p_full[s], wpol);
                        }
                    }
                    __syncwarp();
                    if (lane < nr)
                        bulk_load(st + C::P_W + lane * XROW, xrow + (size_t)g * KGROUP_STAGE, XROW, &p_full[s], xpol);
                }
            }
        }
        // every issued copy lands before the CTA exits
        if (lane == 0)
            for (int s = 0; s < C::SP && s < pg; s++) {
                const int last = s + ((pg - 1 - s) / C::SP) * C::SP;
                mbar_wait(&p_full[s], (last / C::SP) & 1, deadline, a.err);
            }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        // the whole warp walks the items (item_of is warp-collective); lane 0 waits and issues
        const uint32_t idesc = umma_idesc_f16(BM, BN, false, false);     // A, B K-major
        int ok = 1, pg = 0, hg = 0;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const Item w = item_of(a, it, n_act);
            for (int p = 0; p < w.npass && ok; p++)
                for (int g = w.g_beg; g < w.g_end && ok; g++, pg++) {
                    if (lane == 0) {
                        const int ds = pg % SD;
                        if (pg >= SD) ok = mbar_wait(&d_empty[ds], ((pg / SD) - 1) & 1, deadline, a.err);
                        tc_fence_after_sync();
                        const uint32_t d = tmem + D_COL0 + ds * DCOLS;
                        for (int h = 0; h < 2 && ok; h++, hg++) {
                            const int as = hg % SA;
                            if (!(ok = mbar_wait(&a_full[as], (hg / SA) & 1, deadline, a.err))) break;
                            tc_fence_after_sync();
                            const uint32_t bb = smem_u32(btiles + as * B_TILE);
                            const uint32_t at = tmem + as * ACOLS;
#pragma unroll
                            for (int kk = 0; kk < HK / 16; kk++) {
                                // B: K-major, 128-byte rows, 8-row groups 1 KB apart, a k step of
                                // 16 is 32 bytes inside the swizzled row; A: 8 columns per k step
                                const uint64_t bd = umma_desc_sw128(bb + kk * 32, 16, 1024);
                                const uint32_t acc = (h | kk) != 0;
#pragma unroll
                                for (int m = 0; m < C::MATS; m++)
                                    umma_f16_tmem_a(d + m * 16, at + m * 32 + kk * 8, bd, idesc, acc);
                                umma_f16_tmem_a(d + 32, tmem + ONES_COL, bd, idesc, acc);
                            }
                            umma_commit(&a_empty[as]);    // the A slot is free once these finish
                        }
                        if (ok) umma_commit(&d_full[ds]);
                    }
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                }
        }
        if (lane == 0) {
            umma_commit(done);                            // every issued MMA has finished
            mbar_wait(done, 0, deadline, a.err);
        }
        __syncwarp();
    } else if (warp < EPI_WARP0) {
        // ------------------------------------------------------------------ decode warps
        const int dw = warp - DEC_WARP0;
        const int m = dw >> 2;                            // matrix (gate, up)
        const int quarter = warp & 3;                     // tensor-memory lanes 32*quarter..+31
        const int c = quarter * 32 + lane;                // output column within the tile
        if (m < C::MATS) {
            bool ok = true;
            int pg = 0, hg = 0;
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
                const Item w = item_of(a, it, n_act);
                for (int p = 0; p < w.npass && ok; p++)
                    for (int gi = w.g_beg; gi < w.g_end; gi++, pg++) {
                        const int ps = pg % C::SP, ds = pg % SD;
                        ok = mbar_wait(&p_full[ps], (pg / C::SP) & 1, deadline, a.err);
                        if (ok && pg >= SD) ok = mbar_wait(&d_empty[ds], ((pg / SD) - 1) & 1, deadline, a.err);
                        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                        const uint8_t* st = pring + (size_t)ps * C::P_SLOT;
                        const uint8_t* blk = st + (size_t)m * COL_BLOCK;
                        {   // the group's scale and zero point of this column
                            const float sc = __half2float(reinterpret_cast<const __half*>(blk + COL_CODES)[c]);
                            const uint32_t zw = reinterpret_cast<const uint32_t*>(blk + COL_CODES + 2 * COL_TILE)[c >> 3];
                            const float z = (float)((zw >> (4 * (c & 7))) & 15u);
                            prm[((size_t)ds * C::MATS + m) * BM + c] = make_float2(sc, 1024.f + z);
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&q_full[ds]);
                        for (int h = 0; h < 2; h++, hg++) {
                            const int as = hg % SA;
                            if (hg >= SA) ok = mbar_wait(&a_empty[as], ((hg / SA) - 1) & 1, deadline, a.err);
                            if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                            // the column's 64 codes of this half: planes 0 and 1, 4 words each
                            const uint4 c0 = *reinterpret_cast<const uint4*>(blk + col_chunk_offset(h, quarter, 0, lane));
                            const uint4 c1 = *reinterpret_cast<const uint4*>(blk + col_chunk_offset(h, quarter, 1, lane));
                            uint32_t v[32];
                            dec_word(c0.x, v + 0);
                            dec_word(c0.y, v + 4);
                            dec_word(c0.z, v + 8);
                            dec_word(c0.w, v + 12);
                            dec_word(c1.x, v + 16);
                            dec_word(c1.y, v + 20);
                            dec_word(c1.z, v + 24);
                            dec_word(c1.w, v + 28);
                            tmem_st32(tmem + ((uint32_t)(quarter * 32) << 16) + as * ACOLS + m * 32, v);
                            if (m == 0) {                 // the rows' 64-k slice, swizzled
                                const int dtid = dw * 32 + lane;   // 0..127
                                const int r = dtid >> 3, ch = dtid & 7;
                                const uint4 xv = *reinterpret_cast<const uint4*>(st + C::P_W + r * XROW + h * 128 + ch * 16);
                                *reinterpret_cast<uint4*>(btiles + as * B_TILE + sw128(r, ch)) = xv;
                                fence_proxy_async_smem();     // generic stores -> the MMA's reads
                            }
                            tmem_st_wait();
                            tc_fence_before_sync();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&a_full[as]);
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&p_empty[ps]);
                        if (!ok) break;
                    }
            }
        }
    } else {
        // ------------------------------------------------------------------ epilogue warps
        const int quarter = warp & 3;                     // tensor-memory lanes 32*quarter..+31
        const int c = quarter * 32 + lane;                // output column within the tile
        bool ok = true;
        int pg = 0;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const Item w = item_of(a, it, n_act);
            const int col = w.mt * BM + c;
            for (int p = 0; p < w.npass && ok; p++) {
                float y0[BN], y1[BN];
#pragma unroll
                for (int n = 0; n < BN; n++) y0[n] = y1[n] = 0.f;
                for (int gi = w.g_beg; gi < w.g_end; gi++, pg++) {
                    const int ds = pg % SD;
                    ok = mbar_wait(&d_full[ds], (pg / SD) & 1, deadline, a.err);
                    if (ok) ok = mbar_wait(&q_full[ds], (pg / SD) & 1, deadline, a.err);
                    if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
                    tc_fence_after_sync();
                    const uint32_t ta = tmem + ((uint32_t)(quarter * 32) << 16) + D_COL0 + ds * DCOLS;
                    uint32_t dg[16], du[16], xs[16];
                    tmem_ld16(ta, dg);
                    if (SWIGLU) tmem_ld16(ta + 16, du);
                    tmem_ld16(ta + 32, xs);
                    tmem_ld_wait();
                    const float2 p0 = prm[((size_t)ds * C::MATS) * BM + c];
#pragma unroll
                    for (int n = 0; n < BN; n++)
                        y0[n] = fmaf(p0.x, fmaf(-p0.y, __uint_as_float(xs[n]), __uint_as_float(dg[n])), y0[n]);
                    if (SWIGLU) {
                        const float2 p1 = prm[((size_t)ds * C::MATS + 1) * BM + c];
#pragma unroll
                        for (int n = 0; n < BN; n++)
                            y1[n] = fmaf(p1.x, fmaf(-p1.y, __uint_as_float(xs[n]), __uint_as_float(du[n])), y1[n]);
                    }
                    tc_fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&d_empty[ds]);
                }
                if (!ok) break;
                const int r0 = w.row_beg + p * BN, nr = min(BN, w.n_e - p * BN);
#pragma unroll
                for (int n = 0; n < BN; n++) {
                    if (n >= nr) break;
                    if (a.ksplit > 1) {
                        const size_t o = (size_t)(r0 + n) * a.N + col;
                        float* P = static_cast<float*>(a.Y) + (size_t)w.z * a.A * a.N * C::MATS;
                        P[o] = y0[n];
                        if (SWIGLU) P[(size_t)a.A * a.N + o] = y1[n];
                    } else {
                        const int orow = a.row_dst ? __ldg(a.row_dst + r0 + n) : r0 + n;
                        const size_t o = (size_t)orow * a.N + col;
                        float v = y0[n];
                        if (SWIGLU) {
                            v = y0[n] / (1.f + __expf(-y0[n])) * y1[n];
                            v = __half2float(__float2half_rn(v));   // h is fp16
                        }
                        if (a.y_f32) static_cast<float*>(a.Y)[o] = v;
                        else static_cast<__half*>(a.Y)[o] = __float2half_rn(v);
                    }
                }
            }
        }
    }

    // every role is out of its loop: its copies landed (producer), its MMAs finished (issuer)
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

ckl_status setup(const DeviceInfo* di) {
    static ckl_status st[64];
    static std::once_flag once[64];
    std::call_once(once[di->device], [di] {
        cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(moe_gemm_col_kernel<true>),
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<true>::SMEM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(reinterpret_cast<const void*>(moe_gemm_col_kernel<false>),
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<false>::SMEM);
        st[di->device] = e == cudaSuccess ? CKL_OK : cuda_status(e, "column-layout moe gemm setup");
    });
    return st[di->device];
}

}  // namespace col

int col_gemm_ksplit(const DeviceInfo* di, const ckl_moe_weights* w, int A) {
    const int busy = (w->N / col::BM) * std::min(w->E, A);
    const int ngroups = w->K / KGROUP_STAGE;
    int ks = 1;
    while (ks * 2 <= ngroups / 2 && busy * ks * 2 <= di->sms) ks *= 2;
    return ks;
}

ckl_status expert_gemm_col(const void* X, const int* row_src, const int* offsets, int A,
                           const ckl_moe_weights* w0, const ckl_moe_weights* w1, void* Y, int y_f32,
                           int ks, void* workspace, int dep, const int* row_dst, cudaStream_t s) {
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    const ckl_status st = col::setup(di);
    if (st != CKL_OK) return st;
    col::Args a;
    a.X = static_cast<const __half*>(X);
    a.row_src = row_src;
    a.offsets = offsets;
    a.W0 = static_cast<const uint8_t*>(w0->packed);
    a.W1 = w1 ? static_cast<const uint8_t*>(w1->packed) : nullptr;
    a.Y = ks > 1 ? workspace : Y;
    a.row_dst = row_dst;
    a.err = di->err_word;
    a.timeout_ns = spin_timeout_ns();
    a.E = w0->E;
    a.K = w0->K;
    a.N = w0->N;
    a.ksplit = ks;
    a.A = A;
    a.y_f32 = y_f32;
    a.mtiles = w0->N / col::BM;
    a.dep = dep;
    const long long upper = (long long)a.mtiles * std::min(w0->E, A) * ks;
    const unsigned grid = (unsigned)std::min<long long>(upper, di->sms);
    void* args[] = {&a};
    const void* fn = w1 ? reinterpret_cast<const void*>(col::moe_gemm_col_kernel<true>)
                        : reinterpret_cast<const void*>(col::moe_gemm_col_kernel<false>);
    const int smem = w1 ? col::Cfg<true>::SMEM : col::Cfg<false>::SMEM;
    CKL_CUDA_TRY(launch(fn, dim3(grid), dim3(col::THREADS), smem, s, args, dep != 0));
    return CKL_OK;
}

}  // namespace moe
}  // namespace ckl
