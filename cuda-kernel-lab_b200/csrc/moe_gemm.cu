// moe_gemm.cu -- weight-only quantised expert GEMM for MoE decode on sm_100a.
//
// Replaces pack_weights / decode_word / gemv_pass / moe_wq_gemv / moe_splitk_reduce /
// QuantWeights of the reference (03_moe_wq_decode.cu:36-333).
//
// Decode gives each expert a handful of rows (tokens), so the expert GEMM streams weights.
// The reference runs it on CUDA cores (fp32 FMA per weight per row); on B200 that is
// compute-bound from ~4 rows per expert. Here the dequantised weights are the A operand of
// mma.sync.m16n8k16 (16 output columns x 16 k, "swap-AB") and up to 8 tokens per MMA are
// the B operand: a warp decodes 8 int4 weights with 9 instructions (fp16 magic number,
// exact (q - z); the fp16 group scale is applied to an fp32 group accumulator) and issues
// one MMA per 8 tokens, accumulating in fp32.
//
// A CTA owns one 64-column quad of one expert (over one K slice): warp 8 is a producer that,
// per stage of two 128-wide k groups, issues one cp.async.bulk of the quad's 4 contiguous
// records (codes + embedded scales/zeros) per group and matrix (two matrices for SwiGLU:
// gate and up) and one copy of each token row's k slice, into a multi-stage shared-memory
// ring with full/empty mbarriers (no multicast). Warps 0-7 consume: warp w computes the
// 16-column tile w % 4 on group w / 4 of the stage, and the two warps of a tile add their
// sums through shared memory at the end of a pass. The CTA's expert is the j-th expert with
// rows, found on the device from the expert offsets, so the launch needs no host sync: the
// grid is an upper bound (min(E, A) expert slots) and surplus CTAs exit
// (02_moe_grouped_gemm.cu:95, 234-235).

#include <algorithm>
#include <mutex>

#include "ckl_internal.h"
#include "ckl_ptx.cuh"
#include "moe_common.cuh"
#include "moe_internal.h"

namespace ckl {
namespace moe {

constexpr int TILES = 4;                     // 16-column tiles per CTA (a 64-column quad)
constexpr int GPS = 2;                       // 128-k groups per pipeline stage
constexpr int CONSUMERS = TILES * GPS;       // warp w: tile w % 4, group (w / 4) of the stage
constexpr int GTHREADS = (CONSUMERS + 1) * 32;
// Shared-memory ring per CTA at OCC resident CTAs per SM: 2 (deep ring, for grids of at most
// one wave) or 3 (more warps to hide latency, for larger grids).
constexpr int ring_bytes(int occ) { return occ == 3 ? 64 * 1024 : 96 * 1024; }
constexpr int XSTRIDE = GPS * 256 + 64;      // smem bytes per staged token row (pad: the two
                                             // rows a quarter-warp reads land on disjoint banks)
constexpr int MAX_STAGES = 16;
constexpr int TMAX = 2;                      // token tiles (8 rows each) per pass, at most

// int4 fragment decode to (q - z) in fp16, exact: z of column g (zc0 = half2(1024+z)) and
// of column g+8 (zc1n = -half2(64+z)); nibble order in moe_common.cuh. 9 instructions on
// 32-bit registers: (w & 0x000F000F) | 0x6400_6400 is half2(1024 + q) for nibbles 0 and 4,
// (w & 0x00F000F0) | 0x6400_6400 is half2(1024 + 16 q) for nibbles 1 and 5 (scaled back by
// 1/16 = 0x2C00 in the fma), and the same on w >> 8 for nibbles 2, 6 and 3, 7.
__device__ __forceinline__ void dec4(uint32_t w, uint32_t zc0, uint32_t zc1n, uint32_t (&a)[4]) {
    asm("{\n\t.reg .b32 t0, t1, t2, t3, w8;\n\t"
        "shr.b32 w8, %4, 8;\n\t"
        "lop3.b32 t0, %4, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 t1, %4, 0x00F000F0, 0x64006400, 0xEA;\n\t"
        "lop3.b32 t2, w8, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 t3, w8, 0x00F000F0, 0x64006400, 0xEA;\n\t"
        "sub.rn.f16x2 %0, t0, %5;\n\t"
        "fma.rn.f16x2 %1, t1, %7, %6;\n\t"
        "sub.rn.f16x2 %2, t2, %5;\n\t"
        "fma.rn.f16x2 %3, t3, %7, %6;\n\t}"
        : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
        : "r"(w), "r"(zc0), "r"(zc1n), "r"(0x2C002C00u));
}
// int8 fragment decode: offset-binary q + 128 -> q exactly ((w & 0x00FF00FF) | 0x6400_6400
// is half2(1024 + q + 128); subtract half2(1152) = 0x6480).
__device__ __forceinline__ void dec8(uint32_t w0, uint32_t w1, uint32_t (&a)[4]) {
    asm("{\n\t.reg .b32 t0, t1, t2, t3, u0, u1;\n\t"
        "shr.b32 u0, %4, 8;\n\t"
        "shr.b32 u1, %5, 8;\n\t"
        "lop3.b32 t0, %4, 0x00FF00FF, 0x64006400, 0xEA;\n\t"
        "lop3.b32 t1, u0, 0x00FF00FF, 0x64006400, 0xEA;\n\t"
        "lop3.b32 t2, %5, 0x00FF00FF, 0x64006400, 0xEA;\n\t"
        "lop3.b32 t3, u1, 0x00FF00FF, 0x64006400, 0xEA;\n\t"
        "sub.rn.f16x2 %0, t0, %6;\n\t"
        "sub.rn.f16x2 %1, t1, %6;\n\t"
        "sub.rn.f16x2 %2, t2, %6;\n\t"
        "sub.rn.f16x2 %3, t3, %6;\n\t}"
        : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
        : "r"(w0), "r"(w1), "r"(0x64806480u));
}

struct GemmArgs {
    const __half* X;          // activation rows [*, K]
    const int* row_src;       // [A] X row of each permuted row (nullptr: X is permuted)
    const int* offsets;       // [E+1] rows of expert e are [offsets[e], offsets[e+1])
    const uint8_t* W0;        // packed weights (the GEMM, or gate for SwiGLU)
    const __half* S0;         // per-channel scales [E][N] (int8 group = K only)
    const uint8_t* W1;        // up projection (SwiGLU)
    const __half* S1;
    void* Y;                  // [A, N] fp16 (or fp32 when y_f32), or fp32 split-K partials
    const int* row_dst;       // [A] Y row of each permuted row (nullptr: row order kept)
    unsigned* err;
    unsigned long long timeout_ns;
    int E, K, N, ksplit, A, y_f32;
    // 0: normal launch. 1: launched dependent on the previous kernel, which produced the
    // offsets: wait before anything. 2: dependent on a kernel that produced only X (the
    // offsets are older): prefetch the first weight stages, then wait before the X rows.
    int dep;
};

// The j-th expert (in id order) that has rows, or -1; its rows [row_beg, row_beg + n_e) come
// from the offsets the search already loaded. Every lane returns the same values.
__device__ __forceinline__ int nth_active_expert(const int* offsets, int E, int j, int& row_beg,
                                                 int& n_e) {
    const int lane = threadIdx.x & 31;
    int seen = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const int lo = e < E ? __ldg(offsets + e) : 0, hi = e < E ? __ldg(offsets + e + 1) : 0;
        const unsigned m = __ballot_sync(0xffffffffu, hi > lo);
        const int c = __popc(m);
        if (seen + c > j) {
            unsigned mm = m;
            for (int r = j - seen; r > 0; r--) mm &= mm - 1;
            const int src = __ffs(mm) - 1;
            row_beg = __shfl_sync(0xffffffffu, lo, src);
            n_e = __shfl_sync(0xffffffffu, hi, src) - row_beg;
            return e0 + src;
        }
        seen += c;
    }
    row_beg = n_e = 0;
    return -1;
}

// TM: token tiles per pass (2, or 1 when no expert can have more than 16 rows: the lighter
// kernel keeps its registers and runs ~5 % faster there).
template <int BITS, bool SWIGLU, bool GROUPED, int OCC, int TM = TMAX>
struct Cfg {
    static constexpr int MATS = SWIGLU ? 2 : 1;
    static constexpr bool EMBED = embeds_params(BITS, GROUPED ? KGROUP_STAGE : 0);
    static constexpr int CODE = group_code_bytes(BITS);
    static constexpr int REC = CODE + (EMBED ? PARAM_BYTES : 0);
    static constexpr int GBLK = TILES * REC;                       // one group of one matrix
    static constexpr int WBYTES = MATS * GPS * GBLK;               // weights per stage
    static constexpr int XROWS = TM * 8;
    static constexpr int RING = ring_bytes(OCC);
    // Ring layout whose stages hold the weights and XT 8-row token tiles: a CTA whose expert
    // has at most 8 rows takes XT = 1, the deeper ring of smaller stages.
    template <int XT>
    struct Ring {
        static constexpr int SB = (WBYTES + XT * 8 * XSTRIDE + 127) / 128 * 128;
        static constexpr int N = RING / SB > MAX_STAGES ? MAX_STAGES : RING / SB;
        static_assert(N >= 1, "ring too small for one stage");
    };
    static constexpr int RVALS = TM * 4 * MATS;                    // fp32 values per lane
    static constexpr int RED = TILES * 32 * RVALS * 4;              // cross-warp reduction
    static constexpr int SMEM = 128 + RING + RED + 2 * MAX_STAGES * 8;
};

// Consumer pass over all stages for `NT` token tiles; returns false on a timeout.
template <int BITS, bool SWIGLU, bool GROUPED, int OCC, int NT, int TM, int XT>
__device__ __forceinline__ bool consume_pass(const GemmArgs& a, const uint8_t* ring, uint64_t* full,
                                             uint64_t* empty, int& seq, int nst, int g_beg,
                                             int g_end, uint64_t deadline,
                                             float (&acc0)[TM][4], float (&acc1)[TM][4]) {
    using C = Cfg<BITS, SWIGLU, GROUPED, OCC, TM>;
    using R = typename C::template Ring<XT>;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int tile = warp % TILES, half = warp / TILES;
    constexpr int SPC = 16 / bytes_per_lane(BITS);         // k16 steps per 16-byte lane chunk
    for (int si = 0; si < nst; si++, seq++) {
        const int s = seq % R::N;
        const bool got = mbar_wait(&full[s], (seq / R::N) & 1, deadline, a.err);
        if (!__all_sync(0xffffffffu, got)) return false;
        const int grp = g_beg + si * GPS + half;
        if (grp < g_end) {
            const uint8_t* st = ring + (size_t)s * R::SB;
            const uint8_t* rec0 = st + half * C::GBLK + tile * C::REC;
            const uint8_t* rec1 = rec0 + GPS * C::GBLK;
            const uint8_t* xs = st + C::WBYTES + (size_t)g * XSTRIDE + half * 256 + 16 * t;
            uint32_t zc0[2] = {0x64086408u, 0x64086408u}, zc1[2] = {0xD480D480u, 0xD480D480u};
            float s_lo[2] = {1.f, 1.f}, s_hi[2] = {1.f, 1.f};
            if (C::EMBED) {
#pragma unroll
                for (int m = 0; m < C::MATS; m++) {
                    const uint8_t* rec = m ? rec1 : rec0;
                    const __half* scp = reinterpret_cast<const __half*>(rec + C::CODE);
                    s_lo[m] = __half2float(scp[g]);
                    s_hi[m] = __half2float(scp[g + 8]);
                    if (BITS == 4) {
                        const uint2 zw = *reinterpret_cast<const uint2*>(rec + C::CODE + 32);
                        const uint32_t z_lo = (zw.x >> (4 * g)) & 15, z_hi = (zw.y >> (4 * g)) & 15;
                        zc0[m] = (0x6400u + z_lo) * 0x10001u;             // half2(1024 + z)
                        zc1[m] = (0xD400u + 16u * z_hi) * 0x10001u;       // half2(-(64 + z))
                    }
                }
            }
            // per-group parameters: accumulate the group apart and scale it; per-channel
            // scales (applied in the epilogue) or none: accumulate into the pass directly
            float gacc0[NT][4], gacc1[NT][4];
#pragma unroll
            for (int i = 0; i < NT; i++)
#pragma unroll
                for (int c = 0; c < 4; c++)
                    if (C::EMBED) gacc0[i][c] = gacc1[i][c] = 0.f;
#pragma unroll
            for (int kb = 0; kb < 4; kb++) {          // 32-wide k blocks of the group
                uint4 xv[NT];
#pragma unroll
                for (int i = 0; i < NT; i++)
                    xv[i] = *reinterpret_cast<const uint4*>(xs + (size_t)i * 8 * XSTRIDE + kb * 64);
#pragma unroll
                for (int hb = 0; hb < 2; hb++) {      // the two k16 steps of the block
                    const int ks = kb * 2 + hb;
                    // one conflict-free 16-byte load per lane chunk
                    const int co = ((ks / SPC) * 32 + lane) * 16;
                    const uint4 c0 = *reinterpret_cast<const uint4*>(rec0 + co);
                    uint4 c1 = c0;
                    if (SWIGLU) c1 = *reinterpret_cast<const uint4*>(rec1 + co);
                    const uint32_t* q0 = reinterpret_cast<const uint32_t*>(&c0);
                    const uint32_t* q1 = reinterpret_cast<const uint32_t*>(&c1);
                    uint32_t w0[4], w1[4];
                    if (BITS == 4) {
                        dec4(q0[ks % 4], zc0[0], zc1[0], w0);
                        if (SWIGLU) dec4(q1[ks % 4], zc0[1], zc1[1], w1);
                    } else if (BITS == 8) {
                        dec8(q0[2 * (ks % 2)], q0[2 * (ks % 2) + 1], w0);
                        if (SWIGLU) dec8(q1[2 * (ks % 2)], q1[2 * (ks % 2) + 1], w1);
                    } else {
                        w0[0] = c0.x; w0[1] = c0.y; w0[2] = c0.z; w0[3] = c0.w;
                        if (SWIGLU) { w1[0] = c1.x; w1[1] = c1.y; w1[2] = c1.z; w1[3] = c1.w; }
                    }
#pragma unroll
                    for (int i = 0; i < NT; i++) {
                        const uint32_t b0 = hb ? xv[i].z : xv[i].x, b1 = hb ? xv[i].w : xv[i].y;
                        mma_16816(C::EMBED ? gacc0[i] : acc0[i], w0[0], w0[1], w0[2], w0[3], b0, b1);
                        if (SWIGLU)
                            mma_16816(C::EMBED ? gacc1[i] : acc1[i], w1[0], w1[1], w1[2], w1[3], b0, b1);
                    }
                }
            }
            // group scale onto the fp32 accumulators (exact dequantisation up to fp32 rounding)
#pragma unroll
            for (int i = 0; i < NT; i++) {
                if (!C::EMBED) break;
                acc0[i][0] += s_lo[0] * gacc0[i][0]; acc0[i][1] += s_lo[0] * gacc0[i][1];
                acc0[i][2] += s_hi[0] * gacc0[i][2]; acc0[i][3] += s_hi[0] * gacc0[i][3];
                if (SWIGLU) {
                    acc1[i][0] += s_lo[1] * gacc1[i][0]; acc1[i][1] += s_lo[1] * gacc1[i][1];
                    acc1[i][2] += s_hi[1] * gacc1[i][2]; acc1[i][3] += s_hi[1] * gacc1[i][3];
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    return true;
}

__device__ __forceinline__ void consumer_bar() {
    asm volatile("bar.sync 1, %0;" ::"n"(CONSUMERS * 32) : "memory");
}
// The same barrier returning the AND of pred over the consumer warps, so that a bounded wait
// that gave up in one warp sends every consumer warp out together (none is left at a barrier).
__device__ __forceinline__ bool consumer_bar_and(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "n"(CONSUMERS * 32)
        : "memory");
    return r != 0;
}

// The CTA's work once its expert is known: the producer warp streams the ring, warps 0-7
// consume it. XT: 8-row token tiles a stage holds (the ring layout Cfg::Ring<XT>).
template <int BITS, bool SWIGLU, bool GROUPED, int OCC, int TM, int XT>
__device__ __forceinline__ void gemm_body(const GemmArgs& a, uint8_t* ring, float* red,
                                          uint64_t* full, uint64_t* empty, int e, int row_beg,
                                          int n_e) {
    using C = Cfg<BITS, SWIGLU, GROUPED, OCC, TM>;
    using R = typename C::template Ring<XT>;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quad = blockIdx.x;
    const int ngroups = a.K / KGROUP_STAGE;
    const int per = (ngroups + a.ksplit - 1) / a.ksplit;
    const int g_beg = min(ngroups, (int)blockIdx.z * per), g_end = min(ngroups, g_beg + per);
    const int nst = (g_end - g_beg + GPS - 1) / GPS;     // stages per pass
    const int npass = (n_e + C::XROWS - 1) / C::XROWS;
    const uint64_t deadline = globaltimer() + a.timeout_ns;
    if (a.dep != 2) pdl_trigger();

    if (warp == CONSUMERS) {
        // ---------------------------------------------------------------- producer warp
        const uint64_t wpol = policy_evict_first();       // weights: streamed once
        const uint64_t xpol = policy_evict_last();        // token rows: re-read by other CTAs
        const int lgroup = C::EMBED ? KGROUP_STAGE : a.K;
        const uint8_t* w0 = a.W0 + block_offset(BITS, lgroup, a.K, a.N, e, quad, 0);
        const uint8_t* w1 = SWIGLU ? a.W1 + block_offset(BITS, lgroup, a.K, a.N, e, quad, 0) : nullptr;
        // dep 2: the weights of the first stages do not depend on the previous kernel --
        // start streaming them, then wait for it before any token row is read. (Issuing
        // them ahead of the row-index reads when nothing is waited for, dep 0/1, measured
        // slower at T = 4-16: the small token-row copies then queue behind the burst.)
        // Every prefetched stage gets its arrival in pass 0 (no wait precedes stage R::N),
        // so no copy is left unaccounted for at exit.
        int npre = 0;
        if (a.dep == 2) {
            npre = min(R::N, nst);
            if (lane == 0)
                for (int si = 0; si < npre; si++) {
                    const int grp = g_beg + si * GPS, ngs = min(GPS, g_end - grp);
                    uint8_t* st = ring + (size_t)si * R::SB;
                    mbar_expect_tx(&full[si], C::MATS * ngs * C::GBLK);
                    bulk_load(st, w0 + (size_t)grp * C::GBLK, ngs * C::GBLK, &full[si], wpol);
                    if (SWIGLU)
                        bulk_load(st + GPS * C::GBLK, w1 + (size_t)grp * C::GBLK, ngs * C::GBLK, &full[si], wpol);
                }
            pdl_wait();
            pdl_trigger();
        }
        int ok = 1, seq = 0;
        for (int p = 0; p < npass && ok; p++) {
            const int r0 = p * C::XROWS, nr = min(C::XROWS, n_e - r0);
            const int my_src = lane < nr ? (a.row_src ? __ldg(a.row_src + row_beg + r0 + lane)
                                                      : row_beg + r0 + lane) : 0;
            const __half* xsrc = a.X + (size_t)my_src * a.K;
            for (int si = 0; si < nst; si++, seq++) {
                const int s = seq % R::N;
                if (lane == 0 && seq >= R::N)            // the slot's previous lap was consumed
                    ok = mbar_wait(&empty[s], ((seq / R::N) - 1) & 1, deadline, a.err);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                uint8_t* st = ring + (size_t)s * R::SB;
                const int grp = g_beg + si * GPS;
                const int ngs = min(GPS, g_end - grp);
                if (lane == 0) {
                    if (seq < npre) {                      // weights already in flight
                        mbar_arrive_expect_tx(&full[s], nr * ngs * 256);
                    } else {
                        mbar_arrive_expect_tx(&full[s], C::MATS * ngs * C::GBLK + nr * ngs * 256);
                        bulk_load(st, w0 + (size_t)grp * C::GBLK, ngs * C::GBLK, &full[s], wpol);
                        if (SWIGLU)
                            bulk_load(st + GPS * C::GBLK, w1 + (size_t)grp * C::GBLK, ngs * C::GBLK, &full[s], wpol);
                    }
                }
                __syncwarp();
                if (lane < nr)
                    bulk_load(st + C::WBYTES + lane * XSTRIDE, xsrc + (size_t)grp * KGROUP_STAGE,
                              ngs * 256, &full[s], xpol);
            }
        }
        // every issued copy must land before the CTA exits
        if (lane == 0) {
            const int issued = seq;
            for (int s = 0; s < R::N && s < issued; s++) {
                const int i_last = s + ((issued - 1 - s) / R::N) * R::N;
                mbar_wait(&full[s], (i_last / R::N) & 1, deadline, a.err);
            }
        }
        return;
    }

    // -------------------------------------------------------------------- consumer warps
    if (a.dep == 2) pdl_trigger();
    const int g = lane >> 2, t = lane & 3;
    const int tile = warp % TILES, half = warp / TILES;
    const int col_lo = quad * 64 + tile * 16 + g, col_hi = col_lo + 8;
    // per-channel scales (int8, group = K) are applied to the fp32 result
    float pc0_lo = 1.f, pc0_hi = 1.f, pc1_lo = 1.f, pc1_hi = 1.f;
    if (!C::EMBED && BITS != 16) {
        pc0_lo = col_lo < a.N ? __half2float(__ldg(a.S0 + (size_t)e * a.N + col_lo)) : 0.f;
        pc0_hi = col_hi < a.N ? __half2float(__ldg(a.S0 + (size_t)e * a.N + col_hi)) : 0.f;
        if (SWIGLU) {
            pc1_lo = col_lo < a.N ? __half2float(__ldg(a.S1 + (size_t)e * a.N + col_lo)) : 0.f;
            pc1_hi = col_hi < a.N ? __half2float(__ldg(a.S1 + (size_t)e * a.N + col_hi)) : 0.f;
        }
    }
    int seq = 0;
    for (int p = 0; p < npass; p++) {
        const int r0 = p * C::XROWS, nr = min(C::XROWS, n_e - r0);
        const int ntl = (nr + 7) / 8;                     // token tiles in use (warp-uniform)
        float acc0[TM][4], acc1[TM][4];
#pragma unroll
        for (int i = 0; i < TM; i++)
#pragma unroll
            for (int c = 0; c < 4; c++) acc0[i][c] = acc1[i][c] = 0.f;
        const bool ok = ntl == 1
            ? consume_pass<BITS, SWIGLU, GROUPED, OCC, 1, TM, XT>(a, ring, full, empty, seq, nst, g_beg, g_end, deadline, acc0, acc1)
            : consume_pass<BITS, SWIGLU, GROUPED, OCC, XT, TM, XT>(a, ring, full, empty, seq, nst, g_beg, g_end, deadline, acc0, acc1);
        // the two warps of a tile hold partial sums over alternate groups: add them
        // [value][tile][lane]: consecutive lanes hit consecutive banks
        float* rw = red + tile * 32 + lane;
        constexpr int RS = TILES * 32;
        if (half == 1 && ok) {
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    rw[(i * 4 + c) * RS] = acc0[i][c];
                    if (SWIGLU) rw[(TM * 4 + i * 4 + c) * RS] = acc1[i][c];
                }
        }
        if (!consumer_bar_and(ok)) return;                // a wait timed out (already recorded)
        if (half == 0) {
            const int row0 = row_beg + r0;
#pragma unroll
            for (int i = 0; i < TM; i++) {
                if (i >= ntl) break;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int r = 8 * i + 2 * t + (c & 1);
                    const int col = (c & 2) ? col_hi : col_lo;
                    if (r >= nr || col >= a.N) continue;
                    float v0 = (acc0[i][c] + rw[(i * 4 + c) * RS]) * ((c & 2) ? pc0_hi : pc0_lo);
                    float v1 = SWIGLU ? (acc1[i][c] + rw[(TM * 4 + i * 4 + c) * RS]) * ((c & 2) ? pc1_hi : pc1_lo) : 0.f;
                    if (a.ksplit > 1) {
                        const size_t o = (size_t)(row0 + r) * a.N + col;
                        float* P = static_cast<float*>(a.Y) + (size_t)blockIdx.z * a.A * a.N * C::MATS;
                        P[o] = v0;
                        if (SWIGLU) P[(size_t)a.A * a.N + o] = v1;
                    } else {
                        const int orow = a.row_dst ? __ldg(a.row_dst + row0 + r) : row0 + r;
                        const size_t o = (size_t)orow * a.N + col;
                        float v = v0;
                        if (SWIGLU) {
                            v = v0 / (1.f + __expf(-v0)) * v1;
                            v = __half2float(__float2half_rn(v));   // h is fp16 (north star)
                        }
                        if (a.y_f32) static_cast<float*>(a.Y)[o] = v;
                        else static_cast<__half*>(a.Y)[o] = __float2half_rn(v);
                    }
                }
            }
        }
        consumer_bar();                                    // red is reused by the next pass
    }
}

// grid = (quads, min(E, A) expert slots, ksplit); 9 warps (8 consumers + 1 producer).
template <int BITS, bool SWIGLU, bool GROUPED, int OCC, int TM>
__global__ void __launch_bounds__(GTHREADS, OCC)
moe_gemm_kernel(const GemmArgs a) {
    using C = Cfg<BITS, SWIGLU, GROUPED, OCC, TM>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = align_ptr<128>(smem_raw);
    float* red = reinterpret_cast<float*>(ring + C::RING);
    uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + C::RED);
    uint64_t* empty = full + MAX_STAGES;

    // the ring's barriers (enough for either layout) are set up while the previous kernel may
    // still run; only the expert lookup waits for it (dep 1: the offsets are its output)
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::template Ring<1>::N; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CONSUMERS);
        }
        fence_barrier_init();
    }
    __syncthreads();
    if (a.dep == 1) pdl_wait();
    int row_beg, n_e;
    const int e = nth_active_expert(a.offsets, a.E, blockIdx.y, row_beg, n_e);
    if (e < 0) {                                         // surplus slot of the upper bound
        pdl_trigger();
        return;
    }
    // stages sized for the CTA's largest pass: one 8-row token tile, or TM
    if (TM == 1 || n_e <= 8)
        gemm_body<BITS, SWIGLU, GROUPED, OCC, TM, 1>(a, ring, red, full, empty, e, row_beg, n_e);
    else
        gemm_body<BITS, SWIGLU, GROUPED, OCC, TM, TM>(a, ring, red, full, empty, e, row_beg, n_e);
}

// Fixed-order sum of split-K partials [ksplit][A][N] (x2 for SwiGLU: gate then up); SwiGLU
// applies silu(gate) * up after the sum. a_rows (device, optional) is the number of rows in
// use (<= A); row_dst (optional) maps row r to output row row_dst[r].
template <bool SWIGLU>
__global__ void splitk_reduce_kernel(const float* __restrict__ P, void* Y, int y_f32, int A, int N,
                                     int ksplit, const int* __restrict__ row_dst,
                                     const int* __restrict__ a_rows) {
    pdl_wait();
    pdl_trigger();
    const size_t n_all = (size_t)A * N;
    const size_t n = a_rows ? (size_t)min(A, __ldg(a_rows)) * N : n_all;
    const size_t stride = SWIGLU ? 2 * n_all : n_all;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        float s = 0.f, u = 0.f;
        for (int z = 0; z < ksplit; z++) {
            s += P[z * stride + i];
            if (SWIGLU) u += P[z * stride + n_all + i];
        }
        if (SWIGLU) s = __half2float(__float2half_rn(s / (1.f + __expf(-s)) * u));
        const size_t o = row_dst ? (size_t)__ldg(row_dst + i / N) * N + i % N : i;
        if (y_f32) static_cast<float*>(Y)[o] = s;
        else static_cast<__half*>(Y)[o] = __float2half_rn(s);
    }
}

// ------------------------------------------------------------------ packing
// Scales (and zeros) per (e, group, column) -- the quantisers of the oracle:
//   symmetric (03_moe_wq_decode.cu:65-72): s = fp16(max|w| / qmax) (1 if 0)
//   asymmetric int4: s = fp16((max(w,0) - min(w,0)) / 15) (1 if equal),
//                    z = clamp(rn(-min(w,0) / s), 0, 15)
// One thread per column (symmetric) or per 8-column zero-point word (asymmetric).
__global__ void quant_params_kernel(const __half* W, __half* S, uint32_t* Z, int E, int K, int N,
                                    int group, int bits, int asym) {
    const int ngr = K / group;
    const int cols_per_item = asym ? 8 : 1;
    const int items_per_row = N / cols_per_item;
    const size_t total = (size_t)E * ngr * items_per_row;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int it = (int)(i % items_per_row);
        const int grp = (int)((i / items_per_row) % ngr);
        const int e = (int)(i / ((size_t)items_per_row * ngr));
        const size_t srow = ((size_t)e * ngr + grp) * N;
        uint32_t word = 0;
        for (int c = 0; c < cols_per_item; c++) {
            const int n = it * cols_per_item + c;
            const __half* w = W + ((size_t)e * K + (size_t)grp * group) * N + n;
            if (asym) {
                float mn = 0.f, mx = 0.f;
                for (int k = 0; k < group; k++) {
                    const float v = __half2float(w[(size_t)k * N]);
                    mn = fminf(mn, v);
                    mx = fmaxf(mx, v);
                }
                const __half hs = __float2half_rn(mx > mn ? __fdiv_rn(mx - mn, 15.f) : 1.f);
                const int z = max(0, min(15, __float2int_rn(__fdiv_rn(-mn, __half2float(hs)))));
                S[srow + n] = hs;
                word |= (uint32_t)z << (4 * c);
            } else {
                const float qmax = bits == 8 ? 127.f : 7.f;
                float m = 0.f;
                for (int k = 0; k < group; k++) m = fmaxf(m, fabsf(__half2float(w[(size_t)k * N])));
                S[srow + n] = __float2half_rn(m > 0.f ? __fdiv_rn(m, qmax) : 1.f);
            }
        }
        if (asym) Z[((size_t)e * ngr + grp) * (N / 8) + it] = word;
    }
}

// Code of weight (e, k, n): offset-binary symmetric or asymmetric with zero point.
__device__ __forceinline__ int quant_code(const __half* W, const __half* S, const uint32_t* Z,
                                          int e, int k, int n, int K, int N, int group, int bits,
                                          int asym) {
    if (n >= N) return asym ? 0 : (bits == 8 ? 128 : 8);     // padding columns decode to 0
    const int ngr = K / group, grp = k / group;
    const float s = __half2float(S[((size_t)e * ngr + grp) * N + n]);
    const int q = __float2int_rn(__fdiv_rn(__half2float(W[((size_t)e * K + k) * N + n]), s));
    if (asym) {
        const int z = (Z[((size_t)e * ngr + grp) * (N / 8) + n / 8] >> (4 * (n % 8))) & 15;
        return max(0, min(15, q + z));
    }
    const int qmax = bits == 8 ? 127 : 7;
    return max(-qmax, min(qmax, q)) + (bits == 8 ? 128 : 8);
}

// Record of (expert e, 16-column tile, k group grp).
__device__ __forceinline__ uint8_t* record_ptr(uint8_t* P, int bits, int group, int K, int N,
                                               int e, int tile, int grp) {
    return P + block_offset(bits, group, K, N, e, tile / 4, grp) +
           (size_t)(tile % 4) * record_bytes(bits, group);
}

// Where the packer takes its codes from: quantising fp16 weights with the scales (and zero
// points) computed by quant_params_kernel.
struct QuantSource {
    const __half* W;
    const __half* S;
    const uint32_t* Z;
    int E, K, N, group, bits, asym;
    __device__ uint16_t half_bits(int e, int k, int n) const {
        return __half_as_ushort(W[((size_t)e * K + k) * N + n]);
    }
    __device__ uint32_t code(int e, int k, int n) const {
        return (uint32_t)quant_code(W, S, Z, e, k, n, K, N, group, bits, asym);
    }
};

// ... or reading them from words the reference's pack_weights<BITS> wrote
// (03_moe_wq_decode.cu:43-87): word widx(e, k, cw) = ((e * (K/4) + k/4) * ncw + cw) * 4 + k%4
// holds columns cw*CPT .. cw*CPT+CPT-1 (CPT = 32/bits) at bit offsets bits*c, as
// offset-binary codes (q + 8 / q + 128) or, for bits 16, two fp16 values. The codes are
// taken as they are: the record stores the same offset-binary codes the quantiser would
// have produced from the same weights.
struct RefPackedSource {
    const uint32_t* P;
    int K, N, bits;
    __device__ uint32_t word(int e, int k, int n) const {
        const int cpt = 32 / bits, ncw = N / cpt;
        return __ldg(P + (((size_t)e * (K / 4) + k / 4) * ncw + n / cpt) * 4 + k % 4);
    }
    __device__ uint16_t half_bits(int e, int k, int n) const {
        return (uint16_t)(word(e, k, n) >> (16 * (n % 2)));
    }
    __device__ uint32_t code(int e, int k, int n) const {
        if (n >= N) return bits == 8 ? 128u : 8u;            // padding columns decode to 0
        const int cpt = 32 / bits;
        return (word(e, k, n) >> (bits * (n % cpt))) & ((1u << bits) - 1u);
    }
};

// One thread per (e, tile, k16 step, lane): writes that lane's fragment bytes; the lane-0
// thread of each group's first step also writes the record's embedded parameters (scales S
// [E][K/group][N] and, for asym, zero nibbles Z, both in the reference's layout).
template <class Src>
__global__ void pack_kernel(Src src, const __half* S, const uint32_t* Z, uint8_t* P,
                            int E, int K, int N, int group, int bits, int asym) {
    const int steps = K / 16;
    const int ntiles = num_quads(N) * 4;
    const size_t total = (size_t)E * ntiles * steps * 32;
    const int bpl = bytes_per_lane(bits);
    const int code = group_code_bytes(bits);
    const bool embed = embeds_params(bits, group);
    const int ngr = K / group;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int lane = (int)(i % 32);
        const int ks = (int)((i / 32) % steps);
        const int nt = (int)((i / ((size_t)32 * steps)) % ntiles);
        const int e = (int)(i / ((size_t)32 * steps * ntiles));
        uint8_t* recp = record_ptr(P, bits, group, K, N, e, nt, ks / 8);
        uint8_t* dst = recp + frag_offset(bits, ks % 8, lane);
        uint32_t out[4] = {0, 0, 0, 0};
        for (int j = 0; j < 8; j++) {
            int k, c;
            frag_coord(ks, lane, j, &k, &c);
            const int n = nt * 16 + c;
            if (bits == 16) {
                const uint16_t h = n < N ? src.half_bits(e, k, n) : 0;
                out[j >> 1] |= (uint32_t)h << (16 * (j & 1));
            } else if (bits == 8) {
                const uint32_t q = src.code(e, k, n);
                const int byte = (j >> 2) * 4 + ((j >> 1) & 1) + 2 * (j & 1);
                out[byte >> 2] |= q << (8 * (byte & 3));
            } else {
                const uint32_t q = src.code(e, k, n);
                const int nib = (j >> 1) + 4 * (j & 1);
                out[0] |= q << (4 * nib);
            }
        }
        for (int wdx = 0; wdx < bpl / 4; wdx++) reinterpret_cast<uint32_t*>(dst)[wdx] = out[wdx];
        if (embed && lane == 0 && ks % 8 == 0) {
            const int grp = (ks * 16) / group;
            __half* sc = reinterpret_cast<__half*>(recp + code);
            uint32_t zw[2] = {0, 0};
            for (int c = 0; c < 16; c++) {
                const int n = nt * 16 + c;
                sc[c] = n < N ? S[((size_t)e * ngr + grp) * N + n] : __float2half(0.f);
                int z = 8;
                if (asym) z = n < N ? (Z[((size_t)e * ngr + grp) * (N / 8) + n / 8] >> (4 * (n % 8))) & 15 : 0;
                if (bits == 4) zw[c / 8] |= (uint32_t)z << (4 * (c % 8));
            }
            uint32_t* pw = reinterpret_cast<uint32_t*>(recp + code + 32);
            pw[0] = zw[0];
            pw[1] = zw[1];
            pw[2] = 0;
            pw[3] = 0;
        }
    }
}

// Dequantised fp32 weights [E][K][N] from the packed codes (for bit-exact checks): the
// exact (q - z) * s of host_weight (03_moe_wq_decode.cu:336-348).
__global__ void dequant_kernel(const uint8_t* P, const __half* S, const uint32_t* Z, float* Wd,
                               int E, int K, int N, int group, int bits, int asym) {
    const size_t total = (size_t)E * K * N;
    const int ngr = K / group;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int n = (int)(i % N);
        const int k = (int)((i / N) % K);
        const int e = (int)(i / ((size_t)N * K));
        const int nt = n / 16, col = n % 16;
        // invert frag_coord: k = blk*32 + 8t + 4s + kq, col = g + 8*(reg&1)
        const int blk = k / 32, r = k % 32, t = r / 8, s = (r % 8) / 4, kq = r % 4;
        const int g = col % 8, hi_col = col / 8;
        const int lane = g * 4 + t, ks = blk * 2 + s;
        const int reg = (kq >= 2 ? 2 : 0) + hi_col, j = reg * 2 + (kq & 1);
        const uint8_t* src = record_ptr(const_cast<uint8_t*>(P), bits, group, K, N, e, nt, ks / 8) +
                             frag_offset(bits, ks % 8, lane);
        float v;
        if (bits == 16) {
            v = __half2float(reinterpret_cast<const __half*>(src)[j]);
        } else {
            int q, z;
            if (bits == 8) {
                const int byte = (j >> 2) * 4 + ((j >> 1) & 1) + 2 * (j & 1);
                q = src[byte];
                z = 128;
            } else {
                const int nib = (j >> 1) + 4 * (j & 1);
                q = (*reinterpret_cast<const uint32_t*>(src) >> (4 * nib)) & 15;
                z = asym ? (Z[((size_t)e * ngr + k / group) * (N / 8) + n / 8] >> (4 * (n % 8))) & 15 : 8;
            }
            v = (float)(q - z) * __half2float(S[((size_t)e * ngr + k / group) * N + n]);
        }
        Wd[i] = v;
    }
}

// ------------------------------------------------------------------ host
using KernelFn = const void*;

struct Variant {
    KernelFn fn;
    int smem;
};
#define CKL_V(B, SW, GR, OCC) \
    Variant{reinterpret_cast<KernelFn>(moe_gemm_kernel<B, SW, GR, OCC, TMAX>), Cfg<B, SW, GR, OCC>::SMEM}
#define CKL_V1(SW, OCC) \
    Variant{reinterpret_cast<KernelFn>(moe_gemm_kernel<4, SW, true, OCC, 1>), Cfg<4, SW, true, OCC, 1>::SMEM}
// 3 CTAs per SM only for int4 (its stages fit twice in 64 KB; measured faster past one wave
// of 2). The int8 and fp16 stages are 1.6-2.4x larger: at 64 KB a ring would hold one stage.
// tm = 1: one token tile per pass (int4 only; for batches where no expert can have more
// than 16 rows).
Variant gemm_variant(int bits, bool swiglu, bool grouped, int occ, int tm = TMAX) {
    if (bits == 4 && tm == 1)
        return occ == 3 ? (swiglu ? CKL_V1(true, 3) : CKL_V1(false, 3))
                        : (swiglu ? CKL_V1(true, 2) : CKL_V1(false, 2));
    if (bits == 4)
        return occ == 3 ? (swiglu ? CKL_V(4, true, true, 3) : CKL_V(4, false, true, 3))
                        : (swiglu ? CKL_V(4, true, true, 2) : CKL_V(4, false, true, 2));
    if (bits == 8) {
        if (grouped) return swiglu ? CKL_V(8, true, true, 2) : CKL_V(8, false, true, 2);
        return swiglu ? CKL_V(8, true, false, 2) : CKL_V(8, false, false, 2);
    }
    return swiglu ? CKL_V(16, true, false, 2) : CKL_V(16, false, false, 2);
}
#undef CKL_V
#undef CKL_V1
bool gemm_occ3(int bits) { return bits == 4; }

ckl_status gemm_setup(const DeviceInfo* di) {
    static ckl_status st[64];
    static std::once_flag once[64];
    std::call_once(once[di->device], [di] {
        st[di->device] = CKL_OK;
        for (int bits : {4, 8, 16})
            for (int occ : {2, 3})
            for (int sw = 0; sw < 2; sw++)
                for (int gr = 0; gr < 2; gr++) {
                    if (occ == 3 && !gemm_occ3(bits)) continue;
                    for (int tm = 1; tm <= TMAX; tm++) {
                        if (tm == 1 && bits != 4) continue;
                        const Variant v = gemm_variant(bits, sw, gr, occ, tm);
                        cudaError_t e = cudaFuncSetAttribute(
                            v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, v.smem);
                        if (e != cudaSuccess) {
                            st[di->device] = cuda_status(e, "moe gemm setup");
                            return;
                        }
                    }
                }
    });
    return st[di->device];
}

ckl_status check_weights(const ckl_moe_weights* w, const char* what) {
    if (!w) return fail(CKL_INVALID_ARG, "%s: weights NULL", what);
    if (w->bits != 4 && w->bits != 8 && w->bits != 16)
        return fail(CKL_UNSUPPORTED_SHAPE, "%s: bits=%d (4, 8 or 16)", what, w->bits);
    if (w->E <= 0 || w->E > 256 || w->K <= 0 || w->K % 128 || w->N <= 0 || w->N % 8)
        return fail(CKL_UNSUPPORTED_SHAPE, "%s: E=%d K=%d N=%d (E<=256, K%%128==0, N%%8==0)", what,
                    w->E, w->K, w->N);
    if (w->bits != 16 && w->group != 128 && w->group != w->K)
        return fail(CKL_UNSUPPORTED_SHAPE, "%s: group=%d (128 or K)", what, w->group);
    if (w->bits == 4 && w->group != 128)
        return fail(CKL_UNSUPPORTED_SHAPE, "%s: int4 needs group 128", what);
    if (w->asym && w->bits != 4) return fail(CKL_UNSUPPORTED_SHAPE, "%s: zero points are int4 only", what);
    if (!w->packed || (w->bits != 16 && !w->scales) || (w->asym && !w->zeros))
        return fail(CKL_INVALID_ARG, "%s: NULL weight buffer", what);
    if ((uintptr_t)w->packed & 15) return fail(CKL_INVALID_ARG, "%s: packed must be 16-byte aligned", what);
    return CKL_OK;
}

// group as laid out in the packed buffer (fp16 has none: records hold codes only)
inline int layout_group(const ckl_moe_weights* w) { return w->bits == 16 ? w->K : w->group; }

int pick_ksplit(const DeviceInfo* di, int quads, int slots, int K) {
    const int busy = quads * slots;
    const int ngroups = K / KGROUP_STAGE;
    int ks = 1;
    while (ks * 2 <= ngroups / 4 && busy * ks * 2 <= di->sms) ks *= 2;
    return ks;
}

}  // namespace moe
}  // namespace ckl


using namespace ckl;
using namespace ckl::moe;

extern "C" {

size_t ckl_moe_packed_bytes(int bits, int E, int K, int N, int group) {
    if (E <= 0 || K <= 0 || N <= 0 || K % KGROUP_STAGE) return 0;
    return packed_bytes(bits, bits == 16 ? K : group, E, K, N);
}

size_t ckl_moe_scale_count(int E, int K, int N, int group) {
    return group > 0 ? (size_t)E * (K / group) * N : 0;
}

size_t ckl_moe_zero_words(int E, int K, int N, int group) {
    return group > 0 ? (size_t)E * (K / group) * (N / 8) : 0;
}

ckl_status ckl_moe_pack_weights(const void* W, ckl_moe_weights* w, void* stream) {
    ckl_status st = check_weights(w, "moe_pack_weights");
    if (st != CKL_OK) return st;
    if (!W) return fail(CKL_INVALID_ARG, "moe_pack_weights: W is NULL");
    const cudaStream_t s = (cudaStream_t)stream;
    const int group = layout_group(w);
    if (w->bits != 16) {
        quant_params_kernel<<<1024, 256, 0, s>>>(static_cast<const __half*>(W),
                                                 static_cast<__half*>(w->scales),
                                                 static_cast<uint32_t*>(w->zeros), w->E, w->K, w->N,
                                                 group, w->bits, w->asym);
        CKL_CUDA_TRY(cudaGetLastError());
    }
    const QuantSource src{static_cast<const __half*>(W), static_cast<const __half*>(w->scales),
                          static_cast<const uint32_t*>(w->zeros), w->E, w->K, w->N, group,
                          w->bits, w->asym};
    pack_kernel<<<2048, 256, 0, s>>>(src, static_cast<const __half*>(w->scales),
                                     static_cast<const uint32_t*>(w->zeros),
                                     static_cast<uint8_t*>(w->packed), w->E, w->K, w->N, group,
                                     w->bits, w->asym);
    CKL_CUDA_TRY(cudaGetLastError());
    return CKL_OK;
}

ckl_status ckl_moe_import_reference_packed(const uint32_t* P, const void* Sc, ckl_moe_weights* w,
                                           void* stream) {
    ckl_status st = check_weights(w, "moe_import_reference_packed");
    if (st != CKL_OK) return st;
    if (w->asym) return fail(CKL_UNSUPPORTED_SHAPE, "moe_import_reference_packed: the reference's codes are symmetric (asym must be 0)");
    if (w->bits != 16 && w->group != KGROUP_STAGE)
        return fail(CKL_UNSUPPORTED_SHAPE, "moe_import_reference_packed: the reference's groups are 128 along K (group=%d)", w->group);
    if (!P || (w->bits != 16 && !Sc)) return fail(CKL_INVALID_ARG, "moe_import_reference_packed: P/Sc NULL");
    if ((uintptr_t)P & 3) return fail(CKL_INVALID_ARG, "moe_import_reference_packed: P must be 4-byte aligned");
    const cudaStream_t s = (cudaStream_t)stream;
    if (w->bits != 16 && Sc != w->scales)    // the scales keep the reference's layout
        CKL_CUDA_TRY(cudaMemcpyAsync(w->scales, Sc, ckl_moe_scale_count(w->E, w->K, w->N, w->group) * sizeof(__half),
                                     cudaMemcpyDeviceToDevice, s));
    const RefPackedSource src{P, w->K, w->N, w->bits};
    pack_kernel<<<2048, 256, 0, s>>>(src, static_cast<const __half*>(w->bits != 16 ? w->scales : nullptr),
                                     nullptr, static_cast<uint8_t*>(w->packed), w->E, w->K, w->N,
                                     layout_group(w), w->bits, 0);
    CKL_CUDA_TRY(cudaGetLastError());
    return CKL_OK;
}

ckl_status ckl_moe_dequant_weights(const ckl_moe_weights* w, float* W_out, void* stream) {
    ckl_status st = check_weights(w, "moe_dequant_weights");
    if (st != CKL_OK) return st;
    if (!W_out) return fail(CKL_INVALID_ARG, "moe_dequant_weights: output NULL");
    dequant_kernel<<<2048, 256, 0, (cudaStream_t)stream>>>(
        static_cast<const uint8_t*>(w->packed), static_cast<const __half*>(w->scales),
        static_cast<const uint32_t*>(w->zeros), W_out, w->E, w->K, w->N, layout_group(w), w->bits,
        w->asym);
    CKL_CUDA_TRY(cudaGetLastError());
    return CKL_OK;
}

size_t ckl_moe_gemm_workspace_size(const ckl_moe_weights* w, int A, int swiglu, int force_ksplit) {
    if (!w || A <= 0 || w->K <= 0) return 0;
    const DeviceInfo* di = device_info();
    if (!di) return 0;
    const int ks = force_ksplit > 0 ? std::min(force_ksplit, w->K / KGROUP_STAGE)
                                    : pick_ksplit(di, num_quads(w->N), std::min(w->E, A), w->K);
    if (ks <= 1) return 0;
    return (size_t)ks * A * w->N * sizeof(float) * (swiglu ? 2 : 1);
}

ckl_status ckl_moe_expert_gemm_ex(const void* X, const int* row_src, const int* offsets, int A,
                                  const ckl_moe_weights* w0, const ckl_moe_weights* w1, void* Y,
                                  int y_f32, int force_ksplit, void* workspace,
                                  size_t workspace_bytes, void* stream) {
    return ckl::moe::expert_gemm(X, row_src, offsets, A, A, w0, w1, Y, y_f32, force_ksplit,
                                 workspace, workspace_bytes, stream);
}

}  // extern "C"

namespace ckl {
namespace moe {

// max_rows bounds the rows of any one expert (A in general; T for a routed batch, since a
// token reaches an expert at most once); it sizes the token tiles of a pass.
ckl_status expert_gemm(const void* X, const int* row_src, const int* offsets, int A, int max_rows,
                       const ckl_moe_weights* w0, const ckl_moe_weights* w1, void* Y, int y_f32,
                       int force_ksplit, void* workspace, size_t workspace_bytes, void* stream,
                       int dep, const int* row_dst, const int* a_rows) {
    ckl_status st = check_weights(w0, "moe_expert_gemm");
    if (st != CKL_OK) return st;
    const bool swiglu = w1 != nullptr;
    if (swiglu) {
        st = check_weights(w1, "moe_expert_gemm (up)");
        if (st != CKL_OK) return st;
        if (w1->bits != w0->bits || w1->E != w0->E || w1->K != w0->K || w1->N != w0->N ||
            w1->group != w0->group || w1->asym != w0->asym)
            return fail(CKL_INVALID_ARG, "moe_expert_gemm: gate/up weights differ in format");
    }
    if (A < 0) return fail(CKL_INVALID_ARG, "moe_expert_gemm: A < 0");
    if (A == 0) return CKL_OK;
    if (!X || !offsets || !Y) return fail(CKL_INVALID_ARG, "moe_expert_gemm: NULL tensor");
    if ((uintptr_t)X & 15) return fail(CKL_INVALID_ARG, "moe_expert_gemm: X must be 16-byte aligned");
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    st = gemm_setup(di);
    if (st != CKL_OK) return st;
    const int quads = num_quads(w0->N);
    const int slots = std::min(w0->E, A);
    const int ks = force_ksplit > 0 ? std::min(force_ksplit, w0->K / KGROUP_STAGE)
                                    : pick_ksplit(di, quads, slots, w0->K);
    const size_t need = ks > 1 ? (size_t)ks * A * w0->N * sizeof(float) * (swiglu ? 2 : 1) : 0;
    if (ks > 1 && (!workspace || workspace_bytes < need))
        return fail(CKL_WORKSPACE_TOO_SMALL, "moe_expert_gemm needs %zu workspace bytes, got %zu",
                    need, workspace_bytes);
    const bool grouped = embeds_params(w0->bits, w0->group);   // int4, or int8 group 128
    // one token tile per pass when no expert can have more than 16 rows (int4): a lighter
    // kernel; otherwise passes of up to 16 rows
    const int tm = (w0->bits == 4 && grouped && max_rows <= 16) ? 1 : TMAX;
    GemmArgs a;
    a.X = static_cast<const __half*>(X);
    a.row_src = row_src;
    a.offsets = offsets;
    a.W0 = static_cast<const uint8_t*>(w0->packed);
    a.S0 = static_cast<const __half*>(w0->scales);
    a.W1 = swiglu ? static_cast<const uint8_t*>(w1->packed) : nullptr;
    a.S1 = swiglu ? static_cast<const __half*>(w1->scales) : nullptr;
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
    a.dep = dep;
    void* args[] = {&a};
    // 3 CTAs per SM (64 KB rings) when the grid is more than one wave of 2 (int4), else the
    // deeper rings of 2 CTAs per SM
    const int occ = gemm_occ3(w0->bits) && (long long)quads * slots * ks > 2LL * di->sms ? 3 : 2;
    const Variant v = gemm_variant(w0->bits, swiglu, grouped, occ, tm);
    dim3 grid((unsigned)quads, (unsigned)slots, (unsigned)ks);
    const cudaStream_t s = (cudaStream_t)stream;
    CKL_CUDA_TRY(launch(v.fn, grid, dim3(GTHREADS), v.smem, s, args, dep != 0));
    if (ks > 1) {
        const float* P = static_cast<const float*>(workspace);
        int ksv = ks, Av = A, Nv = w0->N;
        void* rargs[] = {&P, &Y, &y_f32, &Av, &Nv, &ksv, &row_dst, &a_rows};
        const void* rfn = swiglu ? reinterpret_cast<const void*>(splitk_reduce_kernel<true>)
                                 : reinterpret_cast<const void*>(splitk_reduce_kernel<false>);
        CKL_CUDA_TRY(launch(rfn, dim3(256), dim3(256), 0, s, rargs, dep != 0));
    }
    return CKL_OK;
}

}  // namespace moe
}  // namespace ckl

extern "C" {

ckl_status ckl_moe_expert_gemm(const void* Xp, void* Yp, const int* offsets, int A,
                               const ckl_moe_weights* w, int force_ksplit, void* workspace,
                               size_t workspace_bytes, void* stream) {
    return ckl_moe_expert_gemm_ex(Xp, nullptr, offsets, A, w, nullptr, Yp, 0, force_ksplit,
                                  workspace, workspace_bytes, stream);
}

}  // extern "C"
