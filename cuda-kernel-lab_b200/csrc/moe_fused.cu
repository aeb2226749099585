// moe_fused.cu -- the W4A16 SwiGLU MoE decode layer's two expert GEMMs as ONE persistent
// kernel (gate/up with SwiGLU, then down), for the decode sizes of the fine-grained MoE
// (int4 group-128 weights, d and F <= 2048).
//
// Replaces, for that case, the per-GEMM launches of moe_gemm.cu (the reference's
// QuantWeights::run / moe_wq_gemv, 03_moe_wq_decode.cu:124-333, and MoeDecode's chain,
// 03:350-391). Why one kernel: a decode step streams each active expert's weights once, so
// the layer is bound by HBM; short per-(quad, expert) CTAs launched wave after wave pay a
// pipeline ramp per CTA and a partial last wave, and the down GEMM cannot start streaming
// before the gate/up launch ends. Here:
//
//   * one CTA per SM; each CTA takes an equal share of the gate/up weight stream and an equal
//     share of the down stream, cut at 128-k group granularity in (expert, pass, quad, group)
//     order -- every SM streams the same number of bytes whatever the routing;
//   * a unit (expert, pass of <= 16 rows, 64-column quad) cut between CTAs is summed by the
//     last CTA to finish its part, in CTA order (fp32 partials in the workspace), so the
//     result does not depend on timing;
//   * warp 12 streams weights into a ring of 25 KB stages (cp.async.bulk, evict-first; no
//     multicast), warp 13 stages each (expert, pass)'s activation rows ONCE for all of its
//     quads (full K; gate/up rows gathered from X by row_src, down rows = h), and 12 consumer
//     warps (4 column tiles x 3 group slots) decode and multiply with mma.sync exactly as
//     moe_gemm.cu does (swap-AB: weights the M=16 operand, up to 8 tokens the N operand);
//   * the down stream does not wait for gate/up: its weights fill the ring while the expert's
//     h rows are still being produced; only the row copy waits, on a per-expert counter of
//     finished (gate/up unit-pass, tile) results (release/acquire at gpu scope, bounded).
//
// The routing (offsets, row_src) comes from route_kernel (moe_layer.cu), which also zeroes the
// counters this kernel uses; the combine (fixed slot order) runs after it. Both are chained
// with programmatic dependent launch.

#include <algorithm>
#include <mutex>

#include "ckl_internal.h"
#include "ckl_ptx.cuh"
#include "moe_common.cuh"
#include "moe_internal.h"

namespace ckl {
namespace moe {
namespace fused {

constexpr int TILES = 4;                      // 16-column tiles of a 64-column quad
constexpr int SLOTS = 3;                      // group slots: consumer warp = slot * 4 + tile
constexpr int CONS = TILES * SLOTS;           // 12 consumer warps (14 warps in all: 128 registers)
constexpr int WPROD = CONS;                   // warp 12: weight producer
constexpr int XPROD = CONS + 1;               // warp 13: activation-row producer
constexpr int THREADS = (CONS + 2) * 32;
constexpr int ROWS = 16;                      // rows per pass (two 8-token MMA tiles)
constexpr int TMAX = ROWS / 8;
constexpr int GPS0 = SLOTS;                   // 128-k groups per stage, gate/up (2 matrices)
constexpr int GPS1 = 2 * SLOTS;               // ... down (1 matrix): the same stage bytes
constexpr int REC = 1024 + PARAM_BYTES;       // int4 record: 16 columns x 128 k + parameters
constexpr int GBLK = TILES * REC;             // one group of one matrix for a quad
constexpr int SLOT = 2 * GPS0 * GBLK;         // stage bytes (== GPS1 * GBLK)
constexpr int MAXK = 2048;                    // K of either matrix: full-K rows in smem
constexpr int RVALS = TMAX * 4 * 2;           // fp32 accumulators per lane (tiles x 4 x mats)
constexpr int PART_FLOATS = RVALS * 32;       // one tile's partial (lane-major)
constexpr int RED_BYTES = (SLOTS - 1) * TILES * PART_FLOATS * 4;
constexpr int MAX_E = 256;
constexpr int SMEM_LIMIT = 232448;            // opt-in dynamic shared memory per block (227 KB)
static_assert(GPS1 * GBLK == SLOT, "stages of both phases have the same size");

struct Args {
    const __half* X;          // [T][d] layer input
    const int* offsets;       // [E+1] expert row ranges (from the routing)
    const int* row_src;       // [A] token of each expert-sorted row
    const uint8_t* Wg;        // packed gate [E][d][F]
    const uint8_t* Wu;        // packed up   [E][d][F]
    const uint8_t* Wd;        // packed down [E][F][d]
    __half* h;                // [A][F] fp16(silu(gate) * up), expert order
    float* y;                 // [A][d] fp32 down output, expert order
    float* part;              // [grid][2][TILES][PART_FLOATS] partials of cut units
    int* cnt0;                // [unit-passes][TILES] arrivals at cut gate/up units
    int* cnt1;                // [unit-passes][TILES] ... down units
    int* hdone;               // [E] finished (gate/up unit-pass, tile) results per expert
    unsigned* err;
    unsigned long long timeout_ns;
    int E, d, F, stages, xstride, xrows;   // X staging: xrows rows of xstride bytes
};

// Work of one phase: unit-passes ordered by (active expert j, pass p, quad q), each G groups
// of 128 k; pre[j] = first unit-pass of active expert j (pre[nact] = total).
struct Phase {
    const int* pre;
    int P, Q, G;
    long long N;              // groups in all (pre[nact] * G)
    long long lo, hi;         // this CTA's range [lo, hi)
};

struct Seg {
    int j, p, q, up, g0, g1;  // groups [g0, g1) of unit-pass up = (j, p, q)
    long long i0;             // its first global group index
};

__device__ __forceinline__ int find_expert(const int* pre, int nact, int up) {
    int lo = 0, hi = nact - 1;               // largest j with pre[j] <= up
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= up) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ Seg seg_at(const Phase& ph, int nact, long long i) {
    Seg s;
    s.up = (int)(i / ph.G);
    s.g0 = (int)(i - (long long)s.up * ph.G);
    const long long end = min(ph.hi, (long long)(s.up + 1) * ph.G);
    s.g1 = s.g0 + (int)(end - i);
    s.j = find_expert(ph.pre, nact, s.up);
    const int rem = s.up - ph.pre[s.j];
    s.p = rem / ph.Q;
    s.q = rem - s.p * ph.Q;
    s.i0 = i;
    return s;
}

// The CTA whose range holds global group index i (ranges are [c*N/nc, (c+1)*N/nc)).
__device__ __forceinline__ int cta_of(long long i, long long N, int nc) {
    return (int)(((i + 1) * nc - 1) / N);
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// int4 fragment decode to exact (q - z) in fp16 (layout and arithmetic of moe_gemm.cu's dec4:
// nibble order in moe_common.cuh, fp16 magic number 0x6400).
__device__ __forceinline__ void dec4f(uint32_t w, uint32_t zc0, uint32_t zc1n, uint32_t (&a)[4]) {
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

// One 128-k group of one 16-column tile for NT token tiles: MATS matrices (gate and up share
// the activation fragments). acc += s * sum_k (q - z) x, per matrix.
template <int NT, int MATS>
__device__ __forceinline__ void group_mma(const uint8_t* rec0, const uint8_t* rec1, const uint8_t* xs,
                                          int xstride, float (&acc)[RVALS]) {
    const int lane = threadIdx.x & 31, g = lane >> 2;
    uint32_t zc0[2], zc1[2];
    float s_lo[2], s_hi[2];
#pragma unroll
    for (int m = 0; m < MATS; m++) {
        const uint8_t* rec = m ? rec1 : rec0;
        const __half* scp = reinterpret_cast<const __half*>(rec + 1024);
        s_lo[m] = __half2float(scp[g]);
        s_hi[m] = __half2float(scp[g + 8]);
        const uint2 zw = *reinterpret_cast<const uint2*>(rec + 1024 + 32);
        const uint32_t z_lo = (zw.x >> (4 * g)) & 15, z_hi = (zw.y >> (4 * g)) & 15;
        zc0[m] = (0x6400u + z_lo) * 0x10001u;             // half2(1024 + z)
        zc1[m] = (0xD400u + 16u * z_hi) * 0x10001u;       // half2(-(64 + z))
    }
    float gacc[MATS][NT][4];
#pragma unroll
    for (int m = 0; m < MATS; m++)
#pragma unroll
        for (int i = 0; i < NT; i++)
#pragma unroll
            for (int c = 0; c < 4; c++) gacc[m][i][c] = 0.f;
#pragma unroll
    for (int kc = 0; kc < 2; kc++) {                      // 16-byte lane chunks: 4 k16 steps each
        const uint4 c0 = *reinterpret_cast<const uint4*>(rec0 + kc * 512 + lane * 16);
        uint4 c1 = c0;
        if (MATS == 2) c1 = *reinterpret_cast<const uint4*>(rec1 + kc * 512 + lane * 16);
        const uint32_t q0[4] = {c0.x, c0.y, c0.z, c0.w};
        const uint32_t q1[4] = {c1.x, c1.y, c1.z, c1.w};
#pragma unroll
        for (int kb2 = 0; kb2 < 2; kb2++) {               // 32-wide k blocks of the chunk
            const int kb = kc * 2 + kb2;
            uint4 xv[NT];
#pragma unroll
            for (int i = 0; i < NT; i++)
                xv[i] = *reinterpret_cast<const uint4*>(xs + (size_t)i * 8 * xstride + kb * 64);
#pragma unroll
            for (int hb = 0; hb < 2; hb++) {              // the two k16 steps of the block
                uint32_t w0[4], w1[4];
                dec4f(q0[kb2 * 2 + hb], zc0[0], zc1[0], w0);
                if (MATS == 2) dec4f(q1[kb2 * 2 + hb], zc0[1], zc1[1], w1);
#pragma unroll
                for (int i = 0; i < NT; i++) {
                    const uint32_t b0 = hb ? xv[i].z : xv[i].x, b1 = hb ? xv[i].w : xv[i].y;
                    mma16816(gacc[0][i], w0, b0, b1);
                    if (MATS == 2) mma16816(gacc[1][i], w1, b0, b1);
                }
            }
        }
    }
#pragma unroll
    for (int m = 0; m < MATS; m++)
#pragma unroll
        for (int i = 0; i < NT; i++) {
            float* a = acc + m * (TMAX * 4) + i * 4;
            a[0] += s_lo[m] * gacc[m][i][0];
            a[1] += s_lo[m] * gacc[m][i][1];
            a[2] += s_hi[m] * gacc[m][i][2];
            a[3] += s_hi[m] * gacc[m][i][3];
        }
}

__device__ __forceinline__ void tile_bar(int tile) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + tile), "n"(SLOTS * 32) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(THREADS, 1) moe_layer_fused_kernel(const Args a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = align_ptr<128>(smem_raw);
    uint8_t* xbuf = ring + (size_t)a.stages * SLOT;
    float* red = reinterpret_cast<float*>(xbuf + (size_t)a.xrows * a.xstride);
    uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + RED_BYTES);
    uint64_t* empty = full + a.stages;
    uint64_t* xfull = empty + a.stages;
    uint64_t* xempty = xfull + 1;
    int* act = reinterpret_cast<int*>(xempty + 1);      // [E] active experts, id order
    int* pre0 = act + a.E;                               // [E+1]
    int* pre1 = pre0 + a.E + 1;                          // [E+1]
    int& s_nact = pre1[a.E + 1];                         // active experts

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nc = gridDim.x;
    const int Q0 = num_quads(a.F), G0 = a.d / KGROUP_STAGE;     // gate/up: N = F, K = d
    const int Q1 = num_quads(a.d), G1 = a.F / KGROUP_STAGE;     // down:    N = d, K = F

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CONS);
        }
        mbar_init(xfull, 1);
        mbar_init(xempty, CONS);
        fence_barrier_init();
    }
    pdl_wait();                                          // the routing kernel's results
    if (warp == 0) {
        // active experts in id order with their pass counts, then the unit-pass prefixes
        int n = 0;
        for (int e0 = 0; e0 < a.E; e0 += 32) {
            const int e = e0 + lane;
            const int ne = e < a.E ? __ldg(a.offsets + e + 1) - __ldg(a.offsets + e) : 0;
            const unsigned m = __ballot_sync(0xffffffffu, ne > 0);
            if (ne > 0) {
                const int pos = n + __popc(m & ((1u << lane) - 1u));
                act[pos] = e;
                pre0[pos] = (ne + ROWS - 1) / ROWS;
            }
            n += __popc(m);
        }
        __syncwarp();
        int carry = 0;
        for (int j0 = 0; j0 < n; j0 += 32) {
            const int j = j0 + lane;
            const int pj = j < n ? pre0[j] : 0;
            int inc = pj;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            __syncwarp();
            if (j < n) {
                pre0[j] = (carry + inc - pj) * Q0;
                pre1[j] = (carry + inc - pj) * Q1;
            }
            carry += __shfl_sync(0xffffffffu, inc, 31);
        }
        if (lane == 0) {
            pre0[n] = carry * Q0;
            pre1[n] = carry * Q1;
            s_nact = n;
        }
    }
    __syncthreads();
    pdl_trigger();
    const int nact = s_nact;
    if (nact == 0) return;
    const uint64_t deadline = globaltimer() + a.timeout_ns;

    // a phase's schedule, rebuilt from shared memory where each role enters it
    auto make_phase = [&](int P) {
        Phase f;
        f.pre = P ? pre1 : pre0;
        f.P = P;
        f.Q = P ? Q1 : Q0;
        f.G = P ? G1 : G0;
        f.N = (long long)f.pre[nact] * f.G;
        f.lo = (long long)blockIdx.x * f.N / nc;
        f.hi = (long long)(blockIdx.x + 1) * f.N / nc;
        return f;
    };

    if (warp == WPROD) {
        // ------------------------------------------------------------ weight producer
        const uint64_t wpol = policy_evict_first();
        int sidx = 0, ok = 1;
        for (int P = 0; P < 2 && ok; P++) {
            const Phase cur = make_phase(P);
            const int gps = P ? GPS1 : GPS0;
            const int K = P ? a.F : a.d, N = P ? a.d : a.F;
            for (long long i = cur.lo; i < cur.hi && ok;) {
                const Seg sg = seg_at(cur, nact, i);
                const int e = act[sg.j];
                for (int g = sg.g0; g < sg.g1; g += gps, sidx++) {
                    const int s = sidx % a.stages;
                    if (lane == 0 && sidx >= a.stages)
                        ok = mbar_wait(&empty[s], ((sidx / a.stages) - 1) & 1, deadline, a.err);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    if (lane == 0) {
                        const int ngs = min(gps, sg.g1 - g);
                        uint8_t* st = ring + (size_t)s * SLOT;
                        const size_t off = block_offset(4, KGROUP_STAGE, K, N, e, sg.q, g);
                        if (P == 0) {
                            mbar_arrive_expect_tx(&full[s], 2 * ngs * GBLK);
                            bulk_load(st, a.Wg + off, ngs * GBLK, &full[s], wpol);
                            bulk_load(st + GPS0 * GBLK, a.Wu + off, ngs * GBLK, &full[s], wpol);
                        } else {
                            mbar_arrive_expect_tx(&full[s], ngs * GBLK);
                            bulk_load(st, a.Wd + off, ngs * GBLK, &full[s], wpol);
                        }
                    }
                    __syncwarp();
                }
                i = (long long)sg.up * cur.G + sg.g1;
            }
        }
        if (lane == 0) {                                 // every copy lands before exit
            const int issued = sidx;
            for (int s = 0; s < a.stages && s < issued; s++) {
                const int last = s + ((issued - 1 - s) / a.stages) * a.stages;
                mbar_wait(&full[s], (last / a.stages) & 1, deadline, a.err);
            }
        }
        return;
    }

    if (warp == XPROD) {
        // ------------------------------------------------------------ activation rows
        const uint64_t xpol = policy_evict_last();
        int xrun = -1, ok = 1;
        int cP = -1, cj = -1, cp = -1;
        for (int P = 0; P < 2 && ok; P++) {
            const Phase cur = make_phase(P);
            for (long long i = cur.lo; i < cur.hi && ok;) {
                const Seg sg = seg_at(cur, nact, i);
                i = (long long)sg.up * cur.G + sg.g1;
                if (P == cP && sg.j == cj && sg.p == cp) continue;
                cP = P; cj = sg.j; cp = sg.p;
                xrun++;
                const int e = act[sg.j];
                if (xrun >= 1) {
                    if (lane == 0) ok = mbar_wait(xempty, (xrun - 1) & 1, deadline, a.err);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                }
                if (P == 1) {
                    // the expert's h rows: every (gate/up unit-pass, tile) result of e
                    const int pj = (pre0[sg.j + 1] - pre0[sg.j]) / Q0;
                    const int target = TILES * Q0 * pj;
                    if (lane == 0) {
                        while (ld_acquire_gpu(a.hdone + e) < target) {
                            if (globaltimer() > deadline) {
                                atomicOr(a.err, DEVERR_TIMEOUT);
                                ok = 0;
                                break;
                            }
                            __nanosleep(32);
                        }
                    }
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    // every lane acquires the count itself, then orders its bulk copy (async
                    // proxy) after the generic-proxy writes of h that the count covers
                    (void)ld_acquire_gpu(a.hdone + e);
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                }
                const int rb = __ldg(a.offsets + e) + ROWS * sg.p;
                const int nr = min(ROWS, __ldg(a.offsets + e + 1) - rb);
                const int rowbytes = (P ? a.F : a.d) * 2;
                if (lane == 0) mbar_arrive_expect_tx(xfull, nr * rowbytes);
                __syncwarp();
                if (lane < nr) {
                    const __half* src = P ? a.h + (size_t)(rb + lane) * a.F
                                          : a.X + (size_t)__ldg(a.row_src + rb + lane) * a.d;
                    bulk_load(xbuf + (size_t)lane * a.xstride, src, rowbytes, xfull, xpol);
                }
            }
        }
        if (lane == 0 && xrun >= 0) mbar_wait(xfull, xrun & 1, deadline, a.err);
        return;
    }

    // ---------------------------------------------------------------- consumer warps
    // A warp whose bounded wait gave up (recorded in a.err) does no more work but keeps
    // walking the schedule, so the other warps of its tile never wait at tile_bar for it.
    const int tile = warp % TILES, slot = warp / TILES;
    const int g = lane >> 2, t = lane & 3;
    int sidx = 0, xrun = -1;
    int cP = -1, cj = -1, cp = -1;
    bool dead = false;
    for (int P = 0; P < 2; P++) {
        const Phase cur = make_phase(P);
        const int gps = P ? GPS1 : GPS0;
        const int N = P ? a.d : a.F;
        int* cnt = P ? a.cnt1 : a.cnt0;
        for (long long i = cur.lo; i < cur.hi;) {
            const Seg sg = seg_at(cur, nact, i);
            i = (long long)sg.up * cur.G + sg.g1;
            const int e = act[sg.j];
            if (!(P == cP && sg.j == cj && sg.p == cp)) {
                if (xrun >= 0 && !dead) {                 // the previous rows are no longer read
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xempty);
                }
                cP = P; cj = sg.j; cp = sg.p;
                xrun++;
                if (!dead) dead = !__all_sync(0xffffffffu, mbar_wait(xfull, xrun & 1, deadline, a.err));
            }
            const int rb = __ldg(a.offsets + e) + ROWS * sg.p;
            const int nr = min(ROWS, __ldg(a.offsets + e + 1) - rb);
            const int ntl = (nr + 7) >> 3;
            float acc[RVALS];
#pragma unroll
            for (int v = 0; v < RVALS; v++) acc[v] = 0.f;
            for (int g0 = sg.g0; g0 < sg.g1; g0 += gps, sidx++) {
                if (dead) continue;
                const int s = sidx % a.stages;
                if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (sidx / a.stages) & 1, deadline, a.err))) {
                    dead = true;
                    continue;
                }
                const int ngs = min(gps, sg.g1 - g0);
                const uint8_t* st = ring + (size_t)s * SLOT;
                for (int gi = slot; gi < ngs; gi += SLOTS) {
                    const uint8_t* rec0 = st + gi * GBLK + tile * REC;
                    const uint8_t* xs = xbuf + (size_t)g * a.xstride + (size_t)(g0 + gi) * 256 + 16 * t;
                    if (P == 0) {
                        const uint8_t* rec1 = rec0 + GPS0 * GBLK;
                        if (ntl == 1) group_mma<1, 2>(rec0, rec1, xs, a.xstride, acc);
                        else group_mma<2, 2>(rec0, rec1, xs, a.xstride, acc);
                    } else {
                        if (ntl == 1) group_mma<1, 1>(rec0, rec0, xs, a.xstride, acc);
                        else group_mma<2, 1>(rec0, rec0, xs, a.xstride, acc);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }

            // ---- the slot warps of this tile add their groups (fixed order)
            if (slot > 0) {
                float* rw = red + ((slot - 1) * TILES + tile) * PART_FLOATS + lane;
#pragma unroll
                for (int v = 0; v < RVALS; v++) rw[v * 32] = acc[v];
            }
            tile_bar(tile);
            if (slot == 0) {
#pragma unroll
                for (int sl = 1; sl < SLOTS; sl++) {
                    const float* rr = red + ((sl - 1) * TILES + tile) * PART_FLOATS + lane;
#pragma unroll
                    for (int v = 0; v < RVALS; v++) acc[v] += rr[v * 32];
                }
            }
            tile_bar(tile);
            if (slot != 0 || __any_sync(0xffffffffu, dead)) continue;

            // ---- a unit cut between CTAs: partial out; the last CTA to finish its part sums
            // all parts in CTA order (so the result does not depend on which CTA is last)
            const long long u_beg = (long long)sg.up * cur.G, u_end = u_beg + cur.G;
            const int ufirst = cta_of(u_beg, cur.N, nc);
            const int ulast = cta_of(u_end - 1, cur.N, nc);
            if (ufirst != ulast) {
                const int mypos = sg.i0 == cur.lo ? 0 : 1;
                float* pp = a.part + (((size_t)blockIdx.x * 2 + mypos) * TILES + tile) * PART_FLOATS + lane;
#pragma unroll
                for (int v = 0; v < RVALS; v++) __stcg(pp + v * 32, acc[v]);
                // contributors: the CTAs in [ufirst, ulast] whose range is not empty
                int parts = 0;
                for (int c = ufirst; c <= ulast; c++)
                    parts += (long long)(c + 1) * cur.N / nc > (long long)c * cur.N / nc;
                __threadfence();
                __syncwarp();
                int old = 0;
                if (lane == 0) old = atomicAdd(cnt + sg.up * TILES + tile, 1);
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old != parts - 1) continue;           // another CTA finishes the unit
                __threadfence();
                float sum[RVALS];
#pragma unroll
                for (int v = 0; v < RVALS; v++) sum[v] = 0.f;
                for (int c = ufirst; c <= ulast; c++) {
                    const long long clo = (long long)c * cur.N / nc;
                    if ((long long)(c + 1) * cur.N / nc == clo) continue;   // empty range
                    if (c == (int)blockIdx.x) {
#pragma unroll
                        for (int v = 0; v < RVALS; v++) sum[v] += acc[v];
                        continue;
                    }
                    // the unit is c's first segment when c's range starts inside it
                    const int cpos = clo >= u_beg ? 0 : 1;
                    const float* op = a.part + (((size_t)c * 2 + cpos) * TILES + tile) * PART_FLOATS + lane;
#pragma unroll
                    for (int v = 0; v < RVALS; v++) sum[v] += __ldcg(op + v * 32);
                }
#pragma unroll
                for (int v = 0; v < RVALS; v++) acc[v] = sum[v];
            }

            // ---- final epilogue: h = fp16(silu(gate) * up), or the fp32 down rows
            const int col_lo = sg.q * 64 + tile * 16 + g;
#pragma unroll
            for (int ti = 0; ti < TMAX; ti++) {
                if (ti >= ntl) break;
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const int r = 8 * ti + 2 * t + (c & 1);
                    const int col = col_lo + ((c & 2) ? 8 : 0);
                    if (r >= nr || col >= N) continue;
                    const float v0 = acc[ti * 4 + c];
                    if (P == 0) {
                        const float v1 = acc[TMAX * 4 + ti * 4 + c];
                        const float hv = v0 / (1.f + __expf(-v0)) * v1;
                        a.h[(size_t)(rb + r) * a.F + col] = __float2half_rn(hv);
                    } else {
                        a.y[(size_t)(rb + r) * a.d + col] = v0;
                    }
                }
            }
            if (P == 0) {                                 // publish this tile's h columns
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(a.hdone + e, 1);
            }
        }
    }
}

}  // namespace fused

// Host side -----------------------------------------------------------------------------

// Whether the layer runs as the fused persistent kernel: int4 group-128 weights for all three
// matrices, and activation rows of both GEMMs (<= 16 rows x K) fitting the staging buffer.
bool fused_eligible(const ckl_moe_weights* g, const ckl_moe_weights* u, const ckl_moe_weights* d) {
    for (const ckl_moe_weights* w : {g, u, d})
        if (w->bits != 4 || w->group != KGROUP_STAGE) return false;
    if (g->K > fused::MAXK || g->N > fused::MAXK || g->E > fused::MAX_E) return false;
    if (g->K % 64 || g->N % 64) return false;            // full quads, 128-byte row pitch
    const DeviceInfo* di = device_info();
    return di && di->smem_optin >= fused::SMEM_LIMIT && di->cc_major == 10;
}

// Workspace of the fused path beyond the layer's own buffers: partials, then counters.
FusedWs fused_ws(int T, int k, int E, int d, int F, int sms) {
    FusedWs w{};
    const int A = T * k;
    const int passes_max = A / fused::ROWS + std::min(E, A) + 1;   // sum_j ceil(n_j / 16)
    w.up0_max = passes_max * num_quads(F);
    w.up1_max = passes_max * num_quads(d);
    w.cnt_words = (w.up0_max + w.up1_max) * fused::TILES + E;
    w.part = 0;
    w.cnt = align_up((size_t)sms * 2 * fused::TILES * fused::PART_FLOATS * sizeof(float), 256);
    w.total = w.cnt + align_up((size_t)w.cnt_words * sizeof(int), 256);
    return w;
}

ckl_status fused_setup(const DeviceInfo* di) {
    static ckl_status st[64];
    static std::once_flag once[64];
    std::call_once(once[di->device], [di] {
        st[di->device] = cuda_status(
            cudaFuncSetAttribute(reinterpret_cast<const void*>(fused::moe_layer_fused_kernel),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, fused::SMEM_LIMIT),
            "fused MoE layer setup");
    });
    return st[di->device];
}

// Launches the fused gate/up + down kernel (programmatic dependent launch on the routing).
ckl_status launch_fused(const void* X, const int* offsets, const int* row_src, int T, int k,
                        const ckl_moe_weights* gate, const ckl_moe_weights* up,
                        const ckl_moe_weights* down, __half* h, float* y, void* fws,
                        cudaStream_t s) {
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    ckl_status st = fused_setup(di);
    if (st != CKL_OK) return st;
    const int E = gate->E, d = gate->K, F = gate->N;
    const FusedWs L = fused_ws(T, k, E, d, F, di->sms);
    int* cnt = reinterpret_cast<int*>(static_cast<uint8_t*>(fws) + L.cnt);
    fused::Args a;
    a.X = static_cast<const __half*>(X);
    a.offsets = offsets;
    a.row_src = row_src;
    a.Wg = static_cast<const uint8_t*>(gate->packed);
    a.Wu = static_cast<const uint8_t*>(up->packed);
    a.Wd = static_cast<const uint8_t*>(down->packed);
    a.h = h;
    a.y = y;
    a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(fws) + L.part);
    a.cnt0 = cnt;
    a.cnt1 = cnt + L.up0_max * fused::TILES;
    a.hdone = cnt + (L.up0_max + L.up1_max) * fused::TILES;
    a.err = di->err_word;
    a.timeout_ns = spin_timeout_ns();
    a.E = E;
    a.d = d;
    a.F = F;
    // an expert has at most T rows; consumers read whole 8-row token tiles, so the staging
    // rows are rounded up to a multiple of 8 (rows past nr are read but never used)
    a.xrows = std::min(fused::ROWS, (T + 7) / 8 * 8);
    a.xstride = std::max(d, F) * 2 + 64;                 // 64 mod 128: conflict-free row pairs
    auto smem_for = [&](int stages) {
        return 128 + (size_t)stages * fused::SLOT + (size_t)a.xrows * a.xstride + fused::RED_BYTES +
               (size_t)(2 * stages + 2) * 8 + (size_t)(3 * E + 3) * sizeof(int);
    };
    int stages = 16;
    while (stages >= 2 && smem_for(stages) > (size_t)fused::SMEM_LIMIT) stages--;
    if (stages < 2) return fail(CKL_UNSUPPORTED_SHAPE, "fused MoE layer: shared memory");
    a.stages = stages;
    const size_t smem = smem_for(stages);
    void* args[] = {&a};
    CKL_CUDA_TRY(launch(reinterpret_cast<const void*>(fused::moe_layer_fused_kernel), dim3(di->sms),
                        dim3(fused::THREADS), smem, s, args, true));
    return CKL_OK;
}

}  // namespace moe
}  // namespace ckl
