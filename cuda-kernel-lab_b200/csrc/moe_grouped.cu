// moe_grouped.cu -- dense grouped fp16 expert GEMM on the 5th-generation tensor cores.
//
// Replaces moe_grouped_gemm<TileCfg> (02_moe_grouped_gemm.cu:86-186), the path for batches
// with tens of tokens or more per expert (prefill-sized MoE): Yp[r] = Xp[r] . W[e] for the
// rows r of every expert e (rows [offsets[e], offsets[e+1]) of the expert-sorted Xp), fp16
// in, fp32 accumulate, fp16 out, in one launch with a device-side schedule.
//
// At the reference's shapes the weight stream bounds the job (T=512, E=8, top-2, d=4096,
// f=14336: 940 MB of fp16 weights for ~128 tokens per expert, 120 GFLOP), so the kernel is
// built to keep every SM's share of the weight stream equal and in flight:
//
//   work item   (row chunk j, 256 output columns mt): chunk j is the j-th run of <= 256 rows
//               in expert order (an expert with n rows has ceil(n / 256) chunks); the weight
//               tile W[e][:, mt*256 .. +256) is read from HBM once, the chunk's rows (L2
//               resident) once per 256 columns.
//   schedule    persistent, one CTA per SM, stream-K: the items' 64-wide k blocks, laid end
//               to end (Q = items x d/64), are cut into gridDim.x equal ranges, so every CTA
//               streams the same weight bytes whatever the item count (no wave tail). An item
//               cut between CTAs is finished by the CTA holding its first k block: the others
//               (whose range starts inside it, so they do it first) leave fp32 partial tiles in
//               the workspace and raise a flag; the finisher adds them in CTA order
//               (deterministic) after its own part and clears the flags.
//   warp 0      TMA producer of the weights: per k block four 64x64 boxes (MN-major, 128-byte
//               swizzle) into a 4-stage ring of 32 KB
//   warp 2      TMA producer of the rows: 32-row boxes (K-major, 128-byte swizzle) into a
//               3-stage ring of 32 KB; the two rings run ahead independently
//   warp 1      MMA issuer: per k block 2 x 4 tcgen05.mma (M=128 each half of the columns, N =
//               rows rounded up to 16, K=16), fp32 accumulators in TMEM columns [0, 256) and
//               [256, 512); tcgen05.commit frees the stages, then signals the epilogue
//   warps 4-11  epilogue: tcgen05.ld of each warp's 32 TMEM lanes (= output columns) of one
//               half, fp16 rows to Yp (or fp32 partials to the workspace)
//
// The rings (224 KB) cover the epilogue: the producers keep streaming the next item while it
// runs. The grid is <= the SM count with one CTA per SM (shared memory), so every CTA is
// resident and a finisher's wait ends; every wait is bounded. No multicast.

#include <algorithm>
#include <mutex>

#include "ckl_internal.h"
#include "ckl_ptx.cuh"

namespace ckl {
namespace grouped {

constexpr int BM = 256;                     // output columns per item
constexpr int HALF = 128;                   // the MMA's M (one accumulator)
constexpr int BN_MAX = 256;                 // rows per chunk (the MMA's N, max)
constexpr int BK = 64;                      // k per stage (one 128-byte swizzle row)
constexpr int XBOX = 32;                    // rows per TMA box of Xp
constexpr int WBOX_BYTES = 64 * BK * 2;     // 8 KB: 64 columns x 64 k
constexpr int W_STAGE = 4 * WBOX_BYTES;     // 32 KB
constexpr int X_STAGE = BN_MAX * BK * 2;    // 32 KB
constexpr int XBOX_BYTES = XBOX * BK * 2;   // 4 KB
constexpr int WSTAGES = 4;
constexpr int XSTAGES = 3;
constexpr int E_MAX = 256;
constexpr int NBARS = 2 * WSTAGES + 2 * XSTAGES + 3;
constexpr int SMEM = 1024 + WSTAGES * W_STAGE + XSTAGES * X_STAGE + NBARS * 8 + 16;
constexpr int EPI_WARP0 = 4;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = (EPI_WARP0 + EPI_WARPS) * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr size_t SLOT_FLOATS = (size_t)BN_MAX * BM;       // a partial tile, [rows][256 columns]
constexpr size_t FLAGS_BYTES = 1024;                      // room for 256 CTA flags

struct Args {
    __half* Y;
    const int* offsets;
    unsigned* flags;          // [gridDim.x] partial-tile flags, zero between launches
    float* slots;             // [gridDim.x][SLOT_FLOATS]
    unsigned* err;
    unsigned long long timeout_ns;
    int E, d, f, mtiles;      // mtiles = ceil(f / 256)
};

// One CTA's part of one item: k blocks [kb0, kb1) of item `item`.
struct Portion {
    long long item;
    int e, r0, n, mt, kb0, kb1, halves;
};

// First k block of CTA c's range.
__device__ __forceinline__ long long range_start(int c, long long Q, int G) {
    return (long long)((unsigned long long)c * (unsigned long long)Q / (unsigned long long)G);
}

// The portion that starts at global k block x (< end); cp = chunk prefix per expert.
__device__ __forceinline__ Portion portion_at(long long x, long long end, int nkb, const int* cp,
                                              const Args& a) {
    Portion p;
    p.item = x / nkb;
    p.kb0 = (int)(x - p.item * nkb);
    p.kb1 = (int)min((long long)nkb, p.kb0 + (end - x));
    const int j = (int)(p.item / a.mtiles);
    p.mt = (int)(p.item - (long long)j * a.mtiles);
    int lo = 0, hi = a.E;                  // cp[lo] <= j < cp[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (cp[mid] <= j) lo = mid;
        else hi = mid;
    }
    p.e = lo;
    const int k = j - cp[lo];
    const int base = __ldg(a.offsets + lo);
    p.r0 = base + k * BN_MAX;
    p.n = min(BN_MAX, __ldg(a.offsets + lo + 1) - base - k * BN_MAX);
    p.halves = p.mt * BM + HALF < a.f ? 2 : 1;
    return p;
}

// The next CTA >= w whose (non-empty) range starts inside the item that ends at global k block
// wend, i.e. the next writer of that item's partial tiles; G if none.
__device__ __forceinline__ int next_writer(int w, long long wend, long long Q, int G) {
    for (; w < G; w++) {
        const long long s0 = range_start(w, Q, G);
        if (s0 >= wend) return G;
        if (range_start(w + 1, Q, G) > s0) return w;
    }
    return G;
}

__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Barrier over the epilogue warps (named barrier 1) returning the AND of pred over them.
__device__ __forceinline__ bool epi_bar_and(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "n"(EPI_WARPS * 32)
        : "memory");
    return r != 0;
}

__global__ void __launch_bounds__(THREADS, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                    const Args a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* wring = align_ptr<1024>(smem_raw);           // 128-byte swizzle wants 1 KB alignment
    uint8_t* xring = wring + WSTAGES * W_STAGE;
    uint64_t* fullW = reinterpret_cast<uint64_t*>(xring + XSTAGES * X_STAGE);
    uint64_t* emptyW = fullW + WSTAGES;
    uint64_t* fullX = emptyW + WSTAGES;
    uint64_t* emptyX = fullX + XSTAGES;
    uint64_t* tfull = emptyX + XSTAGES;                   // accumulators ready (MMA -> epilogue)
    uint64_t* tempty = tfull + 1;                         // accumulators read (epilogue -> MMA)
    uint64_t* mma_done = tempty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    __shared__ int s_cp[E_MAX + 1];                       // chunk prefix per expert
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (warp == 0) {                                      // chunks per expert, exclusive scan
        int carry = 0;
        for (int e0 = 0; e0 < a.E; e0 += 32) {
            const int e = e0 + lane;
            const int ne = e < a.E ? __ldg(a.offsets + e + 1) - __ldg(a.offsets + e) : 0;
            const int c = (ne + BN_MAX - 1) / BN_MAX;
            int inc = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            if (e < a.E) s_cp[e] = carry + inc - c;
            carry += __shfl_sync(0xffffffffu, inc, 31);
        }
        if (lane == 0) s_cp[a.E] = carry;
    }
    if (threadIdx.x == 32) {
        for (int s = 0; s < WSTAGES; s++) {
            mbar_init(&fullW[s], 1);
            mbar_init(&emptyW[s], 1);
        }
        for (int s = 0; s < XSTAGES; s++) {
            mbar_init(&fullX[s], 1);
            mbar_init(&emptyX[s], 1);
        }
        mbar_init(tfull, 1);
        mbar_init(tempty, EPI_WARPS);
        mbar_init(mma_done, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
    }
    if (warp == 3) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint64_t deadline = globaltimer() + a.timeout_ns;
    const int nkb = a.d / BK;
    const int G = gridDim.x, c = blockIdx.x;
    const long long Q = (long long)s_cp[a.E] * a.mtiles * nkb;
    const long long begin = range_start(c, Q, G), end = range_start(c + 1, Q, G);

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ weights producer
        const uint64_t pol = policy_evict_first();       // read once
        unsigned g = 0;
        bool ok = true;
        for (long long x = begin; ok && x < end;) {
            const Portion p = portion_at(x, end, nkb, s_cp, a);
            for (int kb = p.kb0; kb < p.kb1; kb++, g++) {
                const int s = g % WSTAGES;
                if (g >= WSTAGES && !mbar_wait(&emptyW[s], ((g / WSTAGES) - 1) & 1, deadline, a.err)) {
                    ok = false;
                    break;
                }
                uint8_t* st = wring + (size_t)s * W_STAGE;
                mbar_arrive_expect_tx(&fullW[s], p.halves * 2 * WBOX_BYTES);
                const int wy = p.e * a.d + kb * BK;
                for (int b = 0; b < 2 * p.halves; b++)
                    tma_load_2d(st + b * WBOX_BYTES, &tmW, p.mt * BM + b * 64, wy, &fullW[s], pol);
            }
            x += p.kb1 - p.kb0;
        }
        // every issued copy must land before the CTA exits
        for (unsigned s = 0; s < WSTAGES && s < g; s++) {
            const unsigned last = s + ((g - 1 - s) / WSTAGES) * WSTAGES;
            mbar_wait(&fullW[s], (last / WSTAGES) & 1, deadline, a.err);
        }
    } else if (warp == 2 && lane == 0) {
        // ------------------------------------------------------------ rows producer
        const uint64_t pol = policy_evict_last();        // re-read by the other column tiles
        unsigned g = 0;
        bool ok = true;
        for (long long x = begin; ok && x < end;) {
            const Portion p = portion_at(x, end, nkb, s_cp, a);
            const int nbox = (p.n + XBOX - 1) / XBOX;
            for (int kb = p.kb0; kb < p.kb1; kb++, g++) {
                const int s = g % XSTAGES;
                if (g >= XSTAGES && !mbar_wait(&emptyX[s], ((g / XSTAGES) - 1) & 1, deadline, a.err)) {
                    ok = false;
                    break;
                }
                uint8_t* st = xring + (size_t)s * X_STAGE;
                mbar_arrive_expect_tx(&fullX[s], nbox * XBOX_BYTES);
                for (int b = 0; b < nbox; b++)
                    tma_load_2d(st + b * XBOX_BYTES, &tmX, kb * BK, p.r0 + b * XBOX, &fullX[s], pol);
            }
            x += p.kb1 - p.kb0;
        }
        for (unsigned s = 0; s < XSTAGES && s < g; s++) {
            const unsigned last = s + ((g - 1 - s) / XSTAGES) * XSTAGES;
            mbar_wait(&fullX[s], (last / XSTAGES) & 1, deadline, a.err);
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        unsigned g = 0, pidx = 0;
        bool ok = true;
        for (long long x = begin; ok && x < end;) {
            const Portion p = portion_at(x, end, nkb, s_cp, a);
            if (pidx > 0 && !mbar_wait(tempty, (pidx - 1) & 1, deadline, a.err)) break;
            tc_fence_after_sync();
            const uint32_t idesc = umma_idesc_f16(HALF, (p.n + 15) & ~15, /*A MN-major*/ true,
                                                  /*B K-major*/ false);
            for (int kb = p.kb0; kb < p.kb1; kb++, g++) {
                const int sw = g % WSTAGES, sx = g % XSTAGES;
                if (!mbar_wait(&fullW[sw], (g / WSTAGES) & 1, deadline, a.err) ||
                    !mbar_wait(&fullX[sx], (g / XSTAGES) & 1, deadline, a.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after_sync();
                const uint32_t wa = smem_u32(wring + (size_t)sw * W_STAGE);
                const uint32_t xa = smem_u32(xring + (size_t)sx * X_STAGE);
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++) {
                    // A: weights, MN-major: 64-column atoms 8 KB apart (LBO), 8-row k groups
                    //    1 KB apart (SBO); k step of 16 = two groups = 2 KB; the second half of
                    //    the columns starts two boxes (16 KB) in.
                    // B: rows, K-major: 8-row groups 1 KB apart (SBO); k step of 16 = 32 bytes
                    //    inside the swizzled 128-byte row.
                    const uint64_t bd = umma_desc_sw128(xa + kk * 32, 16, 1024);
                    const uint32_t acc = (kb > p.kb0 || kk > 0) ? 1u : 0u;
                    umma_f16(tmem, umma_desc_sw128(wa + kk * 2048, WBOX_BYTES, 1024), bd, idesc, acc);
                    if (p.halves == 2)
                        umma_f16(tmem + 256, umma_desc_sw128(wa + 2 * WBOX_BYTES + kk * 2048, WBOX_BYTES, 1024),
                                 bd, idesc, acc);
                }
                umma_commit(&emptyW[sw]);                 // stages free once these MMAs finish
                umma_commit(&emptyX[sx]);
            }
            if (!ok) break;
            umma_commit(tfull);                           // this portion's sums are complete
            x += p.kb1 - p.kb0;
            pidx++;
        }
        umma_commit(mma_done);                            // every issued MMA has finished
        mbar_wait(mma_done, 0, deadline, a.err);
    } else if (warp >= EPI_WARP0) {
        // ------------------------------------------------------------ epilogue (8 warps)
        const int ew = warp - EPI_WARP0;
        const int h = ew >> 2, q = warp & 3;              // column half; TMEM lane quarter
        const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)h * 256;
        const int lcol = h * HALF + q * 32 + lane;        // column inside the item
        unsigned pidx = 0;
        for (long long x = begin; x < end;) {
            const Portion p = portion_at(x, end, nkb, s_cp, a);
            bool ok = mbar_wait(tfull, pidx & 1, deadline, a.err);
            tc_fence_after_sync();
            const bool head = p.kb0 == 0, tail = p.kb1 == nkb;
            const bool active = h < p.halves;
            const int N = (p.n + 15) & ~15;
            long long wend = 0;                           // writers: CTAs c+1 .. while start < wend
            if (head && !tail) {
                wend = (p.item + 1) * nkb;
                if (ew == 0 && lane == 0) {
                    for (int w = next_writer(c + 1, wend, Q, G); ok && w < G;
                         w = next_writer(w + 1, wend, Q, G)) {
                        while (ld_acquire_gpu(a.flags + w) == 0u) {
                            if (globaltimer() > deadline) {
                                atomicOr(a.err, DEVERR_TIMEOUT);
                                ok = false;
                                break;
                            }
                            __nanosleep(32);
                        }
                    }
                }
            }
            if (!epi_bar_and(ok)) break;                  // uniform over the epilogue warps
            if (!head) {
                // a writer: this CTA's partial tile to its slot, then the flag
                float* slot = a.slots + (size_t)c * SLOT_FLOATS + lcol;
                for (int c0 = 0; c0 < N; c0 += 16) {
                    uint32_t v[16];
                    tmem_ld16(lane_addr + c0, v);
                    tmem_ld_wait();
                    if (active) {
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            if (c0 + i < p.n) __stcg(slot + (size_t)(c0 + i) * BM, __uint_as_float(v[i]));
                    }
                }
                __threadfence();
                epi_bar_and(true);
                if (ew == 0 && lane == 0) st_release_gpu(a.flags + c, 1u);
            } else {
                const int col = p.mt * BM + lcol;
                __half* yrow = a.Y + (size_t)p.r0 * a.f + col;
                for (int c0 = 0; c0 < N; c0 += 16) {
                    uint32_t v[16];
                    tmem_ld16(lane_addr + c0, v);
                    tmem_ld_wait();
                    float acc[16];
#pragma unroll
                    for (int i = 0; i < 16; i++) acc[i] = __uint_as_float(v[i]);
                    if (active) {
                        for (int w = next_writer(c + 1, wend, Q, G); w < G;
                             w = next_writer(w + 1, wend, Q, G)) {
                            const float* slot = a.slots + (size_t)w * SLOT_FLOATS + lcol;
#pragma unroll
                            for (int i = 0; i < 16; i++)
                                if (c0 + i < p.n) acc[i] += __ldcg(slot + (size_t)(c0 + i) * BM);
                        }
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            if (c0 + i < p.n) yrow[(size_t)(c0 + i) * a.f] = __float2half_rn(acc[i]);
                    }
                }
                if (wend && ew == 0 && lane == 0)
                    for (int w = next_writer(c + 1, wend, Q, G); w < G; w = next_writer(w + 1, wend, Q, G))
                        a.flags[w] = 0u;
            }
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty);
            x += p.kb1 - p.kb0;
            pidx++;
        }
    }
    __syncwarp();
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 3) tmem_dealloc(tmem, TMEM_COLS);
}

ckl_status setup_once(const DeviceInfo* di) {
    static ckl_status st[64];
    static std::once_flag once[64];
    std::call_once(once[di->device], [di] {
        st[di->device] = cuda_status(
            cudaFuncSetAttribute(reinterpret_cast<const void*>(grouped_gemm_kernel),
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM),
            "grouped gemm setup");
    });
    return st[di->device];
}

int grid_ctas(const DeviceInfo* di) { return std::min(di->sms, (int)(FLAGS_BYTES / sizeof(unsigned))); }

}  // namespace grouped
}  // namespace ckl

using namespace ckl;
using namespace ckl::grouped;

extern "C" {

size_t ckl_moe_grouped_gemm_workspace_size(void) {
    const DeviceInfo* di = device_info();
    if (!di) return SIZE_MAX;
    return FLAGS_BYTES + (size_t)grid_ctas(di) * SLOT_FLOATS * sizeof(float);
}

ckl_status ckl_moe_grouped_gemm(const void* Xp, const void* W, void* Yp, const int* offsets, int A,
                                int E, int d, int f, void* workspace, size_t workspace_bytes,
                                void* stream) {
    if (A < 0 || E <= 0 || E > E_MAX || d <= 0 || f <= 0)
        return fail(CKL_INVALID_ARG, "moe_grouped_gemm: A=%d E=%d d=%d f=%d", A, E, d, f);
    if (d % BK || f % HALF)
        return fail(CKL_UNSUPPORTED_SHAPE, "moe_grouped_gemm: d %% %d and f %% %d must be 0 (d=%d f=%d)",
                    BK, HALF, d, f);
    if ((long long)E * d > 0x7fffffffLL)
        return fail(CKL_UNSUPPORTED_SHAPE, "moe_grouped_gemm: E*d = %lld rows too many", (long long)E * d);
    if (A == 0) return CKL_OK;
    if (!Xp || !W || !Yp || !offsets) return fail(CKL_INVALID_ARG, "moe_grouped_gemm: NULL tensor");
    if (((uintptr_t)Xp | (uintptr_t)W) & 15)
        return fail(CKL_INVALID_ARG, "moe_grouped_gemm: Xp/W need 16-byte alignment");
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    const size_t need = ckl_moe_grouped_gemm_workspace_size();
    if (!workspace || workspace_bytes < need)
        return fail(CKL_WORKSPACE_TOO_SMALL, "moe_grouped_gemm needs %zu workspace bytes, got %zu", need,
                    workspace_bytes);
    if ((uintptr_t)workspace & 15) return fail(CKL_INVALID_ARG, "moe_grouped_gemm: workspace alignment");
    ckl_status st = setup_once(di);
    if (st != CKL_OK) return st;

    CUtensorMap tmW, tmX;
    {   // W as a 2-D [E*d rows][f columns] matrix; boxes of 64 columns x 64 k rows
        const uint64_t dims[2] = {(uint64_t)f, (uint64_t)E * d};
        const uint64_t strides[1] = {(uint64_t)f * 2};
        const uint32_t box[2] = {64, BK};
        st = encode_tiled(&tmW, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(W), dims, strides,
                          box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (st != CKL_OK) return st;
    }
    {   // Xp [A rows][d]; boxes of 64 k x 32 rows
        const uint64_t dims[2] = {(uint64_t)d, (uint64_t)A};
        const uint64_t strides[1] = {(uint64_t)d * 2};
        const uint32_t box[2] = {BK, XBOX};
        st = encode_tiled(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(Xp), dims, strides,
                          box, CU_TENSOR_MAP_SWIZZLE_128B);
        if (st != CKL_OK) return st;
    }
    Args a;
    a.Y = static_cast<__half*>(Yp);
    a.offsets = offsets;
    a.flags = static_cast<unsigned*>(workspace);
    a.slots = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + FLAGS_BYTES);
    a.err = di->err_word;
    a.timeout_ns = spin_timeout_ns();
    a.E = E;
    a.d = d;
    a.f = f;
    a.mtiles = (f + BM - 1) / BM;
    // upper bound of the k blocks (chunks <= ceil(A/256) + min(E, A)); no CTA without work
    const long long qmax = ((long long)(A + BN_MAX - 1) / BN_MAX + std::min(E, A)) * a.mtiles * (d / BK);
    const int grid = (int)std::min<long long>(grid_ctas(di), qmax);
    void* args[] = {&tmW, &tmX, &a};
    CKL_CUDA_TRY(cudaLaunchKernel(reinterpret_cast<const void*>(grouped_gemm_kernel), dim3((unsigned)grid),
                                  dim3(THREADS), args, SMEM, (cudaStream_t)stream));
    return CKL_OK;
}

}  // extern "C"
