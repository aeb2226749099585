// moe_grouped.cu -- dense grouped fp16 expert GEMM on the 5th-generation tensor cores.
//
// Replaces moe_grouped_gemm<TileCfg> (02_moe_grouped_gemm.cu:86-186), the path for batches
// with tens of tokens or more per expert (prefill-sized MoE): Yp[r] = Xp[r] . W[e] for the
// rows r of every expert e (rows [offsets[e], offsets[e+1]) of the expert-sorted Xp), fp16
// in, fp32 accumulate, fp16 out, in one launch with a device-side schedule.
//
// At the reference's shapes the weight stream bounds the job (T=512, E=8, top-2, d=4096,
// f=14336: 940 MB of fp16 weights for ~128 tokens per expert, 120 GFLOP), so every weight
// tile is read from HBM once: a CTA owns (expert, 128 output columns, up to 256 of the
// expert's rows) and runs tcgen05.mma with the weights as the M=128 operand (swap-AB) and
// the expert's rows as the N operand (N = rows rounded up to 16, so a 48-row expert wastes
// nothing on padding), accumulating in tensor memory:
//
//   warp 0 lane 0   TMA producer: per 64-wide k block, the weight tile (two 64x64 boxes of
//                   W[e], MN-major, 128-byte swizzle) and the rows (32-row boxes of Xp,
//                   K-major, 128-byte swizzle) into a 4-stage ring (full/empty mbarriers)
//   warp 1 lane 0   MMA issuer: 4 x tcgen05.mma (M=128, N, K=16) per stage, fp32 D in TMEM;
//                   tcgen05.commit frees the stage when its MMAs complete
//   warps 0-3       epilogue: tcgen05.ld of each warp's 32 TMEM lanes (= output columns),
//                   fp16 rows to Yp
//
// Work item w = (chunk j, column tile mt): chunk j is the j-th run of <= 256 rows in expert
// order (an expert with n rows has ceil(n / 256) chunks), found on the device from the
// offsets; the grid is an upper bound (ceil(A/256) + min(E, A) chunks) and surplus CTAs exit
// (no host sync, 02:95-105, 234-235). No multicast; every wait bounded.

#include <algorithm>
#include <mutex>

#include "ckl_internal.h"
#include "ckl_ptx.cuh"

namespace ckl {
namespace grouped {

constexpr int BM = 128;                 // output columns per CTA (the MMA's M)
constexpr int BN_MAX = 256;             // rows per chunk (the MMA's N, max)
constexpr int BK = 64;                  // k per stage (one 128-byte swizzle row)
constexpr int XBOX = 32;                // rows per TMA box of Xp
constexpr int W_BYTES = BM * BK * 2;    // 16 KB: two 64-column boxes of 64 k rows
constexpr int XBOX_BYTES = XBOX * BK * 2;   // 4 KB
constexpr int STAGES = 4;
constexpr int X_BYTES = BN_MAX * BK * 2;   // 32 KB
constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + 256;
constexpr int THREADS = 128;
constexpr uint32_t TMEM_COLS = 256;

struct Args {
    __half* Y;
    const int* offsets;
    unsigned* err;
    unsigned long long timeout_ns;
    int E, d, f, A, mtiles;
};

// Chunk j -> (expert, first row, rows); false if j is past the last chunk. Warp-collective.
__device__ __forceinline__ bool find_chunk(const int* offsets, int E, int j, int* e_out, int* r0,
                                           int* n) {
    const int lane = threadIdx.x & 31;
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const int ne = e < E ? __ldg(offsets + e + 1) - __ldg(offsets + e) : 0;
        const int c = (ne + BN_MAX - 1) / BN_MAX;
        int inc = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
        }
        const int excl = carry + inc - c;
        const unsigned hit = __ballot_sync(0xffffffffu, c > 0 && excl <= j && j < excl + c);
        if (hit) {
            const int src = __ffs(hit) - 1;
            const int he = __shfl_sync(0xffffffffu, e, src);
            const int hx = __shfl_sync(0xffffffffu, excl, src);
            const int hn = __shfl_sync(0xffffffffu, ne, src);
            const int k = j - hx;
            *e_out = he;
            *r0 = __ldg(offsets + he) + k * BN_MAX;
            *n = min(BN_MAX, hn - k * BN_MAX);
            return true;
        }
        carry += __shfl_sync(0xffffffffu, inc, 31);
    }
    return false;
}

__global__ void __launch_bounds__(THREADS, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                    const Args a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = align_ptr<1024>(smem_raw);            // 128-byte swizzle wants 1 KB alignment
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + STAGES * STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* done = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    __shared__ int s_item[3];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int mt = blockIdx.x % a.mtiles, j = blockIdx.x / a.mtiles;
    if (warp == 0) {
        int e = -1, r0 = 0, n = 0;
        if (!find_chunk(a.offsets, a.E, j, &e, &r0, &n)) e = -1;
        if (lane == 0) {
            s_item[0] = e;
            s_item[1] = r0;
            s_item[2] = n;
        }
    }
    __syncthreads();
    const int e = s_item[0], r0 = s_item[1], nrows = s_item[2];
    if (e < 0) return;                                    // surplus CTA of the upper bound
    const int nbox = (nrows + XBOX - 1) / XBOX;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint64_t deadline = globaltimer() + a.timeout_ns;
    const int nkb = a.d / BK;
    const int N = (nrows + 15) & ~15;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA producer
        const uint64_t wpol = policy_evict_first();      // weights: read once
        const uint64_t xpol = policy_evict_last();       // rows: re-read by the other column tiles
        const uint32_t tx = W_BYTES + nbox * XBOX_BYTES;
        int issued = 0;
        for (int kb = 0; kb < nkb; kb++) {
            const int s = kb % STAGES;
            if (kb >= STAGES && !mbar_wait(&empty[s], ((kb / STAGES) - 1) & 1, deadline, a.err)) break;
            uint8_t* st = ring + (size_t)s * STAGE_BYTES;
            mbar_arrive_expect_tx(&full[s], tx);
            const int wy = e * a.d + kb * BK;
            tma_load_2d(st, &tmW, mt * BM, wy, &full[s], wpol);
            tma_load_2d(st + W_BYTES / 2, &tmW, mt * BM + 64, wy, &full[s], wpol);
            for (int b = 0; b < nbox; b++)
                tma_load_2d(st + W_BYTES + b * XBOX_BYTES, &tmX, kb * BK, r0 + b * XBOX, &full[s], xpol);
            issued = kb + 1;
        }
        // every issued copy must land before the CTA exits
        for (int s = 0; s < STAGES && s < issued; s++) {
            const int last = s + ((issued - 1 - s) / STAGES) * STAGES;
            mbar_wait(&full[s], (last / STAGES) & 1, deadline, a.err);
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        const uint32_t idesc = umma_idesc_f16(BM, N, /*A MN-major*/ true, /*B K-major*/ false);
        for (int kb = 0; kb < nkb; kb++) {
            const int s = kb % STAGES;
            if (!mbar_wait(&full[s], (kb / STAGES) & 1, deadline, a.err)) break;
            tc_fence_after_sync();
            const uint32_t wa = smem_u32(ring + (size_t)s * STAGE_BYTES);
            const uint32_t xa = wa + W_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; kk++) {
                // A: weights, MN-major: 64-column atoms 8 KB apart (LBO), 8-row k groups 1 KB
                //    apart (SBO); k step of 16 = two groups = 2 KB.
                // B: rows, K-major: 8-row groups 1 KB apart (SBO); k step of 16 = 32 bytes
                //    inside the swizzled 128-byte row.
                const uint64_t ad = umma_desc_sw128(wa + kk * 2048, W_BYTES / 2, 1024);
                const uint64_t bd = umma_desc_sw128(xa + kk * 32, 16, 1024);
                umma_f16(tmem, ad, bd, idesc, (kb | kk) != 0);
            }
            umma_commit(&empty[s]);                       // stage free once these MMAs finish
        }
        umma_commit(done);                                // all issued MMAs finished
    }
    __syncwarp();

    // ---------------------------------------------------------------- epilogue (4 warps)
    const bool ok = mbar_wait(done, 0, deadline, a.err);
    tc_fence_after_sync();
    if (__all_sync(0xffffffffu, ok)) {
        const int col = mt * BM + warp * 32 + lane;       // this thread's TMEM lane
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
        __half* yrow = a.Y + (size_t)r0 * a.f + col;
        for (int c0 = 0; c0 < N; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(lane_addr + c0, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; i++)
                if (c0 + i < nrows) yrow[(size_t)(c0 + i) * a.f] = __float2half_rn(__uint_as_float(v[i]));
        }
    }
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
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

}  // namespace grouped
}  // namespace ckl

using namespace ckl;
using namespace ckl::grouped;

extern "C" {

ckl_status ckl_moe_grouped_gemm(const void* Xp, const void* W, void* Yp, const int* offsets, int A,
                                int E, int d, int f, void* stream) {
    if (A < 0 || E <= 0 || E > 256 || d <= 0 || f <= 0)
        return fail(CKL_INVALID_ARG, "moe_grouped_gemm: A=%d E=%d d=%d f=%d", A, E, d, f);
    if (d % BK || f % BM)
        return fail(CKL_UNSUPPORTED_SHAPE, "moe_grouped_gemm: d %% %d and f %% %d must be 0 (d=%d f=%d)",
                    BK, BM, d, f);
    if (A == 0) return CKL_OK;
    if (!Xp || !W || !Yp || !offsets) return fail(CKL_INVALID_ARG, "moe_grouped_gemm: NULL tensor");
    if (((uintptr_t)Xp | (uintptr_t)W) & 15)
        return fail(CKL_INVALID_ARG, "moe_grouped_gemm: Xp/W need 16-byte alignment");
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
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
    a.err = di->err_word;
    a.timeout_ns = spin_timeout_ns();
    a.E = E;
    a.d = d;
    a.f = f;
    a.A = A;
    a.mtiles = f / BM;
    const long long chunks = (A + BN_MAX - 1) / BN_MAX + std::min(E, A);
    const long long grid = chunks * a.mtiles;
    if (grid > 0x7fffffffLL) return fail(CKL_UNSUPPORTED_SHAPE, "moe_grouped_gemm: grid too large");
    void* args[] = {&tmW, &tmX, &a};
    CKL_CUDA_TRY(cudaLaunchKernel(reinterpret_cast<const void*>(grouped_gemm_kernel), dim3((unsigned)grid),
                                  dim3(THREADS), args, SMEM, (cudaStream_t)stream));
    return CKL_OK;
}

}  // extern "C"
