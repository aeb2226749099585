// moe_layer.cu -- MoE routing, permutation, combine and the full SwiGLU decode layer.
//
// Replaces router_topk / moe_count / moe_scan(_offsets) / moe_permute / moe_combine
// (common/moe.cuh:23-119, 02_moe_grouped_gemm.cu:71-82, 03_moe_wq_decode.cu:271-276) and
// MoeDecode (03_moe_wq_decode.cu:350-391).
//
// Routing is one small CTA: the decode batch is at most a few hundred (token, slot)
// assignments, so a single block computes top-k, counts, the scan and the permutation
// without any atomics on the slot order. Unlike the reference's atomicAdd slot allocation
// (common/moe.cuh:86), the slot of assignment i = t*k + j is its stable rank by
// (expert, token, slot): offsets[e] + #{i' < i : ids[i'] = e}, so inv_perm, the expert row
// order and every later result are bit-identical from run to run. Ties in top-k go to the
// lower expert id, as in the reference (common/moe.cuh:55-59).
//
// The full layer (ckl_moe_layer) never materialises the permuted activations: the expert
// GEMM gathers token rows through row_src, the SwiGLU intermediate h (fp16) is written in
// expert order, the down projection writes fp32 rows, and the combine is a fixed-order
// gather. No step reads a device value back to the host.

#include <algorithm>
#include <mutex>

#include "ckl_internal.h"
#include "ckl_ptx.cuh"
#include "moe_internal.h"

namespace ckl {
namespace moe {

constexpr int MAX_E = 256;
constexpr int MAX_K = 8;
constexpr int ROUTE_THREADS = 512;
constexpr int ROUTE_ONE_CTA = 16;   // batches up to this many tokens route in one CTA
constexpr int MAX_A = 4096;      // assignments one routing block handles (T * k)
constexpr int ROUTE_SMEM_LOGITS = 6144;   // logits staged in shared memory (24 KB; with the
                                          // 18 KB of static arrays below the 48 KB default)

// Top-k of one token by one warp (lane l holds experts l, l+32, ... as order-preserving keys
// of their logits, -0 folded into +0 so equal logits tie): k rounds of a warp argmax (max key
// by one reduction, then the lowest id holding it by another), the winner's key retired. This
// is the reference's order: larger value first, ties to the lower id (common/moe.cuh:55-59),
// and round r fills slot r. Softmax is monotonic, so top-k of the logits is top-k of p; the
// weights are the renormalised p: w_j = exp(l_j - l_max) / sum_j' exp(l_j' - l_max)
// (= p_j / sum p, common/moe.cuh:64-70). lg = the token's E logits (shared or global
// memory); writes ids/wts of the token's k slots; s_ids / s_cnt (nullable) receive the ids
// and the histogram.
__device__ __forceinline__ void topk_token(const float* lg, int E, int k, int lane,
                                           int* __restrict__ ids, float* __restrict__ wts,
                                           int* s_ids, int* s_cnt) {
    const int nj = (E + 31) >> 5;                          // experts per lane (<= MAX_E / 32)
    uint32_t key[MAX_E / 32];
#pragma unroll
    for (int j = 0; j < MAX_E / 32; j++) {
        const int e = lane + 32 * j;
        uint32_t u = 0;                                    // below every logit's key
        if (j < nj && e < E) {
            uint32_t bits = __float_as_uint(lg[e]);
            if (bits == 0x80000000u) bits = 0u;
            u = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
        }
        key[j] = u;
    }
    float v0 = 0.f, vmine = 0.f;                           // round 0's logit, round lane's logit
    for (int r = 0; r < k; r++) {
        uint32_t bk = key[0];
        int bj = 0;
#pragma unroll
        for (int j = 1; j < MAX_E / 32; j++) {
            if (j >= nj) break;
            if (key[j] > bk) { bk = key[j]; bj = j; }       // ties keep the lower id
        }
        const uint32_t m = __reduce_max_sync(0xffffffffu, bk);
        const int e = (int)__reduce_min_sync(0xffffffffu, bk == m ? (uint32_t)(lane + 32 * bj) : 0xffffffffu);
#pragma unroll
        for (int j = 0; j < MAX_E / 32; j++)
            if (lane + 32 * j == e) key[j] = 0u;
        const float v = lg[e];
        if (r == 0) v0 = v;
        if (lane == r) vmine = v;
        if (lane == 0) {
            ids[r] = e;
            if (s_ids) s_ids[r] = e;
            if (s_cnt) atomicAdd(&s_cnt[e], 1);             // integer histogram: order-free
        }
    }
    // weights renormalised over the chosen k: lane r < k owns slot r
    float p = 0.f;
    if (lane < k) p = expf(vmine - v0);
    float den = p;
#pragma unroll
    for (int o = 1; o < MAX_K; o <<= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    if (lane < k) wts[lane] = p * __frcp_rn(den);
}

// Counts, offsets (and tile offsets) from the histogram s_cnt, by warp 0: exclusive scan over
// E, 32 at a time. Writes s_off[0..E] too.
__device__ __forceinline__ void scan_offsets(const int* s_cnt, int* s_off, int E, int* __restrict__ counts,
                                             int* __restrict__ offsets, int bm, int* __restrict__ tiles) {
    const int lane = threadIdx.x & 31;
    int carry = 0, tcarry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const int c = e < E ? s_cnt[e] : 0;
        const int tcount = tiles && e < E ? (c + bm - 1) / bm : 0;
        int inc = c, tinc = tcount;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, o);
            const int ty = __shfl_up_sync(0xffffffffu, tinc, o);
            if (lane >= o) { inc += y; tinc += ty; }
        }
        if (e < E) {
            s_off[e] = carry + inc - c;
            offsets[e] = carry + inc - c;
            counts[e] = c;
            if (tiles) tiles[e] = tcarry + tinc - tcount;
        }
        carry += __shfl_sync(0xffffffffu, inc, 31);
        tcarry += __shfl_sync(0xffffffffu, tinc, 31);
    }
    if (lane == 0) {
        s_off[E] = carry;
        offsets[E] = carry;
        if (tiles) tiles[E] = tcarry;
    }
}

// Stable rank, thread per assignment: slot = offsets[e] + #{i' < i : ids[i'] = e}.
__device__ __forceinline__ void rank_slots(const int* s_ids, const int* s_off, int A, int k,
                                           int* __restrict__ inv_perm, int* __restrict__ row_src) {
    for (int i = threadIdx.x; i < A; i += blockDim.x) {
        const int e = s_ids[i];
        int r = 0, j = 0;
        const int4* s4 = reinterpret_cast<const int4*>(s_ids);
#pragma unroll 4
        for (; j + 4 <= i; j += 4) {
            const int4 q = s4[j >> 2];
            r += (q.x == e) + (q.y == e) + (q.z == e) + (q.w == e);
        }
        for (; j < i; j++) r += s_ids[j] == e;
        const int pos = s_off[e] + r;
        inv_perm[i] = pos;
        if (row_src) row_src[pos] = i / k;
    }
}

// grid = 1, block = ROUTE_THREADS (16 warps), for batches of up to ROUTE_ONE_CTA tokens:
//  1. logits staged in shared memory (one coalesced pass); top-k, one warp per token;
//  2. integer histogram (order-free), exclusive scan -> offsets (and tile offsets);
//  3. stable rank.
__global__ void __launch_bounds__(ROUTE_THREADS)
route_kernel(const float* __restrict__ logits, int T, int E, int k, int* __restrict__ ids,
             float* __restrict__ wts, int* __restrict__ counts, int* __restrict__ offsets,
             int* __restrict__ inv_perm, int* __restrict__ row_src, int bm, int* __restrict__ tiles) {
    __shared__ __align__(16) int s_ids[MAX_A];
    __shared__ int s_cnt[MAX_E];
    __shared__ int s_off[MAX_E + 1];
    extern __shared__ float s_lg[];                           // [T][E+1] logits when they fit
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
    pdl_wait();                       // launched early behind the previous kernel: its logits
    pdl_trigger();                    // the expert GEMM may launch; it waits for our results
    const bool staged = T * (E + 1) <= ROUTE_SMEM_LOGITS;    // the launch sized s_lg for this
    const int lg_stride = E + 1;
    if (staged)
        for (int i = threadIdx.x; i < T * E; i += blockDim.x)
            s_lg[(i / E) * lg_stride + i % E] = __ldg(logits + i);
    __syncthreads();
    for (int t = warp; t < T; t += blockDim.x >> 5) {
        const float* lg = staged ? s_lg + (size_t)t * lg_stride : logits + (size_t)t * E;
        topk_token(lg, E, k, lane, ids + t * k, wts + t * k, s_ids + t * k, s_cnt);
        __syncwarp();
    }
    __syncthreads();
    if (warp == 0) scan_offsets(s_cnt, s_off, E, counts, offsets, bm, tiles);
    __syncthreads();
    rank_slots(s_ids, s_off, T * k, k, inv_perm, row_src);
}

// Larger batches in two launches, so the top-k of all tokens runs on many SMs at once:
// route_topk_kernel (one warp per token, ROUTE_THREADS / 32 tokens per CTA) writes ids and
// wts; route_rank_kernel (one CTA, launched behind it with PDL) builds the histogram from
// the ids and runs the same scan and stable rank.
__global__ void __launch_bounds__(ROUTE_THREADS)
route_topk_kernel(const float* __restrict__ logits, int T, int E, int k, int* __restrict__ ids,
                  float* __restrict__ wts) {
    pdl_wait();                       // launched early behind the previous kernel: its logits
    pdl_trigger();                    // the rank kernel may launch; it waits for our results
    const int t = blockIdx.x * (ROUTE_THREADS / 32) + (threadIdx.x >> 5);
    if (t < T) topk_token(logits + (size_t)t * E, E, k, threadIdx.x & 31, ids + t * k, wts + t * k,
                          nullptr, nullptr);
}

__global__ void __launch_bounds__(ROUTE_THREADS)
route_rank_kernel(const int* __restrict__ ids, int T, int E, int k, int* __restrict__ counts,
                  int* __restrict__ offsets, int* __restrict__ inv_perm, int* __restrict__ row_src,
                  int bm, int* __restrict__ tiles) {
    __shared__ __align__(16) int s_ids[MAX_A];
    __shared__ int s_cnt[MAX_E];
    __shared__ int s_off[MAX_E + 1];
    const int A = T * k;
    for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
    pdl_wait();                       // the top-k kernel's ids
    pdl_trigger();                    // the expert GEMM may launch; it waits for our results
    __syncthreads();
    for (int i = threadIdx.x; i < A; i += blockDim.x) {
        const int e = ids[i];
        s_ids[i] = e;
        atomicAdd(&s_cnt[e], 1);
    }
    __syncthreads();
    if ((threadIdx.x >> 5) == 0) scan_offsets(s_cnt, s_off, E, counts, offsets, bm, tiles);
    __syncthreads();
    rank_slots(s_ids, s_off, A, k, inv_perm, row_src);
}

// Xp[inv_perm[i]] = X[i / k] (the reference's moe_permute copy, common/moe.cuh:90-92).
__global__ void permute_rows_kernel(const __half* __restrict__ X, const int* __restrict__ inv_perm,
                                    __half* __restrict__ Xp, int k, int d) {
    const int i = blockIdx.x;
    const int pos = __ldg(inv_perm + i);
    const uint4* src = reinterpret_cast<const uint4*>(X + (size_t)(i / k) * d);
    uint4* dst = reinterpret_cast<uint4*>(Xp + (size_t)pos * d);
    for (int c = threadIdx.x; c < d / 8; c += blockDim.x) dst[c] = __ldg(src + c);
}

// out[t] = sum_{j<k} wts[t][j] * Y[inv_perm[t*k+j]] in fixed j order, fp32 accumulate
// (common/moe.cuh:97-119). Y is fp16 or fp32; 8 columns per thread.
template <bool F32>
__global__ void combine_kernel(const void* __restrict__ Y, const int* __restrict__ inv_perm,
                               const float* __restrict__ wts, __half* __restrict__ out, int k, int f) {
    const int t = blockIdx.x;
    // The k (row, weight) pairs first, so the row loads below do not wait on them one by one.
    // They come from the routing, which completed before the kernel we wait for was launched
    // (the layer's chain; a standalone call is an ordinary launch): read them from L2 before
    // the wait, so that only the rows are left for after it.
    int pos_j[MAX_K];
    float w_j[MAX_K];
#pragma unroll
    for (int j = 0; j < MAX_K; j++) {
        pos_j[j] = j < k ? __ldcg(inv_perm + t * k + j) : 0;
        w_j[j] = j < k ? __ldcg(wts + t * k + j) : 0.f;
    }
    pdl_wait();                       // the rows Y
    pdl_trigger();                    // the next kernel (the next layer's routing) may launch
    for (int c = threadIdx.x; c < f / 8; c += blockDim.x) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < MAX_K; j++) {
            if (j >= k) break;
            const int pos = pos_j[j];
            const float w = w_j[j];
            if (F32) {
                const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(Y) + (size_t)pos * f) + 2 * c;
                const float4 v0 = __ldg(src), v1 = __ldg(src + 1);
                acc[0] += w * v0.x; acc[1] += w * v0.y; acc[2] += w * v0.z; acc[3] += w * v0.w;
                acc[4] += w * v1.x; acc[5] += w * v1.y; acc[6] += w * v1.z; acc[7] += w * v1.w;
            } else {
                const uint4 raw = __ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(Y) + (size_t)pos * f) + c);
                const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float2 v = __half22float2(h[q]);
                    acc[2 * q] += w * v.x;
                    acc[2 * q + 1] += w * v.y;
                }
            }
        }
        __align__(16) __half2 o[4];
#pragma unroll
        for (int q = 0; q < 4; q++) o[q] = __floats2half2_rn(acc[2 * q], acc[2 * q + 1]);
        reinterpret_cast<uint4*>(out + (size_t)t * f)[c] = *reinterpret_cast<uint4*>(o);
    }
}

inline size_t route_smem(int T, int E) {
    const size_t lgs = (size_t)T * (E + 1) <= ROUTE_SMEM_LOGITS ? (size_t)T * (E + 1) : 0;
    return lgs * sizeof(float);
}

// Opt the routing kernel into up to 64 KB of dynamic shared memory, once per device.
ckl_status route_setup() {
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    static ckl_status st[64];
    static std::once_flag once[64];
    std::call_once(once[di->device], [di] {
        const cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(route_kernel),
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   64 * 1024);
        st[di->device] = cuda_status(e, "routing kernel setup");
    });
    return st[di->device];
}

// The routing launches: one CTA up to ROUTE_ONE_CTA tokens, else top-k over many CTAs then
// the rank CTA (PDL).
ckl_status launch_route(const float* logits, int T, int E, int k, int* ids, float* wts,
                        int* counts, int* offsets, int* inv_perm, int* row_src, int bm, int* tiles,
                        cudaStream_t s) {
    ckl_status st = route_setup();
    if (st != CKL_OK) return st;
    // both routing launches may start behind the previous kernel of the stream (programmatic
    // dependent launch) and wait for it before reading anything
    if (T <= ROUTE_ONE_CTA) {
        void* args[] = {&logits, &T, &E, &k, &ids, &wts, &counts, &offsets, &inv_perm, &row_src,
                        &bm, &tiles};
        CKL_CUDA_TRY(launch(reinterpret_cast<const void*>(route_kernel), dim3(1), dim3(ROUTE_THREADS),
                            route_smem(T, E), s, args, true));
        return CKL_OK;
    }
    const int per = ROUTE_THREADS / 32;
    void* targs[] = {&logits, &T, &E, &k, &ids, &wts};
    CKL_CUDA_TRY(launch(reinterpret_cast<const void*>(route_topk_kernel), dim3((T + per - 1) / per),
                        dim3(ROUTE_THREADS), 0, s, targs, true));
    const int* idsc = ids;
    void* args[] = {&idsc, &T, &E, &k, &counts, &offsets, &inv_perm, &row_src, &bm, &tiles};
    CKL_CUDA_TRY(launch(reinterpret_cast<const void*>(route_rank_kernel), dim3(1), dim3(ROUTE_THREADS),
                        0, s, args, true));
    return CKL_OK;
}

// Routing of T tokens (T may be 0: counts and offsets are then all zero).
ckl_status route_tokens(const float* logits, int T, int E, int k, int* ids, float* wts,
                        int* counts, int* offsets, int* inv_perm, int* row_src, cudaStream_t s) {
    return launch_route(logits, T, E, k, ids, wts, counts, offsets, inv_perm, row_src, 1, nullptr, s);
}

ckl_status check_route(int T, int E, int k) {
    if (T < 0 || E <= 0 || E > MAX_E || k <= 0 || k > MAX_K || k > E)
        return fail(CKL_UNSUPPORTED_SHAPE, "routing: T=%d E=%d k=%d (E<=256, k<=8, k<=E)", T, E, k);
    if ((long long)T * k > MAX_A || T > 1024)
        return fail(CKL_UNSUPPORTED_SHAPE, "routing: T=%d, T*k=%lld (T <= 1024, T*k <= %d)", T,
                    (long long)T * k, MAX_A);
    return CKL_OK;
}

// Workspace layout of ckl_moe_layer (256-byte aligned pieces).
struct LayerWs {
    size_t ids, wts, counts, offsets, inv_perm, row_src, h, y, split, total;
};
LayerWs layer_ws(int T, int E, int k, int d, int F, size_t split_bytes) {
    LayerWs w{};
    const size_t A = (size_t)T * k;
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t r = o; o += align_up(std::max<size_t>(bytes, 1), 256); return r; };
    w.ids = take(A * 4);
    w.wts = take(A * 4);
    w.counts = take((size_t)E * 4);
    w.offsets = take((size_t)(E + 1) * 4);
    w.inv_perm = take(A * 4);
    w.row_src = take(A * 4);
    w.h = take(A * F * 2);
    w.y = take(A * d * 4);
    w.split = take(split_bytes);
    w.total = o;
    return w;
}

}  // namespace moe
}  // namespace ckl

using namespace ckl;
using namespace ckl::moe;

extern "C" {

ckl_status ckl_moe_route_permute(const float* logits, const void* X, int T, int E, int k, int d,
                                 int* ids, float* wts, int* counts, int* offsets, int* inv_perm,
                                 void* Xp, int bm, int* tiles, void* stream) {
    ckl_status st = check_route(T, E, k);
    if (st != CKL_OK) return st;
    if (T == 0) return CKL_OK;
    if (!logits || !ids || !wts || !counts || !offsets || !inv_perm)
        return fail(CKL_INVALID_ARG, "moe_route_permute: NULL output");
    if (tiles && bm <= 0) return fail(CKL_INVALID_ARG, "moe_route_permute: bm must be > 0");
    if (Xp && (!X || d <= 0 || d % 8 || ((uintptr_t)X | (uintptr_t)Xp) & 15))
        return fail(CKL_INVALID_ARG, "moe_route_permute: X/Xp need 16-byte alignment, d%%8==0");
    const cudaStream_t s = (cudaStream_t)stream;
    st = launch_route(logits, T, E, k, ids, wts, counts, offsets, inv_perm, nullptr, bm, tiles, s);
    if (st != CKL_OK) return st;
    if (Xp) {
        permute_rows_kernel<<<T * k, 128, 0, s>>>(static_cast<const __half*>(X), inv_perm,
                                                  static_cast<__half*>(Xp), k, d);
        CKL_CUDA_TRY(cudaGetLastError());
    }
    return CKL_OK;
}

ckl_status ckl_moe_combine(const void* Yp, int y_f32, const int* inv_perm, const float* wts,
                           void* out, int T, int k, int f, void* stream) {
    if (T < 0 || k <= 0 || f <= 0 || f % 8) return fail(CKL_INVALID_ARG, "moe_combine: shape");
    if (T == 0) return CKL_OK;
    if (!Yp || !inv_perm || !wts || !out) return fail(CKL_INVALID_ARG, "moe_combine: NULL");
    if (((uintptr_t)Yp | (uintptr_t)out) & 15) return fail(CKL_INVALID_ARG, "moe_combine: alignment");
    const cudaStream_t s = (cudaStream_t)stream;
    if (y_f32)
        combine_kernel<true><<<T, 256, 0, s>>>(Yp, inv_perm, wts, static_cast<__half*>(out), k, f);
    else
        combine_kernel<false><<<T, 256, 0, s>>>(Yp, inv_perm, wts, static_cast<__half*>(out), k, f);
    CKL_CUDA_TRY(cudaGetLastError());
    return CKL_OK;
}

size_t ckl_moe_layer_workspace_size(int T, int k, const ckl_moe_weights* gate,
                                    const ckl_moe_weights* down) {
    if (!gate || !down || T <= 0) return 0;
    const int A = T * k;
    const size_t s1 = ckl_moe_gemm_workspace_size(gate, A, 1, 0);
    const size_t s2 = ckl_moe_gemm_workspace_size(down, A, 0, 0);
    return layer_ws(T, gate->E, k, down->N, gate->N, std::max(s1, s2)).total;
}

ckl_status ckl_moe_layer(const float* logits, const void* X, int T, int k,
                         const ckl_moe_weights* gate, const ckl_moe_weights* up,
                         const ckl_moe_weights* down, void* out, int* ids_out, float* wts_out,
                         void* workspace, size_t workspace_bytes, void* stream) {
    if (!gate || !up || !down) return fail(CKL_INVALID_ARG, "moe_layer: NULL weights");
    const int E = gate->E, d = gate->K, F = gate->N;
    ckl_status st = check_route(T, E, k);
    if (st != CKL_OK) return st;
    if (down->E != E || down->K != F || down->N != d)
        return fail(CKL_INVALID_ARG, "moe_layer: down must be [E][F=%d][d=%d]", F, d);
    if (T == 0) return CKL_OK;
    if (!logits || !X || !out) return fail(CKL_INVALID_ARG, "moe_layer: NULL tensor");
    const int A = T * k;
    const size_t s1 = ckl_moe_gemm_workspace_size(gate, A, 1, 0);
    const size_t s2 = ckl_moe_gemm_workspace_size(down, A, 0, 0);
    const LayerWs L = layer_ws(T, E, k, d, F, std::max(s1, s2));
    if (!workspace || workspace_bytes < L.total)
        return fail(CKL_WORKSPACE_TOO_SMALL, "moe_layer needs %zu workspace bytes, got %zu", L.total,
                    workspace_bytes);
    if ((uintptr_t)workspace & 255) return fail(CKL_INVALID_ARG, "workspace must be 256-byte aligned");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int* ids = ids_out ? ids_out : reinterpret_cast<int*>(ws + L.ids);
    float* wts = wts_out ? wts_out : reinterpret_cast<float*>(ws + L.wts);
    int* counts = reinterpret_cast<int*>(ws + L.counts);
    int* offsets = reinterpret_cast<int*>(ws + L.offsets);
    int* inv_perm = reinterpret_cast<int*>(ws + L.inv_perm);
    int* row_src = reinterpret_cast<int*>(ws + L.row_src);
    __half* h = reinterpret_cast<__half*>(ws + L.h);
    float* y = reinterpret_cast<float*>(ws + L.y);
    void* split = ws + L.split;
    const size_t split_bytes = std::max(s1, s2);
    const cudaStream_t s = (cudaStream_t)stream;

    st = launch_route(logits, T, E, k, ids, wts, counts, offsets, inv_perm, row_src, 1, nullptr, s);
    if (st != CKL_OK) return st;
    // gate/up waits for the routing; down prefetches its first weight stages while gate/up
    // finishes (its offsets are the routing's, one kernel older); combine waits for down.
    st = expert_gemm(X, row_src, offsets, A, T, gate, up, h, 0, 0, split, split_bytes, stream, 1);
    if (st != CKL_OK) return st;
    st = expert_gemm(h, nullptr, offsets, A, T, down, nullptr, y, 1, 0, split, split_bytes, stream,
                     s2 > 0 ? 1 : 2);
    if (st != CKL_OK) return st;
    void* cargs[] = {&y, &inv_perm, &wts, &out, &k, const_cast<int*>(&d)};
    CKL_CUDA_TRY(launch(reinterpret_cast<const void*>(combine_kernel<true>), dim3(T), dim3(256), 0,
                        s, cargs, true));
    return CKL_OK;
}

}  // extern "C"
