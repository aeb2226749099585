// moe_ep.cu -- expert-parallel MoE decode layer over NVLink peer memory.
//
// The reference's MoE layer is single-GPU (MoeDecode, 03_moe_wq_decode.cu:350-391); the
// north star partitions it by expert: rank r owns experts [r*E/n, (r+1)*E/n) and tokens are
// exchanged in an all-to-all for dispatch and combine. Here the exchange is done by the
// layer's own kernels through CUDA-IPC-mapped windows instead of a library collective, so
// nothing waits on the host and each transfer is issued by the kernel that has the data:
//
//   route     (1 CTA)    top-k, counts, offsets, stable slot order for this rank's tokens
//   dispatch  (A CTAs)   writes the token row of assignment i into the owner's window, slab
//                        `rank`, at position inv_perm[i] - offsets[first expert of owner]
//                        (expert order within the slab), plus this rank's per-expert counts
//   receive   (1 CTA)    raises this rank's dispatch flag in every owner's window, waits for
//                        every source's flag, then builds the expert offsets and the gather
//                        map (row -> slab position) over all received rows
//   gate/up   GEMM       SwiGLU over the received rows (gathered through the map)
//   down      GEMM       writes output row a to the window's y at the row's slab position
//   combine   (T CTAs)   raises this rank's ready flag in every source's window, waits for
//                        every owner's ready flag, reads its assignments' rows from the
//                        owners' windows and sums them in fixed slot order
//
// A flag is raised by a release store at system scope from the kernel that follows the
// writes it covers (stream order, griddepcontrol.wait), so the writes of the previous kernel
// -- the dispatch's row stores into peer memory, the down GEMM's outputs -- are ordered
// before it without a fence in every writing thread; a reader acquires the flag, then reads.
// Flags carry epochs (calls completed on the rank, +1), so windows never need resetting.
// One window per rank is enough: a source writes call i+1's rows only after its combine of
// call i saw every owner's ready flag, i.e. after every owner finished reading call i's
// rows; an owner writes call i+1's outputs only after every source's call-i+1 dispatch flag,
// i.e. after every source finished reading call i's outputs. Every wait is bounded; a wait
// that gives up records DEVERR_TIMEOUT and the kernel carries on with what it has (counts
// are clamped to the slab capacity, so no access leaves the windows).

#include <algorithm>

#include "ckl_internal.h"
#include "ckl_ptx.cuh"
#include "moe_internal.h"

namespace ckl {
namespace moe {


ckl_status check_route(int T, int E, int k);

constexpr int EP_MAX_E = 256;
// control block at the start of every window (u32 words)
constexpr int EP_DISP_FLAG = 0;     // [CKL_EP_MAX_RANKS]: epoch of source s's last dispatch
constexpr int EP_READY_FLAG = 64;   // [CKL_EP_MAX_RANKS]: epoch of owner o's last outputs
constexpr int EP_EPOCH = 128;       // calls completed on this rank
constexpr int EP_CNT_COMB = 136;    // combine CTAs finished (last-CTA detection)
constexpr int EP_CTRL_BYTES = 256;
constexpr int RECV_THREADS = 512;

// Window layout (identical on every rank):
//   [0, 256)   control block
//   counts     int32 [world][E_loc]: rows source s sent for each local expert
//   rows       fp16  [world * cap][d]: received token rows, slab s = [s*cap, (s+1)*cap)
//   y          fp32  [world * cap][d]: expert outputs at the rows' slab positions
// cap = T_cap * min(k, E_loc): a token reaches each expert at most once.
struct EpLayout {
    int E_loc = 0, cap = 0, A_max = 0;
    size_t counts = 0, rows = 0, y = 0, total = 0;
};
inline EpLayout ep_layout(int world, int T_cap, int k, int E, int d) {
    EpLayout L;
    L.E_loc = E / world;
    L.cap = T_cap * std::min(k, L.E_loc);
    L.A_max = world * L.cap;
    L.counts = EP_CTRL_BYTES;
    L.rows = align_up(L.counts + (size_t)world * L.E_loc * 4, 256);
    L.y = align_up(L.rows + (size_t)L.A_max * d * 2, 256);
    L.total = align_up(L.y + (size_t)L.A_max * d * 4, 256);
    return L;
}

struct EpArgs {
    uint8_t* win[CKL_EP_MAX_RANKS];
    int rank, world, cap, E_loc, d, k;
    unsigned long long off_counts, off_rows, off_y;
    unsigned* err;
    unsigned long long timeout_ns;
};

__device__ __forceinline__ unsigned* ctrl(uint8_t* w, int off) {
    return reinterpret_cast<unsigned*>(w + off);
}
__device__ __forceinline__ unsigned next_epoch(const EpArgs& p) {
    return *reinterpret_cast<volatile unsigned*>(p.win[p.rank] + EP_EPOCH) + 1u;
}

// grid = max(A, 1), 256 threads: CTA i copies the row of assignment i (16-byte stores into
// the owner's window); CTA 0 also writes this rank's counts into every owner's window.
__global__ void __launch_bounds__(256)
ep_dispatch_kernel(const EpArgs p, const __half* __restrict__ X, const int* __restrict__ ids,
                   const int* __restrict__ inv_perm, const int* __restrict__ offsets,
                   const int* __restrict__ counts, int A) {
    pdl_wait();                                       // routing results
    pdl_trigger();
    const int i = blockIdx.x;
    if (i < A) {
        const int e = __ldg(ids + i);
        const int o = e / p.E_loc;
        const int pos = __ldg(inv_perm + i) - __ldg(offsets + o * p.E_loc);
        const uint4* src = reinterpret_cast<const uint4*>(X + (size_t)(i / p.k) * p.d);
        uint4* dst = reinterpret_cast<uint4*>(p.win[o] + p.off_rows +
                                              ((size_t)p.rank * p.cap + pos) * p.d * 2);
        for (int c = threadIdx.x; c < p.d / 8; c += blockDim.x) dst[c] = __ldg(src + c);
    }
    if (blockIdx.x == 0)
        for (int e = threadIdx.x; e < p.world * p.E_loc; e += blockDim.x) {
            const int o = e / p.E_loc;
            reinterpret_cast<int*>(p.win[o] + p.off_counts)[p.rank * p.E_loc + (e - o * p.E_loc)] =
                __ldg(counts + e);
        }
}

// grid = 1: waits for every source, then the expert offsets over the received rows
// (expert-major, then source, then slab order) and the gather map row_src[a] = slab index.
__global__ void __launch_bounds__(RECV_THREADS)
ep_receive_kernel(const EpArgs p, int* __restrict__ offsets_loc, int* __restrict__ row_src,
                  int rows_bound) {
    // world * E_loc = E <= EP_MAX_E entries, indexed [s][e]
    __shared__ int s_cnt[EP_MAX_E];    // rows of (s, e), clamped to the slab
    __shared__ int s_soff[EP_MAX_E];   // slab offset of (s, e)
    __shared__ int s_base[EP_MAX_E];   // first gathered row of (s, e)
    __shared__ int s_off[EP_MAX_E + 1];
    pdl_wait();                                       // our dispatch has completed
    pdl_trigger();                                    // the gate/up GEMM waits for our results
    const unsigned epoch = next_epoch(p);
    uint8_t* own = p.win[p.rank];
    if (threadIdx.x < p.world) {
        // our rows and counts are in every owner's window: raise our flag there, then wait
        // for every source's flag here
        st_release_sys(ctrl(p.win[threadIdx.x], EP_DISP_FLAG) + p.rank, epoch);
        wait_epoch(ctrl(own, EP_DISP_FLAG) + threadIdx.x, epoch,
                   globaltimer() + p.timeout_ns, p.err);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const int nse = p.world * p.E_loc;
    const int* cnt_g = reinterpret_cast<const int*>(own + p.off_counts);
    // warp s: slab offsets of source s, counts clamped so the slab never overflows
    if (warp < p.world) {
        int carry = 0;
        for (int e0 = 0; e0 < p.E_loc; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < p.E_loc ? min(max(0, __ldcg(cnt_g + warp * p.E_loc + e)), p.cap) : 0;
            int inc = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            const int excl = carry + inc - c;
            if (e < p.E_loc) {
                s_soff[warp * p.E_loc + e] = excl;
                s_cnt[warp * p.E_loc + e] = min(c, max(0, p.cap - excl));
            }
            carry += __shfl_sync(0xffffffffu, inc, 31);
        }
    }
    __syncthreads();
    // warp 0: expert offsets over the sum of all sources
    if (warp == 0) {
        int carry = 0;
        for (int e0 = 0; e0 < p.E_loc; e0 += 32) {
            const int e = e0 + lane;
            int c = 0;
            if (e < p.E_loc)
                for (int s = 0; s < p.world; s++) c += s_cnt[s * p.E_loc + e];
            int inc = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            if (e < p.E_loc) s_off[e] = carry + inc - c;
            carry += __shfl_sync(0xffffffffu, inc, 31);
        }
        __syncwarp();
        if (lane == 0) {
            if (carry > rows_bound) {                 // more rows than the caller's bound: none
                atomicOr(p.err, DEVERR_BOUND);        // is processed (offsets all zero)
                for (int e = 0; e <= p.E_loc; e++) s_off[e] = 0;
                for (int e = 0; e < p.world * p.E_loc; e++) s_cnt[e] = 0;
            } else {
                s_off[p.E_loc] = carry;
            }
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e <= p.E_loc; e += blockDim.x) offsets_loc[e] = s_off[e];
    for (int e = threadIdx.x; e < p.E_loc; e += blockDim.x) {
        int b = s_off[e];
        for (int s = 0; s < p.world; s++) {
            s_base[s * p.E_loc + e] = b;
            b += s_cnt[s * p.E_loc + e];
        }
    }
    __syncthreads();
    for (int se = warp; se < nse; se += nwarps) {
        const int s = se / p.E_loc;
        const int c = s_cnt[se], b = s_base[se], so = s * p.cap + s_soff[se];
        for (int r = lane; r < c; r += 32) row_src[b + r] = so + r;
    }
}

// grid = max(T, 1), 256 threads: every CTA raises this rank's ready flag in every source's
// window (the down GEMM's outputs are complete), waits for every owner's, then
// out[t] = sum_{j<k} wts[t][j] * y_owner[slab row] in fixed j order with fp32 accumulation
// (the arithmetic of the single-GPU combine); the last CTA advances the rank's epoch.
__global__ void __launch_bounds__(256)
ep_combine_kernel(const EpArgs p, const int* __restrict__ ids, const int* __restrict__ inv_perm,
                  const int* __restrict__ offsets, const float* __restrict__ wts,
                  __half* __restrict__ out, int T) {
    // Each assignment's owner, slab row and weight come from the routing, which completed
    // before the kernel we wait for was launched: look them up (from L2) before the wait, so
    // that after the flags only the rows are left to read.
    constexpr int KMAX = 8;                           // k <= 8 (the routing's bound)
    const int t = blockIdx.x;
    int own_j[KMAX], pos_j[KMAX];
    float w_j[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; j++) {
        own_j[j] = 0;
        pos_j[j] = 0;
        w_j[j] = 0.f;
        if (t < T && j < p.k) {
            const int i = t * p.k + j;
            const int o = __ldcg(ids + i) / p.E_loc;
            own_j[j] = o;
            pos_j[j] = __ldcg(inv_perm + i) - __ldcg(offsets + o * p.E_loc);
            w_j[j] = __ldcg(wts + i);
        }
    }
    pdl_wait();                                       // the down GEMM has completed
    pdl_trigger();                                    // the next layer's routing may launch
    const unsigned epoch = next_epoch(p);
    uint8_t* own = p.win[p.rank];
    if ((int)threadIdx.x < p.world) {
        st_release_sys(ctrl(p.win[threadIdx.x], EP_READY_FLAG) + p.rank, epoch);
        wait_epoch(ctrl(own, EP_READY_FLAG) + threadIdx.x, epoch,
                   globaltimer() + p.timeout_ns, p.err);
    }
    __syncthreads();
    if (t < T) {
        for (int c = threadIdx.x; c < p.d / 8; c += blockDim.x) {
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
            for (int j = 0; j < KMAX; j++) {
                if (j >= p.k) break;
                const int o = own_j[j], pos = pos_j[j];
                const float w = w_j[j];
                const float4* src = reinterpret_cast<const float4*>(
                    p.win[o] + p.off_y + ((size_t)p.rank * p.cap + pos) * p.d * 4) + 2 * c;
                const float4 v0 = __ldcg(src), v1 = __ldcg(src + 1);
                acc[0] += w * v0.x; acc[1] += w * v0.y; acc[2] += w * v0.z; acc[3] += w * v0.w;
                acc[4] += w * v1.x; acc[5] += w * v1.y; acc[6] += w * v1.z; acc[7] += w * v1.w;
            }
            __align__(16) __half2 h[4];
#pragma unroll
            for (int q = 0; q < 4; q++) h[q] = __floats2half2_rn(acc[2 * q], acc[2 * q + 1]);
            reinterpret_cast<uint4*>(out + (size_t)t * p.d)[c] = *reinterpret_cast<uint4*>(h);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned* cnt = ctrl(own, EP_CNT_COMB);
        if (atomicAdd(cnt, 1u) == gridDim.x - 1) {    // every CTA has read the epoch
            atomicExch(cnt, 0u);
            __threadfence();
            *reinterpret_cast<volatile unsigned*>(own + EP_EPOCH) = epoch;
        }
    }
}

// Workspace of one rank (256-byte aligned pieces).
struct EpWs {
    size_t ids, wts, counts, offsets, inv_perm, offsets_loc, row_src, h, split, total;
};
inline EpWs ep_ws(const ckl_moe_ep_comm* c, const EpLayout& L, int F, size_t split_bytes) {
    EpWs w{};
    const size_t A = (size_t)c->T_cap * c->k;
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t r = o; o += align_up(std::max<size_t>(bytes, 1), 256); return r; };
    w.ids = take(A * 4);
    w.wts = take(A * 4);
    w.counts = take((size_t)c->E * 4);
    w.offsets = take((size_t)(c->E + 1) * 4);
    w.inv_perm = take(A * 4);
    w.offsets_loc = take((size_t)(L.E_loc + 1) * 4);
    w.row_src = take((size_t)L.A_max * 4);
    w.h = take((size_t)L.A_max * F * 2);
    w.split = take(split_bytes);
    w.total = o;
    return w;
}

ckl_status check_comm(const ckl_moe_ep_comm* c) {
    if (!c) return fail(CKL_INVALID_ARG, "moe_ep: comm is NULL");
    if (c->world < 1 || c->world > CKL_EP_MAX_RANKS || c->rank < 0 || c->rank >= c->world)
        return fail(CKL_INVALID_ARG, "moe_ep: rank %d of world %d (world <= %d)", c->rank, c->world,
                    CKL_EP_MAX_RANKS);
    if (c->E <= 0 || c->E > EP_MAX_E || c->E % c->world)
        return fail(CKL_UNSUPPORTED_SHAPE, "moe_ep: E=%d must divide by world=%d (E <= %d)", c->E,
                    c->world, EP_MAX_E);
    if (c->T_cap <= 0 || c->d <= 0 || c->d % 8)
        return fail(CKL_INVALID_ARG, "moe_ep: T_cap=%d d=%d (T_cap > 0, d %% 8 == 0)", c->T_cap, c->d);
    ckl_status st = check_route(c->T_cap, c->E, c->k);
    if (st != CKL_OK) return st;
    for (int i = 0; i < c->world; i++)
        if (!c->windows[i] || ((uintptr_t)c->windows[i] & 255))
            return fail(CKL_INVALID_ARG, "moe_ep: window %d is NULL or not 256-byte aligned", i);
    return CKL_OK;
}

}  // namespace moe
}  // namespace ckl

using namespace ckl;
using namespace ckl::moe;

extern "C" {

size_t ckl_moe_ep_window_bytes(int world, int T_cap, int k, int E, int d) {
    if (world < 1 || world > CKL_EP_MAX_RANKS || E <= 0 || E % world || T_cap <= 0 || k <= 0 || d <= 0)
        return 0;
    return ep_layout(world, T_cap, k, E, d).total;
}

ckl_status ckl_ep_window_alloc(size_t bytes, void** window, void* ipc_handle) {
    if (!window || !ipc_handle || bytes == 0) return fail(CKL_INVALID_ARG, "ep_window_alloc: args");
    static_assert(sizeof(cudaIpcMemHandle_t) <= CKL_IPC_HANDLE_BYTES, "IPC handle size");
    *window = nullptr;
    void* p = nullptr;
    CKL_CUDA_TRY(cudaMalloc(&p, bytes));
    // cudaMemset of device memory is asynchronous to the host: the window must be zero
    // before the handle can reach a peer (which may start writing flags into it)
    cudaError_t e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_status(e, "ep_window_alloc");
    }
    memset(ipc_handle, 0, CKL_IPC_HANDLE_BYTES);
    memcpy(ipc_handle, &h, sizeof(h));
    *window = p;
    return CKL_OK;
}

ckl_status ckl_ep_window_open(const void* ipc_handle, void** window) {
    if (!window || !ipc_handle) return fail(CKL_INVALID_ARG, "ep_window_open: args");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    *window = nullptr;
    CKL_CUDA_TRY(cudaIpcOpenMemHandle(window, h, cudaIpcMemLazyEnablePeerAccess));
    return CKL_OK;
}

ckl_status ckl_ep_window_close(void* window) {
    if (!window) return CKL_OK;
    CKL_CUDA_TRY(cudaIpcCloseMemHandle(window));
    return CKL_OK;
}

ckl_status ckl_ep_window_free(void* window) {
    if (!window) return CKL_OK;
    CKL_CUDA_TRY(cudaFree(window));
    return CKL_OK;
}

size_t ckl_moe_ep_workspace_size(const ckl_moe_ep_comm* comm, const ckl_moe_weights* gate,
                                 const ckl_moe_weights* down) {
    if (!comm || !gate || !down || comm->world < 1 || comm->E % comm->world) return 0;
    const EpLayout L = ep_layout(comm->world, comm->T_cap, comm->k, comm->E, comm->d);
    const size_t s1 = ckl_moe_gemm_workspace_size(gate, L.A_max, 1, 0);
    const size_t s2 = ckl_moe_gemm_workspace_size(down, L.A_max, 0, 0);
    return ep_ws(comm, L, gate->N, std::max(s1, s2)).total;
}

ckl_status ckl_moe_ep_layer(const ckl_moe_ep_comm* comm, const float* logits, const void* X, int T,
                            const ckl_moe_weights* gate, const ckl_moe_weights* up,
                            const ckl_moe_weights* down, void* out, int* ids_out, float* wts_out,
                            void* workspace, size_t workspace_bytes, void* stream) {
    return ckl_moe_ep_layer_ex(comm, 0, logits, X, T, gate, up, down, out, ids_out, wts_out, workspace,
                               workspace_bytes, stream);
}

ckl_status ckl_moe_ep_layer_ex(const ckl_moe_ep_comm* comm, int T_max, const float* logits,
                               const void* X, int T, const ckl_moe_weights* gate,
                               const ckl_moe_weights* up, const ckl_moe_weights* down, void* out,
                               int* ids_out, float* wts_out, void* workspace,
                               size_t workspace_bytes, void* stream) {
    ckl_status st = check_comm(comm);
    if (st != CKL_OK) return st;
    if (T_max < 0 || T_max > comm->T_cap)
        return fail(CKL_INVALID_ARG, "moe_ep_layer: T_max=%d outside [0, T_cap=%d]", T_max, comm->T_cap);
    if (!gate || !up || !down) return fail(CKL_INVALID_ARG, "moe_ep_layer: NULL weights");
    const EpLayout L = ep_layout(comm->world, comm->T_cap, comm->k, comm->E, comm->d);
    const int d = comm->d, F = gate->N, k = comm->k;
    if (gate->E != L.E_loc || gate->K != d || down->E != L.E_loc || down->K != F || down->N != d)
        return fail(CKL_INVALID_ARG,
                    "moe_ep_layer: local experts must be gate/up [%d][%d][F], down [%d][F][%d]",
                    L.E_loc, d, L.E_loc, d);
    if (T < 0 || T > comm->T_cap)
        return fail(CKL_INVALID_ARG, "moe_ep_layer: T=%d outside [0, T_cap=%d]", T, comm->T_cap);
    if (T_max > 0 && T > T_max)
        return fail(CKL_INVALID_ARG, "moe_ep_layer: T=%d above this call's T_max=%d", T, T_max);
    // rows any rank can receive this call: the GEMM grids' bound
    const int A_bound = T_max > 0 ? comm->world * T_max * std::min(k, L.E_loc) : L.A_max;
    if (T > 0 && (!logits || !X || !out)) return fail(CKL_INVALID_ARG, "moe_ep_layer: NULL tensor");
    if (((uintptr_t)X | (uintptr_t)out) & 15)
        return fail(CKL_INVALID_ARG, "moe_ep_layer: X/out need 16-byte alignment");
    const size_t s1 = ckl_moe_gemm_workspace_size(gate, L.A_max, 1, 0);
    const size_t s2 = ckl_moe_gemm_workspace_size(down, L.A_max, 0, 0);
    const size_t split_bytes = std::max(s1, s2);
    const EpWs W = ep_ws(comm, L, F, split_bytes);
    if (!workspace || workspace_bytes < W.total)
        return fail(CKL_WORKSPACE_TOO_SMALL, "moe_ep_layer needs %zu workspace bytes, got %zu",
                    W.total, workspace_bytes);
    if ((uintptr_t)workspace & 255) return fail(CKL_INVALID_ARG, "workspace must be 256-byte aligned");
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;

    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int* ids = ids_out ? ids_out : reinterpret_cast<int*>(ws + W.ids);
    float* wts = wts_out ? wts_out : reinterpret_cast<float*>(ws + W.wts);
    int* counts = reinterpret_cast<int*>(ws + W.counts);
    int* offsets = reinterpret_cast<int*>(ws + W.offsets);
    int* inv_perm = reinterpret_cast<int*>(ws + W.inv_perm);
    int* offsets_loc = reinterpret_cast<int*>(ws + W.offsets_loc);
    int* row_src = reinterpret_cast<int*>(ws + W.row_src);
    __half* h = reinterpret_cast<__half*>(ws + W.h);
    void* split = ws + W.split;
    const cudaStream_t s = (cudaStream_t)stream;

    EpArgs p{};
    for (int i = 0; i < comm->world; i++) p.win[i] = static_cast<uint8_t*>(comm->windows[i]);
    p.rank = comm->rank;
    p.world = comm->world;
    p.cap = L.cap;
    p.E_loc = L.E_loc;
    p.d = d;
    p.k = k;
    p.off_counts = L.counts;
    p.off_rows = L.rows;
    p.off_y = L.y;
    p.err = di->err_word;
    p.timeout_ns = spin_timeout_ns();
    uint8_t* own = p.win[p.rank];

    st = route_tokens(logits, T, comm->E, k, ids, wts, counts, offsets, inv_perm, nullptr, s);
    if (st != CKL_OK) return st;
    int A = T * k;
    {
        const __half* Xh = static_cast<const __half*>(X);
        void* args[] = {&p, &Xh, &ids, &inv_perm, &offsets, &counts, &A};
        CKL_CUDA_TRY(launch(reinterpret_cast<const void*>(ep_dispatch_kernel), dim3(std::max(A, 1)),
                            dim3(256), 0, s, args, true));
    }
    {
        int bound = A_bound;
        void* args[] = {&p, &offsets_loc, &row_src, &bound};
        CKL_CUDA_TRY(launch(reinterpret_cast<const void*>(ep_receive_kernel), dim3(1),
                            dim3(RECV_THREADS), 0, s, args, true));
    }
    const int* a_rows = offsets_loc + L.E_loc;
    st = expert_gemm(own + L.rows, row_src, offsets_loc, A_bound, comm->T_cap * comm->world, gate,
                     up, h, 0, 0, split, split_bytes, stream, 1, nullptr, a_rows);
    if (st != CKL_OK) return st;
    st = expert_gemm(h, nullptr, offsets_loc, A_bound, comm->T_cap * comm->world, down, nullptr,
                     own + L.y, 1, 0, split, split_bytes, stream, s2 > 0 ? 1 : 2, row_src, a_rows);
    if (st != CKL_OK) return st;
    {
        __half* o16 = static_cast<__half*>(out);
        void* args[] = {&p, &ids, &inv_perm, &offsets, &wts, &o16, &T};
        CKL_CUDA_TRY(launch(reinterpret_cast<const void*>(ep_combine_kernel), dim3(std::max(T, 1)),
                            dim3(256), 0, s, args, true));
    }
    return CKL_OK;
}

}  // extern "C"
