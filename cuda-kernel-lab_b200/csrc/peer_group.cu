// peer_group.cu -- completion flags for a gather into one rank's buffers over NVLink.
//
// Head-parallel attention writes each rank's output rows straight into the root's buffers
// (ckl_decode_attention_gather). The root learns that every rank's rows have landed from
// one epoch flag per rank in its flag window: a rank's signal kernel runs after its writing
// kernels (stream order), fences at system scope and release-stores its epoch into the
// root's slot; the root's wait kernel acquires every slot up to its own epoch (bounded).
//
// A barrier of the group (ckl_peer_barrier) works the same way in every direction: each rank
// release-stores its barrier epoch into every rank's slot for it and waits for every slot of
// its own window.
//
// Window layout (u32): [0, 8) gather flags by source rank, [16] signals sent by this rank,
// [17] waits completed by this rank, [32, 40) barrier flags by source rank, [48] barriers
// passed by this rank.

#include "ckl_internal.h"
#include "ckl_ptx.cuh"

namespace ckl {
namespace peer {

constexpr int FLAGS = 0;
constexpr int SENT = 16;
constexpr int WAITED = 17;
constexpr int BAR_FLAGS = 32;
constexpr int BAR_EPOCH = 48;

struct GroupArgs {
    unsigned* win[8];
    int rank, world;
    unsigned* err;
    unsigned long long timeout_ns;
};

__global__ void gather_signal_kernel(const GroupArgs g, int root) {
    if (threadIdx.x != 0) return;
    volatile unsigned* sent = g.win[g.rank] + SENT;
    const unsigned epoch = *sent + 1u;
    *sent = epoch;
    __threadfence_system();                  // the rows this rank wrote before this kernel
    st_release_sys(g.win[root] + FLAGS + g.rank, epoch);
}

__global__ void gather_wait_kernel(const GroupArgs g) {
    __shared__ unsigned s_epoch;
    volatile unsigned* waited = g.win[g.rank] + WAITED;
    if (threadIdx.x == 0) s_epoch = *waited + 1u;
    __syncthreads();
    const unsigned epoch = s_epoch;
    if ((int)threadIdx.x < g.world)
        wait_epoch(g.win[g.rank] + FLAGS + threadIdx.x, epoch, globaltimer() + g.timeout_ns, g.err);
    __syncthreads();
    if (threadIdx.x == 0) *waited = epoch;
}

__global__ void peer_barrier_kernel(const GroupArgs g) {
    __shared__ unsigned s_epoch;
    volatile unsigned* passed = g.win[g.rank] + BAR_EPOCH;
    if (threadIdx.x == 0) s_epoch = *passed + 1u;
    __syncthreads();
    const unsigned epoch = s_epoch;
    if ((int)threadIdx.x < g.world) {
        __threadfence_system();              // this rank's work before the barrier
        st_release_sys(g.win[threadIdx.x] + BAR_FLAGS + g.rank, epoch);
        wait_epoch(g.win[g.rank] + BAR_FLAGS + threadIdx.x, epoch, globaltimer() + g.timeout_ns,
                   g.err);
    }
    __syncthreads();
    if (threadIdx.x == 0) *passed = epoch;
}

ckl_status make_args(const ckl_peer_group* g, GroupArgs* a) {
    if (!g || g->world < 1 || g->world > 8 || g->rank < 0 || g->rank >= g->world)
        return fail(CKL_INVALID_ARG, "peer group: rank/world");
    for (int i = 0; i < g->world; i++) {
        if (!g->windows[i] || ((uintptr_t)g->windows[i] & 255))
            return fail(CKL_INVALID_ARG, "peer group: window %d NULL or not 256-byte aligned", i);
        a->win[i] = static_cast<unsigned*>(g->windows[i]);
    }
    a->rank = g->rank;
    a->world = g->world;
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    a->err = di->err_word;
    a->timeout_ns = spin_timeout_ns();
    return CKL_OK;
}

}  // namespace peer
}  // namespace ckl

using namespace ckl;
using namespace ckl::peer;

extern "C" {

ckl_status ckl_gather_signal(const ckl_peer_group* g, int root, void* stream) {
    GroupArgs a{};
    ckl_status st = make_args(g, &a);
    if (st != CKL_OK) return st;
    if (root < 0 || root >= g->world) return fail(CKL_INVALID_ARG, "gather_signal: root %d", root);
    gather_signal_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(a, root);
    CKL_CUDA_TRY(cudaGetLastError());
    return CKL_OK;
}

ckl_status ckl_peer_barrier(const ckl_peer_group* g, void* stream) {
    GroupArgs a{};
    ckl_status st = make_args(g, &a);
    if (st != CKL_OK) return st;
    peer_barrier_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(a);
    CKL_CUDA_TRY(cudaGetLastError());
    return CKL_OK;
}

ckl_status ckl_gather_wait(const ckl_peer_group* g, void* stream) {
    GroupArgs a{};
    ckl_status st = make_args(g, &a);
    if (st != CKL_OK) return st;
    gather_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(a);
    CKL_CUDA_TRY(cudaGetLastError());
    return CKL_OK;
}

}  // extern "C"
