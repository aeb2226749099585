// cascade.cu -- shared-prefix (cascade) decode for sm_100a.
//
// Replaces shared_prefix_pages / plan_cascade / cascade_prefix / cascade_decode of the
// reference (01_decode_attention.cu:446-712). When every sequence of a batch starts with
// the same physical pages (prefix caching), the plain kernel reads those pages once per
// sequence. The cascade reads them once per kv head:
//
//   1. host: the longest run of physical pages every sequence starts with (each keeps >= 1
//      private page), from the caller's host copy of the page table;
//   2. prefix kernel: the B*G query rows that share a kv head are stacked into 128-row tiles
//      (8 consumer warps x 16 rows); a producer warp TMA-loads each shared page once into an
//      8-stage ring and every consumer warp runs Q K^T and P V on it with mma.sync, with a
//      single-pass online softmax (the reference makes two passes because WMMA cannot
//      rescale its accumulators; register fragments can);
//   3. suffix: the split-KV partial kernel from kv_start = prefix length;
//   4. one LSE merge over prefix and suffix slots.

#include <algorithm>
#include <cstring>
#include <mutex>
#include <numeric>
#include <vector>

#include "attn_common.cuh"

namespace ckl {
namespace cascade {

using namespace attn;

constexpr int PWARPS = 4;                     // consumer warps, 16 stacked query rows each
constexpr int PROWS = PWARPS * 16;            // query rows per CTA
constexpr int PTHREADS = (PWARPS + 1) * 32;   // + one TMA producer warp
constexpr int PSTAGES = 8;
constexpr int P_RING = PSTAGES * STAGE_BYTES;
constexpr int P_SMEM = 1024 + P_RING + 2 * PSTAGES * 8;

struct PrefixArgs {
    const __half* q;
    const int* prefix_pages;
    // prefix-tree mode (items != NULL): CTA x runs work item x, two int4 each:
    //   {first page (index into kv_indices), pages, first member (position in perm), members},
    //   {first stacked query row, partial slot, 0, 0}
    const int4* items;
    const int* indices;
    const int* perm;
    float* part_o;
    float* part_lse;
    unsigned* err;
    unsigned long long timeout_ns;
    int B, Hq, Hkv, G, prefix_len, chunk_tokens, part_stride;
    float scale_log2;
};

// grid = (prefix chunks, ceil(B*G / 128), Hkv). Writes the normalised partial (o, lse) of
// every stacked query row it covers into slot blockIdx.x. Prefix-tree mode: grid = (work
// items, 1, Hkv); item x covers a run of pages shared by the sequences perm[m0, m0 + members)
// and its stacked rows [row0, row0 + 128) of members x G, written into the item's slot.
__global__ void __launch_bounds__(PTHREADS, 2)
cascade_prefix_kernel(const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const PrefixArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = align_ptr<1024>(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + P_RING);
    uint64_t* empty = full + PSTAGES;

    const int kvh = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int* pages;          // this CTA's run of physical page ids
    int npg, kend;             // pages, and keys of the run (tokens from its first page)
    int nq, row0, m0, slot;    // stacked rows, first row of this tile, first member, slot
    if (a.items) {
        const int4 w0 = __ldg(a.items + 2 * blockIdx.x), w1 = __ldg(a.items + 2 * blockIdx.x + 1);
        pages = a.indices + w0.x;
        npg = w0.y;
        kend = npg * PAGE;     // shared runs never hold a sequence's last page: all full
        m0 = w0.z;
        nq = w0.w * a.G;
        row0 = w1.x;
        slot = w1.y;
    } else {
        const int kbeg = blockIdx.x * a.chunk_tokens;
        const int kstop = min(a.prefix_len, kbeg + a.chunk_tokens);
        pages = a.prefix_pages + kbeg / PAGE;
        npg = kstop > kbeg ? (kstop - kbeg + PAGE - 1) / PAGE : 0;
        kend = kstop - kbeg;
        m0 = 0;
        nq = a.B * a.G;
        row0 = blockIdx.y * PROWS;
        slot = blockIdx.x;
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < PSTAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], PWARPS);
        }
        fence_barrier_init();
    }
    __syncthreads();
    const uint64_t deadline = globaltimer() + a.timeout_ns;
    pdl_trigger();                   // the suffix kernel (independent slots) may start now

    if (warp == PWARPS) {
        // ---------------------------------------------------------------- producer warp
        if (lane == 0) {
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
        }
        // the prefix is re-read by the other query tiles of this kv head: keep it in L2
        const uint64_t pol = policy_evict_last();
        int ok = 1, issued = 0;
        for (int base = 0; base < npg && ok; base += 32) {
            const int cnt = min(32, npg - base);
            const int my_page = lane < cnt ? __ldg(pages + base + lane) : 0;
            for (int j = 0; j < cnt; j++) {
                const int page = __shfl_sync(0xffffffffu, my_page, j);
                if (lane == 0) {
                    const int i = base + j, s = i % PSTAGES;
                    if (i >= PSTAGES) ok = mbar_wait(&empty[s], ((i / PSTAGES) - 1) & 1, deadline, a.err);
                    if (ok) {
                        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                        load_page(ring + s * STAGE_BYTES, &tmK, &tmV, kvh, page, &full[s], pol);
                        issued = i + 1;
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
        }
        if (lane == 0) {
            for (int s = 0; s < PSTAGES && s < issued; s++) {
                const int i_last = s + ((issued - 1 - s) / PSTAGES) * PSTAGES;
                mbar_wait(&full[s], (i_last / PSTAGES) & 1, deadline, a.err);
            }
        }
        return;
    }

    // -------------------------------------------------------------------- consumer warps
    const int g = lane >> 2, t = lane & 3;
    const int r_lo = row0 + warp * 16 + g, r_hi = r_lo + 8;
    const bool ok_lo = r_lo < nq, ok_hi = r_hi < nq;
    const bool active = row0 + warp * 16 < nq;   // warp-uniform
    size_t qrow_lo = 0, qrow_hi = 0;
    if (ok_lo) {
        const int seq = a.perm ? __ldg(a.perm + m0 + r_lo / a.G) : r_lo / a.G;
        qrow_lo = (size_t)seq * a.Hq + (size_t)kvh * a.G + r_lo % a.G;
    }
    if (ok_hi) {
        const int seq = a.perm ? __ldg(a.perm + m0 + r_hi / a.G) : r_hi / a.G;
        qrow_hi = (size_t)seq * a.Hq + (size_t)kvh * a.G + r_hi % a.G;
    }

    uint32_t qa0[8], qa1[8], qa2[8], qa3[8];
#pragma unroll
    for (int kk = 0; kk < 8; kk++) qa0[kk] = qa1[kk] = qa2[kk] = qa3[kk] = 0u;
    if (ok_lo) {
        const uint32_t* qr = reinterpret_cast<const uint32_t*>(a.q + qrow_lo * D);
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
            qa0[kk] = __ldg(qr + 8 * kk + t);
            qa2[kk] = __ldg(qr + 8 * kk + 4 + t);
        }
    }
    if (ok_hi) {
        const uint32_t* qr = reinterpret_cast<const uint32_t*>(a.q + qrow_hi * D);
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
            qa1[kk] = __ldg(qr + 8 * kk + t);
            qa3[kk] = __ldg(qr + 8 * kk + 4 + t);
        }
    }
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
    const int k_key = (lane & 7) + ((lane >> 4) << 3), k_hi = (lane >> 3) & 1;
    const int v_key = (lane & 7) + (((lane >> 3) & 1) << 3), v_hi = lane >> 4;

    bool ok = true;
    for (int i = 0; i < npg; i++) {
        const int s = i % PSTAGES;
        const bool got = mbar_wait(&full[s], (i / PSTAGES) & 1, deadline, a.err);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        if (active) {
            const uint32_t kb = smem_u32(ring + s * STAGE_BYTES);
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
            const int kbase = i * PAGE;
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
                for (int c = 0; c < 4; c++) sc[n][c] *= a.scale_log2;
            float mx_lo = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
            float mx_hi = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
            mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
            mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
            mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
            mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
            const bool need = mx_lo > m_lo + RESCALE_THRESHOLD || mx_hi > m_hi + RESCALE_THRESHOLD;
            if (__any_sync(0xffffffffu, need)) {
                const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
                const float c_lo = ex2(m_lo - mn_lo), c_hi = ex2(m_hi - mn_hi);
                m_lo = mn_lo;
                m_hi = mn_hi;
                l_lo *= c_lo;
                l_hi *= c_hi;
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    o[j][0] *= c_lo;
                    o[j][1] *= c_lo;
                    o[j][2] *= c_hi;
                    o[j][3] *= c_hi;
                }
            }
            const float p00 = ex2(sc[0][0] - m_lo), p01 = ex2(sc[0][1] - m_lo);
            const float p10 = ex2(sc[1][0] - m_lo), p11 = ex2(sc[1][1] - m_lo);
            const float q00 = ex2(sc[0][2] - m_hi), q01 = ex2(sc[0][3] - m_hi);
            const float q10 = ex2(sc[1][2] - m_hi), q11 = ex2(sc[1][3] - m_hi);
            l_lo += (p00 + p01) + (p10 + p11);
            l_hi += (q00 + q01) + (q10 + q11);
            const uint32_t pa0 = pack_half2(p00, p01), pa2 = pack_half2(p10, p11);
            const uint32_t pa1 = pack_half2(q00, q01), pa3 = pack_half2(q10, q11);
#pragma unroll
            for (int jj = 0; jj < 8; jj++) {
                uint32_t v0, v1, v2, v3;
                ldmatrix_x4_trans(vb + tile_off(v_key, 2 * jj + v_hi), v0, v1, v2, v3);
                mma_16816(o[2 * jj], pa0, pa1, pa2, pa3, v0, v1);
                mma_16816(o[2 * jj + 1], pa0, pa1, pa2, pa3, v2, v3);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!active) return;

    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
    if (!ok) { l_lo = l_hi = 0.f; }
    const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f, inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
    if (ok_lo) {
        const size_t pslot = qrow_lo * a.part_stride + slot;
        float* dst = a.part_o + pslot * D + 2 * t;
#pragma unroll
        for (int j = 0; j < 16; j++)
            *reinterpret_cast<float2*>(dst + 8 * j) = make_float2(o[j][0] * inv_lo, o[j][1] * inv_lo);
        if (t == 0) a.part_lse[pslot] = l_lo > 0.f ? (m_lo + lg2(l_lo)) * LN2 : -INFINITY;
    }
    if (ok_hi) {
        const size_t pslot = qrow_hi * a.part_stride + slot;
        float* dst = a.part_o + pslot * D + 2 * t;
#pragma unroll
        for (int j = 0; j < 16; j++)
            *reinterpret_cast<float2*>(dst + 8 * j) = make_float2(o[j][2] * inv_hi, o[j][3] * inv_hi);
        if (t == 0) a.part_lse[pslot] = l_hi > 0.f ? (m_hi + lg2(l_hi)) * LN2 : -INFINITY;
    }
}

struct PrefixSetup {
    int per_sm = 0;
    ckl_status st = CKL_OK;
};
const PrefixSetup* setup(const DeviceInfo* di) {
    static PrefixSetup ps[64];
    static std::once_flag once[64];
    std::call_once(once[di->device], [di] {
        PrefixSetup& p = ps[di->device];
        const void* fn = reinterpret_cast<const void*>(cascade_prefix_kernel);
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM);
        if (e == cudaSuccess)
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&p.per_sm, fn, PTHREADS, P_SMEM);
        if (e != cudaSuccess) p.st = cuda_status(e, "cascade prefix kernel setup");
    });
    return &ps[di->device];
}

ckl_status launch_prefix(const ckl_cascade_plan_t* cp, float* part_o, float* part_lse,
                         cudaStream_t stream) {
    const ckl_decode_params& b = cp->suffix;
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    const PrefixSetup* ps = setup(di);
    if (ps->st != CKL_OK) return ps->st;
    CUtensorMap tmK, tmV;
    ckl_status st = encode_kv_maps(b.k_cache, b.v_cache, b.Hkv, b.num_pages, &tmK, &tmV);
    if (st != CKL_OK) return st;
    PrefixArgs a{};
    a.q = static_cast<const __half*>(b.q);
    a.prefix_pages = cp->prefix_page_ids;
    a.part_o = part_o;
    a.part_lse = part_lse;
    a.err = di->err_word;
    a.timeout_ns = spin_timeout_ns();
    a.B = b.B;
    a.Hq = b.Hq;
    a.Hkv = b.Hkv;
    a.G = b.Hq / b.Hkv;
    a.prefix_len = cp->prefix_len;
    a.chunk_tokens = cp->prefix_chunk_tokens;
    a.part_stride = b.part_stride;
    a.scale_log2 = b.sm_scale * LOG2E;
    void* args[] = {&tmK, &tmV, &a};
    dim3 grid((unsigned)cp->prefix_chunks, (unsigned)cp->qtiles, (unsigned)b.Hkv);
    CKL_CUDA_TRY(cudaLaunchKernel(reinterpret_cast<const void*>(cascade_prefix_kernel), grid,
                                  dim3(PTHREADS), args, P_SMEM, stream));
    return CKL_OK;
}

ckl_status check_plan(const ckl_cascade_plan_t* cp) {
    if (!cp) return fail(CKL_INVALID_ARG, "cascade plan is NULL");
    if (!cp->use) return CKL_OK;
    if (!cp->prefix_page_ids || cp->prefix_len <= 0 || cp->prefix_len % PAGE ||
        cp->prefix_chunks <= 0 || cp->prefix_chunk_tokens <= 0 || cp->prefix_chunk_tokens % PAGE ||
        cp->qtiles <= 0 || cp->suffix.chunk_base != cp->prefix_chunks ||
        cp->suffix.kv_start != cp->prefix_len)
        return fail(CKL_INVALID_ARG, "inconsistent cascade plan");
    if ((long long)cp->qtiles * PROWS < (long long)cp->suffix.B * (cp->suffix.Hq / cp->suffix.Hkv))
        return fail(CKL_INVALID_ARG, "cascade plan: qtiles do not cover B*G query rows");
    if (cp->prefix_chunks > 0x7fffffff / 1 || cp->qtiles > 65535 || cp->suffix.Hkv > 65535)
        return fail(CKL_UNSUPPORTED_SHAPE, "cascade grid too large");
    return CKL_OK;
}

// ------------------------------------------------------------------ prefix tree
// Device tables of the tree cascade, one buffer: seq_tab int2[B] {private suffix start in
// tokens, first suffix slot}, perm int[B], then the prefix work items, 2 x int4 each.
struct TreeTables {
    size_t perm, items, bytes;
};
TreeTables tree_tables(int B, int items) {
    TreeTables t;
    t.perm = align_up((size_t)B * 8, 16);
    t.items = t.perm + align_up((size_t)B * 4, 16);
    t.bytes = t.items + (size_t)items * 32;
    return t;
}

ckl_status launch_tree_prefix(const ckl_cascade_tree_plan_t* tp, const uint8_t* tables,
                              float* part_o, float* part_lse, cudaStream_t stream) {
    const ckl_decode_params& b = tp->suffix;
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    const PrefixSetup* ps = setup(di);
    if (ps->st != CKL_OK) return ps->st;
    CUtensorMap tmK, tmV;
    ckl_status st = encode_kv_maps(b.k_cache, b.v_cache, b.Hkv, b.num_pages, &tmK, &tmV);
    if (st != CKL_OK) return st;
    const TreeTables tt = tree_tables(b.B, tp->items);
    PrefixArgs a{};
    a.q = static_cast<const __half*>(b.q);
    a.items = reinterpret_cast<const int4*>(tables + tt.items);
    a.indices = b.kv_indices;
    a.perm = reinterpret_cast<const int*>(tables + tt.perm);
    a.part_o = part_o;
    a.part_lse = part_lse;
    a.err = di->err_word;
    a.timeout_ns = spin_timeout_ns();
    a.B = b.B;
    a.Hq = b.Hq;
    a.Hkv = b.Hkv;
    a.G = b.Hq / b.Hkv;
    a.part_stride = b.part_stride;
    a.scale_log2 = b.sm_scale * LOG2E;
    void* args[] = {&tmK, &tmV, &a};
    dim3 grid((unsigned)tp->items, 1, (unsigned)b.Hkv);
    CKL_CUDA_TRY(cudaLaunchKernel(reinterpret_cast<const void*>(cascade_prefix_kernel), grid,
                                  dim3(PTHREADS), args, P_SMEM, stream));
    return CKL_OK;
}

ckl_status check_tree_plan(const ckl_cascade_tree_plan_t* tp, const void* d_tables, int* G) {
    if (!tp) return fail(CKL_INVALID_ARG, "cascade tree plan is NULL");
    if (!tp->use) return fail(CKL_INVALID_ARG, "cascade tree plan has no shared node");
    const ckl_decode_params& sp = tp->suffix;
    ckl_status st = attn::validate(&sp, G);
    if (st != CKL_OK) return st;
    if (tp->nodes <= 0 || tp->items <= 0 || tp->chunk_pages <= 0 || tp->max_path_slots <= 0 ||
        sp.kv_start != 0 || sp.chunk_base != 0 || sp.part_stride != tp->max_path_slots + sp.num_chunks ||
        tp->table_bytes != tree_tables(sp.B, tp->items).bytes)
        return fail(CKL_INVALID_ARG, "inconsistent cascade tree plan");
    if (tp->suffix.Hkv > 65535) return fail(CKL_UNSUPPORTED_SHAPE, "cascade grid too large");
    if (!d_tables || ((uintptr_t)d_tables & 15))
        return fail(CKL_INVALID_ARG, "cascade tree tables must be 16-byte aligned device memory");
    return CKL_OK;
}

}  // namespace cascade
}  // namespace ckl

using namespace ckl;
using namespace ckl::cascade;

extern "C" {

int ckl_shared_prefix_pages(const int* h_indptr, const int* h_indices, int B) {
    if (!h_indptr || B < 2 || !h_indices) return 0;
    for (int P = 0;; P++) {
        for (int b = 0; b < B; b++)
            if (P >= h_indptr[b + 1] - h_indptr[b] - 1) return P;
        const int pg = h_indices[h_indptr[0] + P];
        for (int b = 1; b < B; b++)
            if (h_indices[h_indptr[b] + P] != pg) return P;
    }
}

ckl_status ckl_cascade_plan(const ckl_decode_params* base, const int* h_indptr,
                            const int* h_indices, const int* h_lens, int min_prefix,
                            ckl_cascade_plan_t* plan) {
    if (!plan || !base || !h_indptr || !h_lens) return fail(CKL_INVALID_ARG, "cascade_plan: NULL");
    int G = 0;
    ckl_status st = attn::validate(base, &G);
    if (st != CKL_OK) return st;
    *plan = ckl_cascade_plan_t{};
    plan->suffix = *base;
    int max_len = 0;
    for (int b = 0; b < base->B; b++) max_len = std::max(max_len, h_lens[b]);
    const int pages = ckl_shared_prefix_pages(h_indptr, h_indices, base->B);
    const int Lp = pages * PAGE;
    if (Lp == 0 || Lp < min_prefix) {
        // no usable shared prefix: the plan is the plain split-KV decode
        plan->use = 0;
        st = ckl_decode_plan(G, base->B, base->Hkv, max_len, 0, &plan->suffix.num_chunks,
                             &plan->suffix.chunk_tokens);
        plan->suffix.kv_start = 0;
        plan->suffix.chunk_base = 0;
        plan->suffix.part_stride = plan->suffix.num_chunks;
        return st;
    }
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    const PrefixSetup* ps = setup(di);
    if (ps->st != CKL_OK) return ps->st;
    plan->use = 1;
    plan->prefix_pages = pages;
    plan->prefix_len = Lp;
    plan->qtiles = ceil_div(base->B * G, PROWS);
    // about one wave of prefix CTAs, chunks of >= 256 tokens, a multiple of 32 tokens
    int cpre = std::max(1, di->sms * std::max(1, ps->per_sm) / (plan->qtiles * base->Hkv));
    cpre = std::min(cpre, std::max(1, Lp / 256));
    const int ctok = ceil_div(ceil_div(Lp, cpre), 32) * 32;
    plan->prefix_chunks = ceil_div(Lp, ctok);
    plan->prefix_chunk_tokens = ctok;
    plan->prefix_page_ids = base->kv_indices + h_indptr[0];
    int max_suffix = 0;
    for (int b = 0; b < base->B; b++) max_suffix = std::max(max_suffix, h_lens[b] - Lp);
    st = ckl_decode_plan(G, base->B, base->Hkv, std::max(max_suffix, 1), 0,
                         &plan->suffix.num_chunks, &plan->suffix.chunk_tokens);
    if (st != CKL_OK) return st;
    plan->suffix.kv_start = Lp;
    plan->suffix.chunk_base = plan->prefix_chunks;
    plan->suffix.part_stride = plan->prefix_chunks + plan->suffix.num_chunks;
    return CKL_OK;
}

size_t ckl_cascade_workspace_size(const ckl_cascade_plan_t* plan) {
    if (!plan) return 0;
    if (!plan->use) return ckl_decode_workspace_size(&plan->suffix);
    const ckl_decode_params& s = plan->suffix;
    return attn::part_o_bytes(&s) + align_up((size_t)s.B * s.Hq * s.part_stride * sizeof(float), 256);
}

ckl_status ckl_cascade_prefix(const ckl_cascade_plan_t* plan, float* part_o, float* part_lse,
                              void* stream) {
    ckl_status st = check_plan(plan);
    if (st != CKL_OK) return st;
    if (!plan->use) return fail(CKL_INVALID_ARG, "cascade_prefix: plan has no shared prefix");
    int G = 0;
    st = attn::validate(&plan->suffix, &G);
    if (st != CKL_OK || plan->suffix.B == 0) return st;
    if (!part_o || !part_lse) return fail(CKL_INVALID_ARG, "cascade_prefix: NULL partials");
    return launch_prefix(plan, part_o, part_lse, (cudaStream_t)stream);
}

int ckl_prefix_tree(const int* ip, const int* ix, int B, int min_pages, int* perm, int* nodes,
                    int* start_pages) {
    if (!ip || B < 0 || (B > 0 && (!ix || !perm || !start_pages)) || (B > 1 && !nodes)) return -1;
    for (int b = 0; b < B; b++)
        if (ip[b + 1] < ip[b]) return -1;
    min_pages = std::max(1, min_pages);
    // key of b: its page ids but the last (which stays private)
    auto klen = [&](int b) { return std::max(0, ip[b + 1] - ip[b] - 1); };
    std::vector<int> order(B);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
        const int lx = klen(x), ly = klen(y), n = std::min(lx, ly);
        for (int i = 0; i < n; i++) {
            const int px = ix[ip[x] + i], py = ix[ip[y] + i];
            if (px != py) return px < py;
        }
        return lx < ly;
    });
    for (int i = 0; i < B; i++) {
        perm[i] = order[i];
        start_pages[i] = 0;
    }
    if (B < 2) return 0;
    auto lcp = [&](int x, int y) {
        const int n = std::min(klen(x), klen(y));
        int i = 0;
        while (i < n && ix[ip[x] + i] == ix[ip[y] + i]) i++;
        return i;
    };
    // Every interval [lb, rb] of sorted positions whose keys share their first l > 0 pages
    // (and that no longer run extends) is a trie node; one stack pass over the adjacent
    // common-prefix lengths finds them all with their parents.
    struct Iv { int l, lb, rb, parent; };
    struct Open { int l, lb, id; };
    std::vector<Iv> iv;
    std::vector<Open> stk{{0, 0, -1}};
    for (int i = 1; i <= B; i++) {
        const int cur = i < B ? lcp(order[i - 1], order[i]) : 0;
        int lb = i - 1, last = -1;
        while (cur < stk.back().l) {
            const Open top = stk.back();
            stk.pop_back();
            iv[top.id].rb = i - 1;
            lb = top.lb;
            last = top.id;
            if (cur <= stk.back().l) {
                iv[last].parent = stk.back().id;
                last = -1;
            }
        }
        if (cur > stk.back().l) {
            const int id = (int)iv.size();
            iv.push_back({cur, lb, -1, -1});
            if (last >= 0) iv[last].parent = id;
            stk.push_back({cur, lb, id});
        }
    }
    // parents before children; keep nodes whose own run (from the nearest kept ancestor) is
    // long enough
    std::vector<int> pre((size_t)iv.size());
    std::iota(pre.begin(), pre.end(), 0);
    std::sort(pre.begin(), pre.end(), [&](int x, int y) {
        return iv[x].lb != iv[y].lb ? iv[x].lb < iv[y].lb : iv[x].rb > iv[y].rb;
    });
    std::vector<int> out_id(iv.size(), -1), kept_anc(iv.size(), -1);
    int n = 0;
    for (int id : pre) {
        const int par = iv[id].parent;
        kept_anc[id] = par < 0 ? -1 : (out_id[par] >= 0 ? par : kept_anc[par]);
        const int first = kept_anc[id] < 0 ? 0 : iv[kept_anc[id]].l;
        if (iv[id].l - first < min_pages) continue;
        out_id[id] = n;
        int* nd = nodes + 5 * n;
        nd[0] = first;
        nd[1] = iv[id].l;
        nd[2] = iv[id].lb;
        nd[3] = iv[id].rb + 1;
        nd[4] = kept_anc[id] < 0 ? -1 : out_id[kept_anc[id]];
        for (int i = iv[id].lb; i <= iv[id].rb; i++) start_pages[order[i]] = iv[id].l;
        n++;
    }
    return n;
}

ckl_status ckl_cascade_tree_plan(const ckl_decode_params* base, const int* h_indptr,
                                 const int* h_indices, const int* h_lens, int min_prefix,
                                 ckl_cascade_tree_plan_t* plan, void* tables, size_t table_bytes) {
    if (!plan || !base || !h_indptr || !h_indices || !h_lens)
        return fail(CKL_INVALID_ARG, "cascade_tree_plan: NULL");
    int G = 0;
    ckl_status st = attn::validate(base, &G);
    if (st != CKL_OK) return st;
    *plan = ckl_cascade_tree_plan_t{};
    plan->suffix = *base;
    const int B = base->B;
    std::vector<int> perm(std::max(B, 1)), nodes(5 * (size_t)std::max(B - 1, 1)), start(std::max(B, 1));
    const int n = ckl_prefix_tree(h_indptr, h_indices, B, ceil_div(std::max(min_prefix, 1), PAGE),
                                  perm.data(), nodes.data(), start.data());
    if (n < 0) return fail(CKL_INVALID_ARG, "cascade_tree_plan: bad page table");
    int max_len = 0;
    for (int b = 0; b < B; b++) max_len = std::max(max_len, h_lens[b]);
    if (n == 0) {
        plan->use = 0;
        st = ckl_decode_plan(G, B, base->Hkv, max_len, 0, &plan->suffix.num_chunks,
                             &plan->suffix.chunk_tokens);
        plan->suffix.kv_start = 0;
        plan->suffix.chunk_base = 0;
        plan->suffix.part_stride = plan->suffix.num_chunks;
        return st;
    }
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    const PrefixSetup* ps = setup(di);
    if (ps->st != CKL_OK) return ps->st;
    // about one wave of prefix CTAs over all nodes, >= 16 pages (256 tokens) per work item
    long long work = 0;
    for (int i = 0; i < n; i++) {
        const int* nd = &nodes[5 * i];
        work += (long long)(nd[1] - nd[0]) * ceil_div((nd[3] - nd[2]) * G, PROWS);
    }
    const long long target = std::max(1LL, (long long)di->sms * std::max(1, ps->per_sm) / base->Hkv);
    const int cp = (int)std::max(16LL, (work + target - 1) / target);
    // slots: a node's chunks follow its kept ancestors' chunks
    std::vector<int> nchunks(n), slot0(n);
    int items = 0;
    for (int i = 0; i < n; i++) {
        const int* nd = &nodes[5 * i];
        nchunks[i] = ceil_div(nd[1] - nd[0], cp);
        slot0[i] = nd[4] < 0 ? 0 : slot0[nd[4]] + nchunks[nd[4]];
        items += nchunks[i] * ceil_div((nd[3] - nd[2]) * G, PROWS);
    }
    // per sequence: first suffix slot = end of its deepest node's slots
    std::vector<int> suffix_slot(B, 0);
    for (int i = 0; i < n; i++) {
        const int* nd = &nodes[5 * i];
        for (int m = nd[2]; m < nd[3]; m++) suffix_slot[perm[m]] = slot0[i] + nchunks[i];
    }
    int max_path = 0, max_suffix = 1;
    for (int b = 0; b < B; b++) {
        max_path = std::max(max_path, suffix_slot[b]);
        max_suffix = std::max(max_suffix, h_lens[b] - start[b] * PAGE);
    }
    plan->use = 1;
    plan->nodes = n;
    plan->items = items;
    plan->chunk_pages = cp;
    plan->max_path_slots = max_path;
    st = ckl_decode_plan(G, B, base->Hkv, max_suffix, 0, &plan->suffix.num_chunks,
                         &plan->suffix.chunk_tokens);
    if (st != CKL_OK) return st;
    plan->suffix.kv_start = 0;
    plan->suffix.chunk_base = 0;
    plan->suffix.part_stride = max_path + plan->suffix.num_chunks;
    const TreeTables tt = tree_tables(B, items);
    plan->table_bytes = tt.bytes;
    if (!tables || table_bytes < tt.bytes)
        return fail(CKL_WORKSPACE_TOO_SMALL, "cascade_tree_plan: tables need %zu bytes, got %zu",
                    tt.bytes, tables ? table_bytes : (size_t)0);
    uint8_t* tb = static_cast<uint8_t*>(tables);
    memset(tb, 0, tt.bytes);
    int* seq_tab = reinterpret_cast<int*>(tb);
    for (int b = 0; b < B; b++) {
        seq_tab[2 * b] = start[b] * PAGE;
        seq_tab[2 * b + 1] = suffix_slot[b];
    }
    memcpy(tb + tt.perm, perm.data(), (size_t)B * 4);
    int* it = reinterpret_cast<int*>(tb + tt.items);
    for (int i = 0; i < n; i++) {
        const int* nd = &nodes[5 * i];
        const int members = nd[3] - nd[2], run = nd[1] - nd[0];
        const int page0 = h_indptr[perm[nd[2]]] + nd[0];
        for (int c = 0; c < nchunks[i]; c++)
            for (int row0 = 0; row0 < members * G; row0 += PROWS) {
                it[0] = page0 + c * cp;
                it[1] = std::min(cp, run - c * cp);
                it[2] = nd[2];
                it[3] = members;
                it[4] = row0;
                it[5] = slot0[i] + c;
                it += 8;
            }
    }
    return CKL_OK;
}

size_t ckl_cascade_tree_workspace_size(const ckl_cascade_tree_plan_t* plan) {
    if (!plan) return 0;
    if (!plan->use) return ckl_decode_workspace_size(&plan->suffix);
    const ckl_decode_params& s = plan->suffix;
    return attn::part_o_bytes(&s) + align_up((size_t)s.B * s.Hq * s.part_stride * sizeof(float), 256);
}

ckl_status ckl_cascade_tree_prefix(const ckl_cascade_tree_plan_t* plan, const void* d_tables,
                                   float* part_o, float* part_lse, void* stream) {
    int G = 0;
    ckl_status st = check_tree_plan(plan, d_tables, &G);
    if (st != CKL_OK || plan->suffix.B == 0) return st;
    if (!part_o || !part_lse) return fail(CKL_INVALID_ARG, "cascade_tree_prefix: NULL partials");
    return launch_tree_prefix(plan, static_cast<const uint8_t*>(d_tables), part_o, part_lse,
                              (cudaStream_t)stream);
}

ckl_status ckl_cascade_tree_decode(const ckl_cascade_tree_plan_t* plan, const void* d_tables,
                                   void* out, float* lse, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    if (!plan) return fail(CKL_INVALID_ARG, "cascade tree plan is NULL");
    if (!plan->use)
        return ckl_decode_attention(&plan->suffix, out, lse, workspace, workspace_bytes, stream);
    const ckl_decode_params& sp = plan->suffix;
    int G = 0;
    ckl_status st = check_tree_plan(plan, d_tables, &G);
    if (st != CKL_OK || sp.B == 0) return st;
    if (!out || !lse) return fail(CKL_INVALID_ARG, "cascade_tree_decode: out/lse are NULL");
    if ((uintptr_t)out & 7) return fail(CKL_INVALID_ARG, "out needs 8-byte alignment");
    const size_t need = ckl_cascade_tree_workspace_size(plan);
    if (!workspace || workspace_bytes < need)
        return fail(CKL_WORKSPACE_TOO_SMALL, "cascade_tree_decode needs %zu workspace bytes, got %zu",
                    need, workspace_bytes);
    if ((uintptr_t)workspace & 255) return fail(CKL_INVALID_ARG, "workspace must be 256-byte aligned");
    const cudaStream_t s = (cudaStream_t)stream;
    const uint8_t* tables = static_cast<const uint8_t*>(d_tables);
    const int2* seq_tab = reinterpret_cast<const int2*>(tables);
    float* part_o = static_cast<float*>(workspace);
    float* part_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + attn::part_o_bytes(&sp));
    st = launch_tree_prefix(plan, tables, part_o, part_lse, s);
    if (st != CKL_OK) return st;
    st = attn::launch_partial(&sp, G, false, nullptr, nullptr, part_o, part_lse, s, 0, 0, true, seq_tab);
    if (st != CKL_OK) return st;
    return attn::launch_merge(part_o, part_lse, static_cast<__half*>(out), lse, sp.B * sp.Hq,
                              sp.part_stride, sp.Hq, sp.Hq, 0, seq_tab, sp.num_chunks, s);
}

ckl_status ckl_cascade_decode(const ckl_cascade_plan_t* plan, void* out, float* lse,
                              void* workspace, size_t workspace_bytes, void* stream) {
    ckl_status st = check_plan(plan);
    if (st != CKL_OK) return st;
    if (!plan->use)
        return ckl_decode_attention(&plan->suffix, out, lse, workspace, workspace_bytes, stream);
    int G = 0;
    st = attn::validate(&plan->suffix, &G);
    if (st != CKL_OK || plan->suffix.B == 0) return st;
    if (!out || !lse) return fail(CKL_INVALID_ARG, "cascade_decode: out/lse are NULL");
    const size_t need = ckl_cascade_workspace_size(plan);
    if (!workspace || workspace_bytes < need)
        return fail(CKL_WORKSPACE_TOO_SMALL, "cascade_decode needs %zu workspace bytes, got %zu",
                    need, workspace_bytes);
    if ((uintptr_t)workspace & 255) return fail(CKL_INVALID_ARG, "workspace must be 256-byte aligned");
    const cudaStream_t s = (cudaStream_t)stream;
    float* part_o = static_cast<float*>(workspace);
    float* part_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                               attn::part_o_bytes(&plan->suffix));
    st = launch_prefix(plan, part_o, part_lse, s);
    if (st != CKL_OK) return st;
    // the suffix writes other slots than the prefix: it runs alongside it (programmatic
    // dependent launch) and only its completion waits for the prefix; the merge waits for both
    st = attn::launch_partial(&plan->suffix, G, false, nullptr, nullptr, part_o, part_lse, s, 0, 0,
                              true);
    if (st != CKL_OK) return st;
    return ckl_merge_states(part_o, part_lse, out, lse, plan->suffix.B * plan->suffix.Hq,
                            plan->suffix.part_stride, stream);
}

}  // extern "C"
