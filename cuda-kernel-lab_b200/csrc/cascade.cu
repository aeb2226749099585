// cascade.cu -- shared-prefix (cascade) decode for sm_100a.
//
// Replaces shared_prefix_pages / plan_cascade / cascade_prefix / cascade_decode of the
// reference (01_decode_attention.cu:446-712). When every sequence of a batch starts with
// the same physical pages (prefix caching), the plain kernel reads those pages once per
// sequence. The cascade reads them once per kv head:
//
//   1. host: the longest run of physical pages every sequence starts with (each keeps >= 1
//      private page), from the caller's host copy of the page table;
//   2. prefix kernel: the B*G query rows that share a kv head are stacked into 128-row
//      tiles, the M of tcgen05.mma: a TMA producer streams the shared pages in 64-key blocks,
//      S = Q K^T and O += P V run on the tensor cores with S and O in tensor memory, and
//      eight softmax warps keep a single-pass online softmax (the reference makes two passes
//      because WMMA cannot rescale its accumulators; O in tensor memory can be);
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

// The prefix kernel on the 5th-generation tensor cores. A CTA owns PROWS = 128 stacked
// query rows of one kv head (the M of tcgen05.mma) and streams a run of shared pages in
// blocks of BLK_PAGES pages (64 keys):
//   S = Q K^T   M=128, N=64, K=128: Q (K-major) and the block's K rows (K-major) in shared
//               memory, S in tensor memory (two buffers, so block j+1's S overlaps block j's
//               softmax);
//   softmax     8 warps, two threads per row: half an S row from tensor memory each, the
//               online max / sum in registers, P = exp2(S * scale - m) as fp16 into shared
//               memory in the K-major swizzled layout of an MMA A operand;
//   O += P V    M=128, N=128, K=16 per page: P (K-major) and V (MN-major: dims contiguous)
//               in shared memory, O in tensor memory for the whole run.
// The running max moves lazily (only when a score exceeds it by 2^RESCALE_THRESHOLD); a
// move rescales the row's O in tensor memory after the previous P V has landed.
// Warp 0 lane 0 issues the TMA loads, warp 1 lane 0 the MMAs, warps 2-9 run the softmax:
// two threads per row (warps 2-5 keys 0-31 of a block and O dims 0-63, warps 6-9 the other
// halves), which share the row max through shared memory once per block.
constexpr int PROWS = 128;                    // stacked query rows per CTA (tcgen05 M)
constexpr int BLK_PAGES = 4;                  // pages per key block
constexpr int BLK_KEYS = BLK_PAGES * PAGE;    // 64 keys: the N of S = Q K^T
constexpr int SOFT = 256;                     // softmax threads: 2 per row
constexpr int PTHREADS = 64 + SOFT;
constexpr int PSTAGES = 5;                    // key blocks in flight (160 KB)
constexpr int KV_HALF = BLK_KEYS * 128;       // 64 keys x 64 dims fp16 = 8 KB
constexpr int BLK_BYTES = 4 * KV_HALF;        // K dims 0-63, K 64-127, V 0-63, V 64-127
constexpr int Q_BYTES = PROWS * D * 2;        // 32 KB: dims 0-63 then 64-127
constexpr int P_BYTES = PROWS * BLK_KEYS * 2; // 16 KB per buffer
constexpr int PBUF = 1;                       // P buffers (one: the ring gets the room)
constexpr int P_OFF_Q = 0;
constexpr int P_OFF_RING = Q_BYTES;
constexpr int P_OFF_P = P_OFF_RING + PSTAGES * BLK_BYTES;
constexpr int P_OFF_RED = P_OFF_P + PBUF * P_BYTES;   // [max parity 0, 1; sums][2 halves][128 rows]
constexpr int P_OFF_BAR = P_OFF_RED + 3 * 2 * PROWS * 4;
constexpr int P_NBAR = 2 * PSTAGES + 4 * 2 + 3;
constexpr int P_SMEM = 1024 + P_OFF_BAR + P_NBAR * 8 + 16;
constexpr uint32_t P_TMEM_COLS = 256;         // S buffers at columns 0 and 64, O at 128

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
    int B, Hq, Hkv, G, prefix_len, chunk_tokens, part_stride, num_pages;
    float scale_log2;
};

// Byte offset of 16-byte chunk c (dims/keys 8c..8c+7 of a 128-byte row) of row r in a
// K-major, 128-byte-swizzled operand whose rows are 128 bytes apart (1024-byte aligned).
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

// grid = (prefix chunks, ceil(B*G / 128), Hkv). Writes the normalised partial (o, lse) of
// every stacked query row it covers into slot blockIdx.x. Prefix-tree mode: grid = (work
// items, 1, Hkv); item x covers a run of pages shared by the sequences perm[m0, m0 + members)
// and its stacked rows [row0, row0 + 128) of members x G, written into the item's slot.
__global__ void __launch_bounds__(PTHREADS, 1)
cascade_prefix_kernel(const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const PrefixArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = align_ptr<1024>(smem_raw);
    uint8_t* qs = sm + P_OFF_Q;
    uint8_t* ring = sm + P_OFF_RING;
    uint8_t* ps = sm + P_OFF_P;
    float* red = reinterpret_cast<float*>(sm + P_OFF_RED);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + P_OFF_BAR);
    uint64_t* empty = full + PSTAGES;
    uint64_t* s_full = empty + PSTAGES;       // S buffer b written (MMA -> softmax)
    uint64_t* s_empty = s_full + 2;           // S buffer b read (softmax -> MMA)
    uint64_t* p_full = s_empty + 2;           // P buffer written (softmax -> MMA)
    uint64_t* p_empty = p_full + PBUF;        // P buffer consumed (MMA -> softmax)
    uint64_t* o_done = p_empty + PBUF;        // one phase per P V block
    uint64_t* q_full = o_done + 1;            // Q staged (softmax -> MMA)
    uint64_t* done = q_full + 1;              // every issued MMA finished
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

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
    const int nblk = (npg + BLK_PAGES - 1) / BLK_PAGES;

    if (threadIdx.x == 0) {
        for (int s = 0; s < PSTAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&s_full[b], 1);
            mbar_init(&s_empty[b], SOFT);
        }
        for (int b = 0; b < PBUF; b++) {
            mbar_init(&p_full[b], SOFT);
            mbar_init(&p_empty[b], 1);
        }
        mbar_init(o_done, 1);
        mbar_init(q_full, SOFT);
        mbar_init(done, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, P_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint64_t deadline = globaltimer() + a.timeout_ns;
    pdl_trigger();                   // the suffix kernel (independent slots) may start now

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
        }
        // the prefix is re-read by the other query tiles of this kv head: keep it in L2
        const uint64_t pol = policy_evict_last();
        int ok = 1, issued = 0;
        int ids_at = -32, my_id = 0;     // page ids [ids_at, ids_at + 32): lane l holds one
        for (int j = 0; j < nblk && ok; j++) {
            const int s = j % PSTAGES;
            // the run's page ids, 32 per warp-wide load (one load per 8 blocks, not a
            // dependent load per block); a page past the run reads as zeros (its coordinate
            // is past the tensor map's page extent)
            const int p0 = j * BLK_PAGES;
            if (p0 >= ids_at + 32) {
                ids_at = p0 & ~31;
                my_id = ids_at + lane < npg ? __ldg(pages + ids_at + lane) : a.num_pages;
            }
            const int my_page = __shfl_sync(0xffffffffu, my_id, (p0 & 31) + (lane & (BLK_PAGES - 1)));
            if (lane == 0) {
                if (j >= PSTAGES) ok = mbar_wait(&empty[s], ((j / PSTAGES) - 1) & 1, deadline, a.err);
                if (ok) mbar_arrive_expect_tx(&full[s], BLK_BYTES);
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            uint8_t* st = ring + (size_t)s * BLK_BYTES;
            if (lane < BLK_PAGES) {
                uint8_t* dst = st + lane * (PAGE * 128);
                tma_load_4d(dst, &tmK, 0, kvh, 0, my_page, &full[s], pol);
                tma_load_4d(dst + KV_HALF, &tmK, 64, kvh, 0, my_page, &full[s], pol);
                tma_load_4d(dst + 2 * KV_HALF, &tmV, 0, kvh, 0, my_page, &full[s], pol);
                tma_load_4d(dst + 3 * KV_HALF, &tmV, 64, kvh, 0, my_page, &full[s], pol);
            }
            issued = j + 1;
        }
        // every issued copy must land before the CTA exits
        if (lane == 0)
            for (int s = 0; s < PSTAGES && s < issued; s++) {
                const int last = s + ((issued - 1 - s) / PSTAGES) * PSTAGES;
                mbar_wait(&full[s], (last / PSTAGES) & 1, deadline, a.err);
            }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc_s = umma_idesc_f16(PROWS, BLK_KEYS, false, false);
            const uint32_t idesc_o = umma_idesc_f16(PROWS, D, false, true);
            const uint32_t qa = smem_u32(qs), pa = smem_u32(ps), ra = smem_u32(ring);
            bool ok = mbar_wait(q_full, 0, deadline, a.err);
            // O += P V of block i: one K=16 MMA per page. V is MN-major: its 64-dim atoms
            // (dims 0-63, 64-127) KV_HALF apart, 8-key groups 1 KB apart.
            auto pv = [&](int i) {
                const int s = i % PSTAGES, b = i % PBUF;
                if (!mbar_wait(&p_full[b], (i / PBUF) & 1, deadline, a.err)) return false;
                tc_fence_after_sync();
                const uint32_t vb = ra + (uint32_t)(s * BLK_BYTES + 2 * KV_HALF);
#pragma unroll
                for (int pg = 0; pg < BLK_PAGES; pg++) {
                    const uint64_t ad = umma_desc_sw128(pa + b * P_BYTES + pg * 32, 16, 1024);
                    const uint64_t bd = umma_desc_sw128(vb + pg * (PAGE * 128), KV_HALF, 1024);
                    umma_f16(tmem + 128, ad, bd, idesc_o, (i | pg) != 0);
                }
                umma_commit(&empty[s]);      // K/V block free
                umma_commit(&p_empty[b]);    // P buffer free
                umma_commit(o_done);         // O holds blocks 0..i
                return true;
            };
            if (ok) tc_fence_after_sync();
            for (int j = 0; j < nblk && ok; j++) {
                const int s = j % PSTAGES, b = j & 1;
                ok = mbar_wait(&full[s], (j / PSTAGES) & 1, deadline, a.err);
                if (ok && j >= 2) ok = mbar_wait(&s_empty[b], ((j >> 1) - 1) & 1, deadline, a.err);
                if (!ok) break;
                tc_fence_after_sync();
                const uint32_t kb = ra + (uint32_t)(s * BLK_BYTES);
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    // k step of 16 dims = 32 bytes inside the swizzled row; dims 64-127 in the
                    // second half (Q: 16 KB on, K: KV_HALF on)
                    const uint64_t ad = umma_desc_sw128(qa + (kk >> 2) * (Q_BYTES / 2) + (kk & 3) * 32, 16, 1024);
                    const uint64_t bd = umma_desc_sw128(kb + (kk >> 2) * KV_HALF + (kk & 3) * 32, 16, 1024);
                    umma_f16(tmem + b * BLK_KEYS, ad, bd, idesc_s, kk != 0);
                }
                umma_commit(&s_full[b]);
                if (j >= 1) ok = pv(j - 1);
            }
            if (ok && nblk > 0) pv(nblk - 1);
            umma_commit(done);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------------- softmax warps
        const int quarter = warp & 3;                      // TMEM lanes 32*quarter..+31
        const int hf = (warp - 2) >> 2;                    // which half of the row
        const int r = quarter * 32 + lane;                 // this thread's row of the tile
        const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
        const int rr = row0 + r;                           // stacked row within the run's rows
        const bool real = rr < nq;
        size_t qrow = 0;
        if (real) {
            const int seq = a.perm ? __ldg(a.perm + m0 + rr / a.G) : rr / a.G;
            qrow = (size_t)seq * a.Hq + (size_t)kvh * a.G + rr % a.G;
        }
        // stage this thread's half of the q row (zeros past the rows in use) in the swizzled
        // K-major layout
        {
            const uint4* src = reinterpret_cast<const uint4*>(a.q + qrow * D) + 8 * hf;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const uint4 v = real ? __ldg(src + c) : make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4*>(qs + hf * (Q_BYTES / 2) + sw128(r, c)) = v;
            }
        }
        fence_proxy_async_smem();                          // visible to the tensor core
        mbar_arrive(q_full);

        constexpr int HK = BLK_KEYS / 2;                   // keys of a block per thread
        float m = -INFINITY, l = 0.f;                      // l: this half's sum
        // ok is warp-uniform. After a timeout a warp keeps going round the loop without
        // waiting or computing, so that every softmax thread meets the named barrier the same
        // number of times (nblk + 1).
        bool ok = true;
        for (int j = 0; j < nblk; j++) {
            const int b = j & 1;
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&s_full[b], (j >> 1) & 1, deadline, a.err));
            float sv[HK];
            float mx = -INFINITY;
            if (ok) {
                tc_fence_after_sync();
                uint32_t v[32];
                tmem_ld32(trow + b * BLK_KEYS + hf * HK, v);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < HK; i++) sv[i] = __uint_as_float(v[i]);
                tc_fence_before_sync();
                mbar_arrive(&s_empty[b]);
                const int kbase = j * BLK_KEYS + hf * HK;
                if (kbase + HK > kend) {
#pragma unroll
                    for (int c = 0; c < HK; c++)
                        if (kbase + c >= kend) sv[c] = -INFINITY;
                }
#pragma unroll
                for (int c = 0; c < HK; c++) mx = fmaxf(mx, sv[c]);
                mx *= a.scale_log2;                        // scale > 0: max of the scaled row
            }
            // the row max across both halves
            float* rm = red + b * 2 * PROWS;
            rm[hf * PROWS + r] = mx;
            asm volatile("bar.sync 1, %0;" ::"n"(SOFT) : "memory");
            mx = fmaxf(mx, rm[(hf ^ 1) * PROWS + r]);
            if (!ok) continue;
            const bool need = mx > m + RESCALE_THRESHOLD;
            if (__any_sync(0xffffffffu, need)) {
                const float mn = need ? fmaxf(m, mx) : m;
                const float cf = ex2(m - mn);              // 0 when m = -inf, 1 when unchanged
                if (j > 0) {
                    // O holds blocks 0..j-1 once their P V has landed: rescale this half there
                    ok = __all_sync(0xffffffffu, mbar_wait(o_done, (j - 1) & 1, deadline, a.err));
                    if (!ok) continue;
                    tc_fence_after_sync();
#pragma unroll
                    for (int c0 = 0; c0 < D / 2; c0 += 32) {
                        uint32_t v[32];
                        tmem_ld32(trow + 128 + hf * (D / 2) + c0, v);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; i++) v[i] = __float_as_uint(__uint_as_float(v[i]) * cf);
                        tmem_st32(trow + 128 + hf * (D / 2) + c0, v);
                    }
                    tmem_st_wait();
                    tc_fence_before_sync();
                }
                l *= cf;
                m = mn;
            }
            // P: fp16 exp2(s * scale - m), 8 keys per 16-byte chunk, swizzled
            const int pb = j % PBUF;
            if (j >= PBUF) {
                ok = __all_sync(0xffffffffu, mbar_wait(&p_empty[pb], ((j / PBUF) - 1) & 1, deadline, a.err));
                if (!ok) continue;
            }
            uint8_t* prow = ps + pb * P_BYTES;
            const float nm = -m;
#pragma unroll
            for (int c = 0; c < HK / 8; c++) {
                uint32_t w[4];
#pragma unroll
                for (int h = 0; h < 4; h++) {
                    const float p0 = ex2(fmaf(sv[8 * c + 2 * h], a.scale_log2, nm));
                    const float p1 = ex2(fmaf(sv[8 * c + 2 * h + 1], a.scale_log2, nm));
                    l += p0 + p1;
                    w[h] = pack_half2(p0, p1);
                }
                *reinterpret_cast<uint4*>(prow + sw128(r, hf * (HK / 8) + c)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
            fence_proxy_async_smem();
            mbar_arrive(&p_full[pb]);
        }
        // epilogue: this half of the O row / l, and the lse, into the partial slot
        if (ok && nblk > 0) ok = __all_sync(0xffffffffu, mbar_wait(o_done, (nblk - 1) & 1, deadline, a.err));
        const bool good = ok && nblk > 0;
        // the sums of the two halves (every softmax thread reaches this barrier once)
        float* rl = red + 4 * PROWS;
        rl[hf * PROWS + r] = l;
        asm volatile("bar.sync 1, %0;" ::"n"(SOFT) : "memory");
        l += rl[(hf ^ 1) * PROWS + r];
        if (good) {
            tc_fence_after_sync();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            const size_t pslot = qrow * a.part_stride + slot;
            float4* dst = reinterpret_cast<float4*>(a.part_o + pslot * D + hf * (D / 2));
#pragma unroll
            for (int c0 = 0; c0 < D / 2; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(trow + 128 + hf * (D / 2) + c0, v);
                tmem_ld_wait();
                if (real) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        dst[(c0 + i) / 4] = make_float4(__uint_as_float(v[i]) * inv, __uint_as_float(v[i + 1]) * inv,
                                                        __uint_as_float(v[i + 2]) * inv, __uint_as_float(v[i + 3]) * inv);
                }
            }
            if (real && hf == 0) a.part_lse[pslot] = l > 0.f ? (m + lg2(l)) * LN2 : -INFINITY;
        } else if (nblk == 0 && real) {                    // an empty run: no keys
            const size_t pslot = qrow * a.part_stride + slot;
            for (int c = 0; c < D / 2; c++) a.part_o[pslot * D + hf * (D / 2) + c] = 0.f;
            if (hf == 0) a.part_lse[pslot] = -INFINITY;
        }
    }
    // every MMA must have finished before tensor memory is released
    if (threadIdx.x == 0) mbar_wait(done, 0, deadline, a.err);
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    if (warp == 1) tmem_dealloc(tmem, P_TMEM_COLS);
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
    a.num_pages = b.num_pages;
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
    a.num_pages = b.num_pages;
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
    if (base->B == 0) {                      // an empty batch: the decode call is a no-op
        plan->suffix.num_chunks = plan->suffix.part_stride = 1;
        plan->suffix.chunk_tokens = 32;
        plan->suffix.kv_start = plan->suffix.chunk_base = 0;
        return CKL_OK;
    }
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
    if (B == 0) {                            // an empty batch: the decode call is a no-op
        plan->suffix.num_chunks = plan->suffix.part_stride = 1;
        plan->suffix.chunk_tokens = 32;
        plan->suffix.kv_start = plan->suffix.chunk_base = 0;
        return CKL_OK;
    }
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
    // the smallest chunk that keeps every work item in the one wave (a partial second wave
    // would double the prefix time)
    auto items_for = [&](int c) {
        long long it = 0;
        for (int i = 0; i < n; i++) {
            const int* nd = &nodes[5 * i];
            it += (long long)ceil_div(nd[1] - nd[0], c) * ceil_div((nd[3] - nd[2]) * G, PROWS);
        }
        return it;
    };
    int cp = (int)std::max(16LL, (work + target - 1) / target);
    int max_run = 1;
    for (int i = 0; i < n; i++) max_run = std::max(max_run, nodes[5 * i + 1] - nodes[5 * i]);
    while (cp < max_run && items_for(cp) > target) cp++;
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
