// decode_attention.cu -- paged split-KV GQA decode attention for sm_100a.
//
// Replaces decode_partial<G,V> / merge_states / plan_chunks / decode_attention of the
// reference (01_decode_attention.cu:77-331) with a B200-native design:
//
//   * One CTA per (sequence b, kv head, chunk). Warp 4 is a producer: it reads the chunk's
//     page ids and issues TMA tiled loads (cp.async.bulk.tensor.4d, 128B swizzle, evict-
//     first L2 hint) of whole pages -- 16 keys x 128 dims of K and of V for this head, 4 KB
//     each -- into an 8-stage shared-memory ring guarded by full/empty mbarriers. 64 KB are
//     in flight per CTA, two CTAs per SM.
//   * Warps 0..3 consume pages round-robin. Per page a warp computes S = Q K^T for its G
//     query heads (the GQA group, padded to the 16 rows of an m16n8k16 tile) with
//     mma.sync (K fragments by ldmatrix from the swizzled tile, q fragments held in
//     registers), an online softmax in the log2 domain with a lazy rescale, and O += P V
//     (V fragments by ldmatrix.trans). Tensor-core math leaves the kernel bound by HBM:
//     per 16-key page a warp issues 32 MMAs and 16 ldmatrix, against ~700 warp
//     instructions for the reference's CUDA-core dot products.
//   * The four warps' (m, l, O) states are merged through shared memory; a single-chunk
//     launch writes the final fp16 out and lse directly, otherwise normalised fp32 partials
//     (o, lse) go to the caller's workspace for the LSE merge kernel.
//
// Page-table convention (01_decode_attention.cu:5-9, 93-95, 111-112): seq_len =
// (npages-1)*16 + last_page_len, key -> page kv_indices[indptr[b] + key/16], element
// ((page*16 + key%16)*Hkv + kvh)*128 + d.

#include <cmath>
#include <cstring>
#include <mutex>

#include "attn_common.cuh"

namespace ckl {
namespace attn {

constexpr int CONSUMERS = 4;
constexpr int THREADS = (CONSUMERS + 1) * 32;
constexpr int STAGES = 8;
// Consumer warp w takes pages i = w (mod CONSUMERS) from stage i % STAGES: each stage then has
// one consumer warp, which meets its phases in order (the parity waits rely on it).
static_assert(STAGES % CONSUMERS == 0, "every stage must belong to one consumer warp");
constexpr int RING_BYTES = STAGES * STAGE_BYTES;
constexpr int BAR_BYTES = 2 * STAGES * 8;
constexpr int RED_BYTES = 2 * CONSUMERS * 16 * 4;
constexpr int SMEM_BYTES = 1024 /*alignment slack*/ + RING_BYTES + BAR_BYTES + RED_BYTES;

struct Args {
    const __half* q;
    const int* indptr;
    const int* indices;
    const int* last;
    float* part_o;
    float* part_lse;
    __half* out;
    float* lse;
    unsigned* err;
    unsigned long long timeout_ns;
    int B, Hq, Hkv, chunk_tokens, kv_start, chunk_base, part_stride, direct;
    int out_heads, head_offset;   // direct mode: row (b, h) goes to out row b*out_heads + head_offset + h
    const int2* seq_tab;          // per sequence {kv_start, chunk_base}; NULL: the uniform fields
    float scale_log2;
    // launched early behind the previous kernel of the stream (programmatic dependent launch):
    // 1 = wait for it before reading any input (the general case: it may have written q, the
    // page table or the caches); 0 = the inputs are older, wait only before completing;
    // 2 = the page table and every page but each sequence's last are older: the producer
    // issues the ring's first pages (last pages excluded) before it waits, every other read
    // and every write waits
    int wait_first;
};

template <int G>
__global__ void __launch_bounds__(THREADS, 2)
decode_partial_kernel(const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const Args a) {
    static_assert(G == 1 || G == 2 || G == 4 || G == 8 || G == 16, "GQA group size");
    constexpr bool HI = G > 8;   // rows 8..15 of the MMA tile carry query heads too

    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = align_ptr<1024>(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + RING_BYTES);
    uint64_t* empty = full + STAGES;
    float* m_red = reinterpret_cast<float*>(empty + STAGES);   // [CONSUMERS][16]
    float* l_red = m_red + CONSUMERS * 16;                      // [CONSUMERS][16]

    const int bh = blockIdx.x, chunk = blockIdx.y;
    const int b = bh / a.Hkv, kvh = bh - b * a.Hkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_barrier_init();
    }
    if (warp == CONSUMERS && lane == 0) {
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    __syncthreads();
    // the set-up above overlapped the previous kernel's tail; in mode 2 the producer waits
    // later, after the first pages are in flight
    if (a.wait_first == 1 || (a.wait_first == 2 && warp != CONSUMERS)) pdl_wait();
    const uint64_t deadline = globaltimer() + a.timeout_ns;
    pdl_trigger();                   // a merge launched after us may be scheduled now

    const int page_beg = __ldg(a.indptr + b);
    const int npages = __ldg(a.indptr + b + 1) - page_beg;
    const int seq_len = npages > 0 ? (npages - 1) * PAGE + __ldg(a.last + b) : 0;
    const int kv_start = a.seq_tab ? __ldg(&a.seq_tab[b].x) : a.kv_start;
    const int kbeg = kv_start + chunk * a.chunk_tokens;         // multiple of 16
    const int kend = min(seq_len, kbeg + a.chunk_tokens);
    const int p0 = kbeg / PAGE;
    const int npg = kend > kbeg ? (kend - kbeg + PAGE - 1) / PAGE : 0;

    // consumer state (unused by the producer warp)
    HeadState<G> hs;
    const int g = lane >> 2, t = lane & 3;

    if (warp == CONSUMERS) {
        // ---------------------------------------------------------------- producer warp
        const uint64_t pol = policy_evict_first();
        int ok = 1, issued = 0;
        bool waited = a.wait_first != 2;
        for (int base = 0; base < npg && ok; base += 32) {
            const int cnt = min(32, npg - base);
            const int my_page = lane < cnt ? __ldg(a.indices + page_beg + p0 + base + lane) : 0;
            for (int j = 0; j < cnt; j++) {
                const int page = __shfl_sync(0xffffffffu, my_page, j);
                // mode 2: a sequence's last page (the previous kernel may append to it) and
                // anything past the ring's first fill come after the wait
                if (!waited && (base + j >= STAGES || p0 + base + j == npages - 1)) {
                    pdl_wait();
                    waited = true;
                }
                if (lane == 0) {
                    const int i = base + j, s = i % STAGES;
                    if (i >= STAGES) ok = mbar_wait(&empty[s], ((i / STAGES) - 1) & 1, deadline, a.err);
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
        if (!waited) pdl_wait();     // before the outputs this warp helps write
        // Every issued copy must land before the CTA reuses the ring or exits.
        if (lane == 0) {
            for (int s = 0; s < STAGES && s < issued; s++) {
                const int i_last = s + ((issued - 1 - s) / STAGES) * STAGES;
                mbar_wait(&full[s], (i_last / STAGES) & 1, deadline, a.err);
            }
        }
    } else {
        // ---------------------------------------------------------------- consumer warps
        hs.load_q(a.q + ((size_t)b * a.Hq + (size_t)kvh * G) * D, lane);
        hs.reset();
        bool ok = true;
        for (int i = warp; i < npg; i += CONSUMERS) {
            const int s = i % STAGES;
            const bool got = mbar_wait(&full[s], (i / STAGES) & 1, deadline, a.err);
            if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
            hs.page(smem_u32(ring + s * STAGE_BYTES), (p0 + i) * PAGE, kend, a.scale_log2, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        hs.reduce_l();
        if (!ok) { hs.m_lo = hs.m_hi = -INFINITY; hs.l_lo = hs.l_hi = 0.f; }
        if (t == 0) {
            m_red[warp * 16 + g] = hs.m_lo;
            l_red[warp * 16 + g] = hs.l_lo;
            if (HI) {
                m_red[warp * 16 + g + 8] = hs.m_hi;
                l_red[warp * 16 + g + 8] = hs.l_hi;
            }
        }
    }
    // All consumers are done with the ring and the producer has seen every copy land:
    // the ring can hold the per-warp O states.
    __syncthreads();
    if (warp < CONSUMERS) {
        float* ost = reinterpret_cast<float*>(ring);   // [CONSUMERS][G][128]
        if (g < G) {
#pragma unroll
            for (int j = 0; j < 16; j++) {
                float* dst = ost + ((size_t)warp * G + g) * D + 8 * j + 2 * t;
                dst[0] = hs.o[j][0];
                dst[1] = hs.o[j][1];
            }
        }
        if (HI && g + 8 < G) {
#pragma unroll
            for (int j = 0; j < 16; j++) {
                float* dst = ost + ((size_t)warp * G + g + 8) * D + 8 * j + 2 * t;
                dst[0] = hs.o[j][2];
                dst[1] = hs.o[j][3];
            }
        }
    }
    __syncthreads();

    // ---------------------------------------------------------------- merge the 4 warps
    const float* ost = reinterpret_cast<const float*>(ring);
    for (int idx = threadIdx.x; idx < G * D; idx += THREADS) {
        const int gq = idx / D, d = idx - gq * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < CONSUMERS; w++) M = fmaxf(M, m_red[w * 16 + gq]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < CONSUMERS; w++) {
                const float sw = ex2(m_red[w * 16 + gq] - M);
                L += l_red[w * 16 + gq] * sw;
                O += ost[((size_t)w * G + gq) * D + d] * sw;
            }
        }
        const bool has = L > 0.f;
        const float val = has ? O / L : 0.f;
        const float lse_v = has ? (M + lg2(L)) * LN2 : -INFINITY;
        const size_t row = (size_t)b * a.Hq + (size_t)kvh * G + gq;
        if (a.direct) {
            const size_t orow = (size_t)b * a.out_heads + a.head_offset + (size_t)kvh * G + gq;
            a.out[orow * D + d] = __float2half_rn(val);
            if (d == 0) a.lse[orow] = lse_v;
        } else {
            const int cbase = a.seq_tab ? __ldg(&a.seq_tab[b].y) : a.chunk_base;
            const size_t slot = row * a.part_stride + cbase + chunk;
            a.part_o[slot * D + d] = val;
            if (d == 0) a.part_lse[slot] = lse_v;
        }
    }
    // launched dependent on another kernel (the cascade's suffix after its prefix): do not
    // complete before it, so that a kernel waiting on us has both kernels' partials
    pdl_wait();
}

// LSE merge: one warp per (sequence, q head) row, 4 dims per lane (16-byte loads). Row
// r = b*Hq + h is written to out row b*out_heads + head_offset + h (identity when
// out_heads = Hq and head_offset = 0; a head shard of a wider, possibly peer-mapped, output
// otherwise). Rows are `stride` slots apart; a row of sequence b merges its first
// seq_tab[b].y + tail slots (the prefix-tree cascade, whose sequences own different numbers
// of slots), or all `stride` when seq_tab is NULL.
__global__ void __launch_bounds__(256)
merge_states_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                    __half* __restrict__ out, float* __restrict__ lse_out, int rows, int stride,
                    int Hq, int out_heads, int head_offset, const int2* __restrict__ seq_tab,
                    int tail) {
    pdl_wait();                      // partials of the kernel(s) before us
    pdl_trigger();                   // the next call's kernels may start their set-up
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int b = row / Hq;
    const size_t orow = (size_t)b * out_heads + head_offset + row % Hq;
    const int slots = seq_tab ? min(stride, seq_tab[b].y + tail) : stride;
    const float* L = part_lse + (size_t)row * stride;
    float m = -INFINITY;
    for (int c = lane; c < slots; c += 32) m = fmaxf(m, L[c]);
    m = warp_max(m);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float wsum = 0.f;
    if (m != -INFINITY) {
        const float4* po = reinterpret_cast<const float4*>(part_o + (size_t)row * stride * D) + lane;
#pragma unroll 4
        for (int c = 0; c < slots; c++) {
            const float w = ex2((L[c] - m) * LOG2E);
            const float4 v = po[(size_t)c * (D / 4)];
            wsum += w;
            acc.x += w * v.x;
            acc.y += w * v.y;
            acc.z += w * v.z;
            acc.w += w * v.w;
        }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    __half2 h0 = __floats2half2_rn(acc.x * inv, acc.y * inv);
    __half2 h1 = __floats2half2_rn(acc.z * inv, acc.w * inv);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&h0);
    pk.y = *reinterpret_cast<uint32_t*>(&h1);
    reinterpret_cast<uint2*>(out + orow * D)[lane] = pk;
    if (lane == 0) lse_out[orow] = wsum > 0.f ? m + logf(wsum) : -INFINITY;
}

// The same merge for few rows with many slots (one long sequence split into dozens of chunks):
// one CTA per row, its 8 warps take slots c = w (mod 8) and the warps' sums are added in warp
// order, so a row's slots are read by 8 warps in parallel instead of one walking them all.
__global__ void __launch_bounds__(256)
merge_states_split_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                          __half* __restrict__ out, float* __restrict__ lse_out, int rows,
                          int stride, int Hq, int out_heads, int head_offset,
                          const int2* __restrict__ seq_tab, int tail) {
    __shared__ float4 s_acc[8][32];
    __shared__ float s_w[8];
    pdl_wait();                      // partials of the kernel(s) before us
    pdl_trigger();                   // the next call's kernels may start their set-up
    const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = row / Hq;
    const size_t orow = (size_t)b * out_heads + head_offset + row % Hq;
    const int slots = seq_tab ? min(stride, seq_tab[b].y + tail) : stride;
    const float* L = part_lse + (size_t)row * stride;
    float m = -INFINITY;
    for (int c = lane; c < slots; c += 32) m = fmaxf(m, L[c]);
    m = warp_max(m);                 // every warp finds the same row maximum
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float wsum = 0.f;
    if (m != -INFINITY) {
        const float4* po = reinterpret_cast<const float4*>(part_o + (size_t)row * stride * D) + lane;
#pragma unroll 4
        for (int c = warp; c < slots; c += 8) {
            const float w = ex2((L[c] - m) * LOG2E);
            const float4 v = po[(size_t)c * (D / 4)];
            wsum += w;
            acc.x += w * v.x;
            acc.y += w * v.y;
            acc.z += w * v.z;
            acc.w += w * v.w;
        }
    }
    s_acc[warp][lane] = acc;
    if (lane == 0) s_w[warp] = wsum;
    __syncthreads();
    if (warp != 0) return;
    acc = s_acc[0][lane];
    wsum = s_w[0];
#pragma unroll
    for (int w = 1; w < 8; w++) {
        const float4 v = s_acc[w][lane];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
        wsum += s_w[w];
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    __half2 h0 = __floats2half2_rn(acc.x * inv, acc.y * inv);
    __half2 h1 = __floats2half2_rn(acc.z * inv, acc.w * inv);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&h0);
    pk.y = *reinterpret_cast<uint32_t*>(&h1);
    reinterpret_cast<uint2*>(out + orow * D)[lane] = pk;
    if (lane == 0) lse_out[orow] = wsum > 0.f ? m + logf(wsum) : -INFINITY;
}

template <int G>
const void* kernel_for() { return reinterpret_cast<const void*>(decode_partial_kernel<G>); }

const void* pick(int G) {
    switch (G) {
        case 1: return kernel_for<1>();
        case 2: return kernel_for<2>();
        case 4: return kernel_for<4>();
        case 8: return kernel_for<8>();
        case 16: return kernel_for<16>();
    }
    return nullptr;
}

// Opt every partial kernel into its dynamic shared memory once per device, and record the
// resident CTAs per SM of each (used by the split heuristic).
struct KernelSetup {
    int per_sm[17] = {0};
    ckl_status st = CKL_OK;
};
const KernelSetup* setup(const DeviceInfo* di) {
    static KernelSetup ks[64];
    static std::once_flag once[64];
    std::call_once(once[di->device], [di] {
        KernelSetup& k = ks[di->device];
        for (int G : {1, 2, 4, 8, 16}) {
            const void* fn = pick(G);
            cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
            if (e == cudaSuccess)
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k.per_sm[G], fn, THREADS, SMEM_BYTES);
            if (e != cudaSuccess) {
                k.st = cuda_status(e, "decode kernel setup");
                return;
            }
        }
    });
    return &ks[di->device];
}

ckl_status validate(const ckl_decode_params* p, int* G) {
    if (!p) return fail(CKL_INVALID_ARG, "params is NULL");
    if (p->B < 0 || p->Hq <= 0 || p->Hkv <= 0 || p->Hq % p->Hkv)
        return fail(CKL_INVALID_ARG, "bad head counts B=%d Hq=%d Hkv=%d", p->B, p->Hq, p->Hkv);
    *G = p->Hq / p->Hkv;
    if (!pick(*G)) return fail(CKL_UNSUPPORTED_SHAPE, "unsupported GQA group size %d", *G);
    if (p->B == 0) return CKL_OK;
    if (!p->q || !p->k_cache || !p->v_cache || !p->kv_indptr || !p->kv_indices || !p->kv_last_page_len)
        return fail(CKL_INVALID_ARG, "NULL tensor pointer");
    if (((uintptr_t)p->k_cache | (uintptr_t)p->v_cache) & 15)
        return fail(CKL_INVALID_ARG, "k_cache/v_cache must be 16-byte aligned");
    if ((uintptr_t)p->q & 3) return fail(CKL_INVALID_ARG, "q must be 4-byte aligned");
    if (p->num_pages <= 0) return fail(CKL_INVALID_ARG, "num_pages must be > 0");
    if (p->num_chunks <= 0 || p->chunk_tokens <= 0 || p->chunk_tokens % PAGE)
        return fail(CKL_INVALID_ARG, "num_chunks=%d chunk_tokens=%d (must be >0, multiple of 16)",
                    p->num_chunks, p->chunk_tokens);
    if (p->kv_start < 0 || p->kv_start % PAGE)
        return fail(CKL_INVALID_ARG, "kv_start=%d must be a non-negative multiple of 16", p->kv_start);
    if (p->chunk_base < 0 || p->part_stride < p->chunk_base + p->num_chunks)
        return fail(CKL_INVALID_ARG, "part_stride=%d < chunk_base=%d + num_chunks=%d",
                    p->part_stride, p->chunk_base, p->num_chunks);
    if ((long long)p->B * p->Hkv > 0x7fffffffLL || p->num_chunks > 65535)
        return fail(CKL_UNSUPPORTED_SHAPE, "grid too large");
    // partial slots per row are bounded like the chunk count, so the workspace size
    // (B * Hq * part_stride * 516 bytes) cannot wrap and no slot index leaves the buffer
    size_t bytes = 0;
    if (p->part_stride > 65535 ||
        __builtin_mul_overflow((size_t)p->B * (size_t)p->Hq, (size_t)p->part_stride * (D + 1) * sizeof(float), &bytes))
        return fail(CKL_UNSUPPORTED_SHAPE, "part_stride=%d (at most 65535 partial slots per row)",
                    p->part_stride);
    return CKL_OK;
}

ckl_status launch_partial(const ckl_decode_params* p, int G, bool direct, __half* out,
                          float* lse, float* part_o, float* part_lse, cudaStream_t stream,
                          int out_heads, int head_offset, bool pdl, const int2* seq_tab,
                          int wait_first) {
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    const KernelSetup* ks = setup(di);
    if (ks->st != CKL_OK) return ks->st;

    CUtensorMap tmK, tmV;
    ckl_status st = encode_page_maps(p->k_cache, p->v_cache, p->Hkv, p->num_pages, &tmK, &tmV);
    if (st != CKL_OK) return st;

    Args a;
    a.q = static_cast<const __half*>(p->q);
    a.indptr = p->kv_indptr;
    a.indices = p->kv_indices;
    a.last = p->kv_last_page_len;
    a.part_o = part_o;
    a.part_lse = part_lse;
    a.out = out;
    a.lse = lse;
    a.err = di->err_word;
    a.timeout_ns = spin_timeout_ns();
    a.B = p->B;
    a.Hq = p->Hq;
    a.Hkv = p->Hkv;
    a.chunk_tokens = p->chunk_tokens;
    a.kv_start = p->kv_start;
    a.chunk_base = p->chunk_base;
    a.part_stride = p->part_stride;
    a.direct = direct ? 1 : 0;
    a.out_heads = out_heads > 0 ? out_heads : p->Hq;
    a.head_offset = head_offset;
    a.seq_tab = seq_tab;
    a.scale_log2 = p->sm_scale * LOG2E;
    a.wait_first = wait_first;

    void* args[] = {&tmK, &tmV, &a};
    dim3 grid((unsigned)(p->B * p->Hkv), (unsigned)p->num_chunks);
    CKL_CUDA_TRY(launch(pick(G), grid, dim3(THREADS), SMEM_BYTES, stream, args, pdl));
    return CKL_OK;
}

ckl_status launch_merge(const float* part_o, const float* part_lse, __half* out, float* lse,
                        int rows, int stride, int Hq, int out_heads, int head_offset,
                        const int2* seq_tab, int tail, cudaStream_t stream) {
    void* args[] = {&part_o, &part_lse, &out, &lse, &rows, &stride, &Hq, &out_heads, &head_offset,
                    &seq_tab, &tail};
    // one warp per row unless that leaves the GPU nearly idle with long rows to walk
    const DeviceInfo* di = device_info();
    if (di && stride >= 16 && rows < 4 * di->sms) {
        CKL_CUDA_TRY(launch(reinterpret_cast<const void*>(merge_states_split_kernel), dim3(rows),
                            dim3(256), 0, stream, args, true));
        return CKL_OK;
    }
    CKL_CUDA_TRY(launch(reinterpret_cast<const void*>(merge_states_kernel), dim3(ceil_div(rows, 8)),
                        dim3(256), 0, stream, args, true));
    return CKL_OK;
}

size_t part_o_bytes(const ckl_decode_params* p) {
    return align_up((size_t)p->B * p->Hq * p->part_stride * D * sizeof(float), 256);
}

}  // namespace attn
}  // namespace ckl

using namespace ckl;
using namespace ckl::attn;

extern "C" {

ckl_status ckl_decode_plan(int G, int B, int Hkv, int max_len, int force_chunks,
                           int* num_chunks, int* chunk_tokens) {
    if (!num_chunks || !chunk_tokens || B <= 0 || Hkv <= 0 || max_len < 0)
        return fail(CKL_INVALID_ARG, "decode_plan: bad arguments");
    if (!pick(G)) return fail(CKL_UNSUPPORTED_SHAPE, "unsupported GQA group size %d", G);
    if (max_len == 0) {
        *num_chunks = 1;
        *chunk_tokens = 32;
        return CKL_OK;
    }
    int chunks;
    if (force_chunks > 0) {
        chunks = force_chunks;
    } else {
        const DeviceInfo* di = device_info();
        if (!di) return CKL_CUDA_ERROR;
        const KernelSetup* ks = setup(di);
        if (ks->st != CKL_OK) return ks->st;
        // Round DOWN to at most one wave of resident CTAs; chunks of >= 256 tokens.
        const long long slots = (long long)di->sms * ks->per_sm[G];
        const int want = (int)std::max(1LL, slots / ((long long)B * Hkv));
        const int cap = std::max(1, ceil_div(max_len, 256));
        chunks = std::min(want, cap);
    }
    const int tokens = ceil_div(ceil_div(max_len, chunks), 32) * 32;
    *chunk_tokens = tokens;
    *num_chunks = ceil_div(max_len, tokens);
    return CKL_OK;
}

size_t ckl_decode_workspace_size(const ckl_decode_params* p) {
    if (!p || p->B <= 0) return 0;
    if (p->num_chunks == 1 && p->chunk_base == 0 && p->part_stride == 1) return 0;
    // shapes the launch would reject: report a size no caller can provide
    if (p->Hq <= 0 || p->part_stride <= 0 || p->part_stride > 65535 ||
        (long long)p->B * p->Hq > 0x7fffffffLL)
        return SIZE_MAX;
    return part_o_bytes(p) + align_up((size_t)p->B * p->Hq * p->part_stride * sizeof(float), 256);
}

ckl_status ckl_decode_partial(const ckl_decode_params* p, void* stream) {
    int G = 0;
    ckl_status st = validate(p, &G);
    if (st != CKL_OK || p->B == 0) return st;
    if (!p->part_o || !p->part_lse) return fail(CKL_INVALID_ARG, "part_o/part_lse are NULL");
    return launch_partial(p, G, false, nullptr, nullptr, p->part_o, p->part_lse,
                          (cudaStream_t)stream);
}

ckl_status ckl_merge_states(const float* part_o, const float* part_lse, void* out, float* lse,
                            int rows, int num_slots, void* stream) {
    if (rows < 0 || num_slots <= 0) return fail(CKL_INVALID_ARG, "merge_states: rows/slots");
    if (rows == 0) return CKL_OK;
    if (!part_o || !part_lse || !out || !lse) return fail(CKL_INVALID_ARG, "merge_states: NULL");
    if (((uintptr_t)part_o & 15) || ((uintptr_t)out & 7))
        return fail(CKL_INVALID_ARG, "merge_states: part_o 16-byte / out 8-byte alignment");
    return launch_merge(part_o, part_lse, static_cast<__half*>(out), lse, rows, num_slots, 1, 1, 0,
                        nullptr, 0, (cudaStream_t)stream);
}

}  // extern "C"

namespace ckl {
namespace attn {

// decode_attention with the output rows of (b, h) at b*out_heads + head_offset + h.
ckl_status decode_attention_rows(const ckl_decode_params* p, void* out, float* lse,
                                 void* workspace, size_t workspace_bytes, cudaStream_t s,
                                 int out_heads, int head_offset, int wait_mode) {
    int G = 0;
    ckl_status st = validate(p, &G);
    if (st != CKL_OK || p->B == 0) return st;
    if (!out || !lse) return fail(CKL_INVALID_ARG, "out/lse are NULL");
    if (p->num_chunks == 1 && p->chunk_base == 0 && p->part_stride == 1)
        return launch_partial(p, G, true, static_cast<__half*>(out), lse, nullptr, nullptr, s,
                              out_heads, head_offset, true, nullptr, wait_mode);
    const size_t need = ckl_decode_workspace_size(p);
    if (!workspace || workspace_bytes < need)
        return fail(CKL_WORKSPACE_TOO_SMALL, "decode_attention needs %zu workspace bytes, got %zu",
                    need, workspace_bytes);
    if ((uintptr_t)workspace & 255) return fail(CKL_INVALID_ARG, "workspace must be 256-byte aligned");
    if ((uintptr_t)out & 7) return fail(CKL_INVALID_ARG, "out needs 8-byte alignment");
    float* part_o = static_cast<float*>(workspace);
    float* part_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + part_o_bytes(p));
    st = launch_partial(p, G, false, nullptr, nullptr, part_o, part_lse, s, 0, 0, true, nullptr,
                        wait_mode);
    if (st != CKL_OK) return st;
    return launch_merge(part_o, part_lse, static_cast<__half*>(out), lse, p->B * p->Hq, p->part_stride,
                        p->Hq, out_heads > 0 ? out_heads : p->Hq, head_offset, nullptr, 0, s);
}

}  // namespace attn
}  // namespace ckl

extern "C" {

ckl_status ckl_decode_attention(const ckl_decode_params* p, void* out, float* lse,
                                void* workspace, size_t workspace_bytes, void* stream) {
    return decode_attention_rows(p, out, lse, workspace, workspace_bytes, (cudaStream_t)stream,
                                 p ? p->Hq : 0, 0, 1);
}

ckl_status ckl_decode_attention_ex(const ckl_decode_params* p, void* out, float* lse,
                                   void* workspace, size_t workspace_bytes, unsigned flags,
                                   void* stream) {
    if (flags & ~CKL_DECODE_CACHE_READY)
        return fail(CKL_INVALID_ARG, "decode_attention_ex: unknown flags 0x%x", flags);
    return decode_attention_rows(p, out, lse, workspace, workspace_bytes, (cudaStream_t)stream,
                                 p ? p->Hq : 0, 0, (flags & CKL_DECODE_CACHE_READY) ? 2 : 1);
}

ckl_status ckl_decode_attention_gather(const ckl_decode_params* p, void* out_full,
                                       float* lse_full, int Hq_total, int head_offset,
                                       void* workspace, size_t workspace_bytes, void* stream) {
    if (!p) return fail(CKL_INVALID_ARG, "decode_attention_gather: params NULL");
    if (Hq_total < p->Hq || head_offset < 0 || head_offset + p->Hq > Hq_total)
        return fail(CKL_INVALID_ARG, "decode_attention_gather: heads [%d, %d) outside [0, %d)",
                    head_offset, head_offset + p->Hq, Hq_total);
    return decode_attention_rows(p, out_full, lse_full, workspace, workspace_bytes,
                                 (cudaStream_t)stream, Hq_total, head_offset, 1);
}

ckl_status ckl_validate_page_table(const int* h_indptr, const int* h_indices,
                                   const int* h_last_page_len, int B, int num_pages) {
    if (B < 0 || !h_indptr || (B > 0 && !h_last_page_len))
        return fail(CKL_INVALID_ARG, "validate_page_table: NULL arrays");
    if (h_indptr[0] != 0) return fail(CKL_INVALID_ARG, "kv_indptr[0] = %d, expected 0", h_indptr[0]);
    for (int b = 0; b < B; b++) {
        const int np = h_indptr[b + 1] - h_indptr[b];
        if (np < 0) return fail(CKL_INVALID_ARG, "kv_indptr decreases at %d", b);
        if (np > 0 && (h_last_page_len[b] < 1 || h_last_page_len[b] > PAGE))
            return fail(CKL_INVALID_ARG, "kv_last_page_len[%d] = %d outside [1,16]", b,
                        h_last_page_len[b]);
    }
    if (h_indptr[B] > 0 && !h_indices) return fail(CKL_INVALID_ARG, "kv_indices is NULL");
    for (int i = 0; i < h_indptr[B]; i++)
        if (h_indices[i] < 0 || h_indices[i] >= num_pages)
            return fail(CKL_INVALID_ARG, "kv_indices[%d] = %d outside [0,%d)", i, h_indices[i], num_pages);
    return CKL_OK;
}

}  // extern "C"
