// decode_balanced.cu -- split-KV decode attention with an exactly balanced split.
//
// plan_chunks (01_decode_attention.cu:292-312) splits every sequence into the same number
// of equal chunks, one CTA each: a batch whose (sequence, kv head) units do not fill whole
// waves of CTAs leaves SMs idle for the last wave (64 x 1024: 512 CTAs on 296 slots), and
// more, shorter chunks pay a pipeline ramp per CTA and a larger merge. The reference lists
// a balanced split as not done (README.md:54). Here one persistent wave of CTAs (SMs x
// resident CTAs per SM) divides the pages of all units exactly:
//
//   * The pages of all sequences are laid end to end (P = indptr[B] pages) and divided
//     exactly over NG groups of Hkv CTAs: group k takes pages [k*P/NG, (k+1)*P/NG) -- one
//     contiguous run across sequence boundaries -- and CTA h of the group does kv head h of
//     those pages, so the Hkv CTAs of a group read the same pages' interleaved head rows at
//     the same time, as the chunked kernel's neighbouring CTAs do (a split that walked one
//     head's pages alone left each 256-byte head row an isolated DRAM access and ran at
//     ~60 % of the chunked kernel). Computed on the device from the page table (no host
//     plan, no sync).
//   * Warp 4 streams the run's pages into the 8-stage TMA ring of the decode kernel; warps
//     0..3 take pages round-robin as there, each with its own online-softmax state. At the
//     end of every unit the four states are combined in shared memory (consumer warps only:
//     the producer keeps streaming). A unit that lies inside one CTA's run is written as
//     final fp16 output and lse right there; a unit split over several runs leaves one
//     normalised partial (o, lse) per group in slot h*(B + NG) + b + k. Only a run's first
//     and last unit can be split; at the end of its run a CTA publishes those (fence, atomic
//     count per unit) and the last CTA of a unit merges its partials in group order -- no
//     merge kernel, no wait on another CTA, and the result does not depend on which CTA
//     finished last.
//   * A small kernel clears the per-unit counts and writes the rows of empty sequences; the
//     main kernel is launched dependent on it (programmatic dependent launch) and waits for
//     it only before its first count.
//
// Where it pays: ragged batches (config 2's 256 lengths U[128, 8192]: 0.965 of measured HBM
// against 0.89 for the chunked split). On small uniform batches (64 x 1024, 8 x 8192) the
// chunked plan is already balanced and a CTA's fixed start-up and tail dominate; there the
// chunked kernel is faster (0.72-0.74 against 0.58-0.59).

#include <algorithm>
#include <mutex>

#include "attn_common.cuh"

namespace ckl {
namespace attn {

constexpr int BCONS = 4;                       // consumer warps
constexpr int BTHREADS = (BCONS + 1) * 32;
constexpr int BSTAGES = 8;
static_assert(BSTAGES % BCONS == 0, "every stage must belong to one consumer warp");
static_assert(BCONS * 32 == D, "the split-unit merge gives each consumer thread one column");
// Most head groups per launch: the merge stages a unit's nc <= NG lse rows of G floats in
// o_red, which holds BCONS * D rows.
constexpr int BMAX_GROUPS = BCONS * D;
constexpr int BRING = BSTAGES * STAGE_BYTES;
// ring, mbarriers, per-warp (m, l) [4][16] x 2, per-warp O [4][G][128], flag word
template <int G>
constexpr int bsmem() { return 1024 + BRING + 2 * BSTAGES * 8 + 2 * BCONS * 16 * 4 + BCONS * G * D * 4 + 16; }

struct BalArgs {
    const __half* q;
    const int* indptr;
    const int* indices;
    const int* last;
    float* part_o;      // [slots][G][128], slot h*(B + NG) + b + k
    float* part_lse;    // [slots][G]
    unsigned* count;    // [B*Hkv] CTAs done with each split unit (zero at launch)
    __half* out;
    float* lse;
    unsigned* err;
    unsigned long long timeout_ns;
    int B, Hq, Hkv;
    float scale_log2;
};

// First page of group k's run.
__device__ __forceinline__ long long run_start(int k, long long P, int NG) { return (long long)k * P / NG; }
// The group whose run holds page x.
__device__ __forceinline__ int run_of(long long x, long long P, int NG) { return (int)(((x + 1) * NG - 1) / P); }
// The sequence whose pages [indptr[b], indptr[b+1]) hold page x (x < indptr[B]): the last b
// with indptr[b] <= x. The whole warp searches 32 ways per round (one dependent load per
// round instead of log2(B)); every lane returns the same b.
__device__ __forceinline__ int seq_of(const int* indptr, int B, long long x, int lane) {
    int lo = 0, n = B;                                    // b lies in [lo, lo + n); indptr[lo] <= x
    while (n > 1) {
        const int step = (n + 31) >> 5;
        const int off = lane * step;
        const bool le = off < n && __ldg(indptr + lo + off) <= x;
        const int j = 31 - __clz(__ballot_sync(0xffffffffu, le));   // lane 0 always holds
        lo += j * step;
        n = min(step, n - j * step);
    }
    return lo;
}
__device__ __forceinline__ int npages_of(const int* indptr, int b) {
    return __ldg(indptr + b + 1) - __ldg(indptr + b);
}
// Moves (b, pg) forward by n pages in sequence order, skipping empty sequences.
__device__ __forceinline__ void advance(const int* indptr, int B, int& b, int& pg, int n) {
    while (n > 0 && b < B) {
        const int left = npages_of(indptr, b) - pg;
        if (n < left) {
            pg += n;
            return;
        }
        n -= left;
        pg = 0;
        do { ++b; } while (b < B && npages_of(indptr, b) == 0);
    }
}

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(BCONS * 32) : "memory");
}

template <int G>
__global__ void __launch_bounds__(BTHREADS, 2)
decode_balanced_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const BalArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = align_ptr<1024>(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + BRING);
    uint64_t* empty = full + BSTAGES;
    float* m_red = reinterpret_cast<float*>(empty + BSTAGES);   // [BCONS][16]
    float* l_red = m_red + BCONS * 16;                          // [BCONS][16]
    float* o_red = l_red + BCONS * 16;                          // [BCONS][G][128]
    int* s_last = reinterpret_cast<int*>(o_red + BCONS * G * D);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const long long P = __ldg(a.indptr + a.B);
    const int NG = (int)min((long long)(gridDim.x / a.Hkv), P);
    const int k = blockIdx.x / a.Hkv, h = blockIdx.x - k * a.Hkv;
    if (k >= NG) return;                                  // fewer pages than groups
    const long long x0 = run_start(k, P, NG), x1 = run_start(k + 1, P, NG);
    const int npg = (int)(x1 - x0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < BSTAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_barrier_init();
    }
    __syncthreads();
    const uint64_t deadline = globaltimer() + a.timeout_ns;

    // the sequence and page of the run's first page
    const int b0 = seq_of(a.indptr, a.B, x0, lane);
    const int pg0 = (int)(x0 - __ldg(a.indptr + b0));

    if (warp == BCONS) {
        // ---------------------------------------------------------------- producer warp
        if (lane == 0) {
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
        }
        const uint64_t pol = policy_evict_first();
        int b = b0, pg = pg0;                             // cursor at run page `base`
        int ok = 1, issued = 0;
        for (int base = 0; base < npg && ok; base += 32) {
            const int cnt = min(32, npg - base);
            int my_page = 0;
            if (lane < cnt) {
                int bj = b, pj = pg;
                advance(a.indptr, a.B, bj, pj, lane);
                my_page = __ldg(a.indices + __ldg(a.indptr + bj) + pj);
            }
            for (int j = 0; j < cnt; j++) {
                const int page = __shfl_sync(0xffffffffu, my_page, j);
                if (lane == 0) {
                    const int i = base + j, s = i % BSTAGES;
                    if (i >= BSTAGES) ok = mbar_wait(&empty[s], ((i / BSTAGES) - 1) & 1, deadline, a.err);
                    if (ok) {
                        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                        load_page(ring + s * STAGE_BYTES, &tmK, &tmV, h, page, &full[s], pol);
                        issued = i + 1;
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
            advance(a.indptr, a.B, b, pg, cnt);
        }
        if (lane == 0) {                                  // every issued copy lands before exit
            for (int s = 0; s < BSTAGES && s < issued; s++) {
                const int i_last = s + ((issued - 1 - s) / BSTAGES) * BSTAGES;
                mbar_wait(&full[s], (i_last / BSTAGES) & 1, deadline, a.err);
            }
        }
        return;
    }

    // -------------------------------------------------------------------- consumer warps
    const int g = lane >> 2, t = lane & 3;
    constexpr bool HI = HeadState<G>::HI;
    HeadState<G> hs;
    bool ok = true;
    int b = b0;
    long long ustart = x0 - pg0;                          // first page of sequence b
    int nsplit = 0, split_b[2] = {0, 0}, split_first[2] = {0, 0}, split_last[2] = {0, 0};
    while (b < a.B && ustart < x1) {
        const int np = npages_of(a.indptr, b);
        const long long uend = ustart + np;
        const int lo = (int)(max(x0, ustart) - x0), hi = (int)(min(x1, uend) - x0);
        const int seq_len = (np - 1) * PAGE + __ldg(a.last + b);
        hs.load_q(a.q + ((size_t)b * a.Hq + (size_t)h * G) * D, lane);
        hs.reset();
        for (int i = lo + ((warp - lo) & 3); i < hi && ok; i += BCONS) {
            const int s = i % BSTAGES;
            const bool got = mbar_wait(&full[s], (i / BSTAGES) & 1, deadline, a.err);
            if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
            const int pg = (int)(x0 + i - ustart);
            hs.page(smem_u32(ring + s * STAGE_BYTES), pg * PAGE, seq_len, a.scale_log2, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        hs.reduce_l();
        if (!ok) { hs.m_lo = hs.m_hi = -INFINITY; hs.l_lo = hs.l_hi = 0.f; }

        // ---- combine the four warps' states of this unit
        if (t == 0) {
            m_red[warp * 16 + g] = hs.m_lo;
            l_red[warp * 16 + g] = hs.l_lo;
            if (HI) {
                m_red[warp * 16 + g + 8] = hs.m_hi;
                l_red[warp * 16 + g + 8] = hs.l_hi;
            }
        }
        if (g < G) {
#pragma unroll
            for (int j = 0; j < 16; j++)
                *reinterpret_cast<float2*>(o_red + ((size_t)warp * G + g) * D + 8 * j + 2 * t) =
                    make_float2(hs.o[j][0], hs.o[j][1]);
        }
        if (HI && g + 8 < G) {
#pragma unroll
            for (int j = 0; j < 16; j++)
                *reinterpret_cast<float2*>(o_red + ((size_t)warp * G + g + 8) * D + 8 * j + 2 * t) =
                    make_float2(hs.o[j][2], hs.o[j][3]);
        }
        consumer_sync();
        const bool whole = ustart >= x0 && uend <= x1;    // the sequence lies inside this run
        const size_t slot_base = (size_t)h * (a.B + NG) + b;   // + group
        const size_t slot = slot_base + k;
        for (int idx = threadIdx.x; idx < G * D; idx += BCONS * 32) {
            const int gq = idx / D, d = idx - gq * D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < BCONS; w++) M = fmaxf(M, m_red[w * 16 + gq]);
            float L = 0.f, O = 0.f;
            if (M != -INFINITY) {
#pragma unroll
                for (int w = 0; w < BCONS; w++) {
                    const float sw = ex2(m_red[w * 16 + gq] - M);
                    L += l_red[w * 16 + gq] * sw;
                    O += o_red[((size_t)w * G + gq) * D + d] * sw;
                }
            }
            const bool has = L > 0.f;
            const float val = has ? O / L : 0.f;
            const float lse_v = has ? (M + lg2(L)) * LN2 : -INFINITY;
            if (whole) {
                const size_t row = (size_t)b * a.Hq + (size_t)h * G + gq;
                a.out[row * D + d] = __float2half_rn(val);
                if (d == 0) a.lse[row] = lse_v;
            } else {
                a.part_o[(slot * G + gq) * D + d] = val;
                if (d == 0) a.part_lse[slot * G + gq] = lse_v;
            }
        }
        if (!whole && nsplit < 2) {                       // published at the end of the run
            split_b[nsplit] = b;
            split_first[nsplit] = run_of(ustart, P, NG);
            split_last[nsplit] = run_of(uend - 1, P, NG);
            nsplit++;
        }
        consumer_sync();                                  // o_red / m_red reused by the next unit
        // next sequence
        ustart = uend;
        do { ++b; } while (b < a.B && npages_of(a.indptr, b) == 0);
    }

    // ---- publish the split units; the last CTA of each merges its partials
    if (nsplit == 0) return;
    __threadfence();                                      // this thread's partial stores
    pdl_wait();                                           // the counts were cleared
    consumer_sync();
    if (threadIdx.x < nsplit) {                           // both units counted in one round trip
        const int si = threadIdx.x;
        const unsigned arrived = atomicAdd(a.count + split_b[si] * a.Hkv + h, 1u);
        s_last[si] = arrived == (unsigned)(split_last[si] - split_first[si]);
        __threadfence();
    }
    consumer_sync();
    // Slot columns a thread keeps in registers per round trip of the merge.
    constexpr int CT = G >= 16 ? 2 : G >= 8 ? 4 : 8;
    for (int si = 0; si < nsplit; si++) {
        if (!s_last[si]) continue;                        // uniform: s_last is shared
        const int sb = split_b[si], cf = split_first[si], cl = split_last[si];
        // Slots cf..cl of the unit are contiguous. Their lse rows are staged in o_red (free
        // after the last unit; nc <= NG <= BMAX_GROUPS) while the first CT slots' columns are
        // already in flight. Thread d owns column d of every head row.
        const int nc = cl - cf + 1;
        const size_t first = (size_t)h * (a.B + NG) + sb + cf;
        const int d = threadIdx.x;
        const float* po = a.part_o + first * G * D + d;
        float v[CT][G];
        auto load_cols = [&](int c0) {
#pragma unroll
            for (int j = 0; j < CT; j++)
#pragma unroll
                for (int gq = 0; gq < G; gq++)
                    v[j][gq] = c0 + j < nc ? __ldcg(po + ((size_t)(c0 + j) * G + gq) * D) : 0.f;
        };
        load_cols(0);
        float* s_lse = o_red;                             // [nc][G]
        for (int i = threadIdx.x; i < nc * G; i += BCONS * 32) s_lse[i] = __ldcg(a.part_lse + first * G + i);
        consumer_sync();
        float M[G], L[G], O[G];
#pragma unroll
        for (int gq = 0; gq < G; gq++) {
            float m = -INFINITY;
            for (int c = 0; c < nc; c++) m = fmaxf(m, s_lse[c * G + gq]);
            M[gq] = m;
            L[gq] = 0.f;
            O[gq] = 0.f;
        }
        for (int c0 = 0; c0 < nc; c0 += CT) {
            if (c0) load_cols(c0);
#pragma unroll
            for (int j = 0; j < CT; j++) {
                if (c0 + j >= nc) break;
#pragma unroll
                for (int gq = 0; gq < G; gq++) {
                    const float li = s_lse[(c0 + j) * G + gq];
                    if (M[gq] == -INFINITY || li == -INFINITY) continue;
                    const float w = ex2((li - M[gq]) * LOG2E);
                    L[gq] += w;
                    O[gq] += w * v[j][gq];
                }
            }
        }
#pragma unroll
        for (int gq = 0; gq < G; gq++) {
            const size_t row = (size_t)sb * a.Hq + (size_t)h * G + gq;
            a.out[row * D + d] = __float2half_rn(L[gq] > 0.f ? O[gq] / L[gq] : 0.f);
            if (d == 0) a.lse[row] = L[gq] > 0.f ? M[gq] + logf(L[gq]) : -INFINITY;
        }
        consumer_sync();                                  // o_red reused by the next unit
    }
}

// Clears the per-unit counts and writes the rows of sequences with no pages (out = 0,
// lse = -inf; no CTA touches them). The main kernel may start at once.
__global__ void balanced_prep_kernel(const int* __restrict__ indptr, unsigned* __restrict__ count,
                                     __half* __restrict__ out, float* __restrict__ lse, int B, int Hq,
                                     int Hkv) {
    pdl_trigger();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < B * Hkv; i += gridDim.x * blockDim.x)
        count[i] = 0u;
    const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= B * Hq) return;
    const int b = row / Hq;
    if (npages_of(indptr, b) != 0) return;
    reinterpret_cast<uint2*>(out + (size_t)row * D)[lane] = make_uint2(0u, 0u);
    if (lane == 0) lse[row] = -INFINITY;
}

template <int G>
const void* bal_kernel() { return reinterpret_cast<const void*>(decode_balanced_kernel<G>); }
const void* pick_balanced(int G) {
    switch (G) {
        case 1: return bal_kernel<1>();
        case 2: return bal_kernel<2>();
        case 4: return bal_kernel<4>();
        case 8: return bal_kernel<8>();
        case 16: return bal_kernel<16>();
        default: return nullptr;
    }
}

int balanced_smem(int G) {
    switch (G) {
        case 1: return bsmem<1>();
        case 2: return bsmem<2>();
        case 4: return bsmem<4>();
        case 8: return bsmem<8>();
        default: return bsmem<16>();
    }
}

struct BalSetup {
    int per_sm[17] = {0};
    ckl_status st = CKL_OK;
};
const BalSetup* bal_setup(const DeviceInfo* di) {
    static BalSetup bs[64];
    static std::once_flag once[64];
    std::call_once(once[di->device], [di] {
        BalSetup& k = bs[di->device];
        for (int G : {1, 2, 4, 8, 16}) {
            const void* fn = pick_balanced(G);
            const int smem = balanced_smem(G);
            cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e == cudaSuccess)
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k.per_sm[G], fn, BTHREADS, smem);
            if (e != cudaSuccess || k.per_sm[G] < 1) {
                k.st = e != cudaSuccess ? cuda_status(e, "balanced decode setup")
                                        : fail(CKL_CUDA_ERROR, "balanced decode: no CTA fits an SM");
                return;
            }
        }
    });
    return &bs[di->device];
}

// Checks the fields the balanced split reads; returns G.
ckl_status check_balanced(const ckl_decode_params* p, int* G) {
    if (!p) return fail(CKL_INVALID_ARG, "params is NULL");
    if (p->B < 0 || p->Hq <= 0 || p->Hkv <= 0 || p->Hq % p->Hkv)
        return fail(CKL_INVALID_ARG, "bad head counts B=%d Hq=%d Hkv=%d", p->B, p->Hq, p->Hkv);
    *G = p->Hq / p->Hkv;
    if (!pick_balanced(*G)) return fail(CKL_UNSUPPORTED_SHAPE, "unsupported GQA group size %d", *G);
    if (p->B == 0) return CKL_OK;
    if (!p->q || !p->k_cache || !p->v_cache || !p->kv_indptr || !p->kv_indices || !p->kv_last_page_len)
        return fail(CKL_INVALID_ARG, "NULL tensor pointer");
    if (((uintptr_t)p->k_cache | (uintptr_t)p->v_cache) & 15)
        return fail(CKL_INVALID_ARG, "k_cache/v_cache must be 16-byte aligned");
    if ((uintptr_t)p->q & 3) return fail(CKL_INVALID_ARG, "q must be 4-byte aligned");
    if (p->num_pages <= 0) return fail(CKL_INVALID_ARG, "num_pages must be > 0");
    if (p->kv_start != 0) return fail(CKL_UNSUPPORTED_SHAPE, "balanced split: kv_start must be 0");
    return CKL_OK;
}

// Launch width: one wave of resident CTAs, rounded down to whole groups of Hkv CTAs.
int balanced_grid(const DeviceInfo* di, const BalSetup* bs, int G, int Hkv) {
    return std::min(std::max(1, di->sms * bs->per_sm[G] / Hkv), BMAX_GROUPS) * Hkv;
}

size_t balanced_slots(const ckl_decode_params* p, int grid) {
    return (size_t)p->Hkv * ((size_t)p->B + grid / p->Hkv);
}

// Workspace: part_o [slots][G][128] fp32, part_lse [slots][G], count [B*Hkv] (256-aligned).
struct BalWs {
    size_t o, lse, count, total;
};
BalWs balanced_ws(const ckl_decode_params* p, int G, int grid) {
    BalWs w{};
    const size_t slots = balanced_slots(p, grid);
    w.o = 0;
    w.lse = align_up(slots * G * D * sizeof(float), 256);
    w.count = w.lse + align_up(slots * G * sizeof(float), 256);
    w.total = w.count + align_up((size_t)p->B * p->Hkv * sizeof(unsigned), 256);
    return w;
}

}  // namespace attn
}  // namespace ckl

using namespace ckl;
using namespace ckl::attn;

extern "C" {

size_t ckl_decode_balanced_workspace_size(const ckl_decode_params* p) {
    int G = 0;
    if (check_balanced(p, &G) != CKL_OK || p->B == 0) return 0;
    const DeviceInfo* di = device_info();
    if (!di) return 0;
    const BalSetup* bs = bal_setup(di);
    if (bs->st != CKL_OK) return 0;
    return balanced_ws(p, G, balanced_grid(di, bs, G, p->Hkv)).total;
}

ckl_status ckl_decode_attention_balanced(const ckl_decode_params* p, void* out, float* lse,
                                         void* workspace, size_t workspace_bytes, void* stream) {
    int G = 0;
    ckl_status st = check_balanced(p, &G);
    if (st != CKL_OK || p->B == 0) return st;
    if (!out || !lse) return fail(CKL_INVALID_ARG, "out/lse are NULL");
    if ((uintptr_t)out & 7) return fail(CKL_INVALID_ARG, "out needs 8-byte alignment");
    const DeviceInfo* di = device_info();
    if (!di) return CKL_CUDA_ERROR;
    const BalSetup* bs = bal_setup(di);
    if (bs->st != CKL_OK) return bs->st;
    const int grid = balanced_grid(di, bs, G, p->Hkv);
    const BalWs W = balanced_ws(p, G, grid);
    if (!workspace || workspace_bytes < W.total)
        return fail(CKL_WORKSPACE_TOO_SMALL, "decode_attention_balanced needs %zu workspace bytes, got %zu",
                    W.total, workspace_bytes);
    if ((uintptr_t)workspace & 255) return fail(CKL_INVALID_ARG, "workspace must be 256-byte aligned");
    uint8_t* ws = static_cast<uint8_t*>(workspace);

    CUtensorMap tmK, tmV;
    st = encode_page_maps(p->k_cache, p->v_cache, p->Hkv, p->num_pages, &tmK, &tmV);
    if (st != CKL_OK) return st;
    BalArgs a;
    a.q = static_cast<const __half*>(p->q);
    a.indptr = p->kv_indptr;
    a.indices = p->kv_indices;
    a.last = p->kv_last_page_len;
    a.part_o = reinterpret_cast<float*>(ws + W.o);
    a.part_lse = reinterpret_cast<float*>(ws + W.lse);
    a.count = reinterpret_cast<unsigned*>(ws + W.count);
    a.out = static_cast<__half*>(out);
    a.lse = lse;
    a.err = di->err_word;
    a.timeout_ns = spin_timeout_ns();
    a.B = p->B;
    a.Hq = p->Hq;
    a.Hkv = p->Hkv;
    a.scale_log2 = p->sm_scale * LOG2E;
    const cudaStream_t s = (cudaStream_t)stream;
    const int rows = p->B * p->Hq;
    balanced_prep_kernel<<<ceil_div(rows, 8), 256, 0, s>>>(p->kv_indptr, a.count, a.out, lse, p->B,
                                                           p->Hq, p->Hkv);
    CKL_CUDA_TRY(cudaGetLastError());
    void* args[] = {&tmK, &tmV, &a};
    CKL_CUDA_TRY(launch(pick_balanced(G), dim3(grid), dim3(BTHREADS), balanced_smem(G), s, args, true));
    return CKL_OK;
}

}  // extern "C"
