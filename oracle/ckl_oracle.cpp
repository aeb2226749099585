// ckl_oracle.cpp -- CPU restatement of qilem/cuda-kernel-lab's reference path.
//
// TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA product in
// cuda-kernel-lab_b200/: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
// leg may load it. Nothing in the product links, calls or falls back to it.
//
// Parity pin: the generators and fp64 references below are compared, value for value,
// with the reference's own host code compiled from its sources (oracle/_ref, built by
// oracle/Makefile) and with the reference's published known answers
// (results/moe_decode_counts.txt). See tests/test_oracle.py.
//
// Every function cites the reference file:line it restates. Paths are relative to the
// reference project root.
//
// Conventions: fp16 values cross this boundary as uint16_t bit patterns; all pointers are
// host pointers; every function is reentrant.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <random>
#include <thread>
#include <vector>

namespace {

constexpr int HEAD_DIM = 128;   // 01_decode_attention.cu:45
constexpr int PAGE = 16;        // 01_decode_attention.cu:46
constexpr int GS = 128;         // 03_moe_wq_decode.cu:31

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// IEEE binary32 -> binary16, round to nearest even (what host-side __float2half does).
uint16_t f2h(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t)(sign | (a > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);       // >= 65520 -> inf
    if (a <= 0x33000000u) return (uint16_t)sign;                    // <= 2^-25 -> 0
    const int e = (int)(a >> 23);
    uint32_t m = a & 0x7fffffu;
    if (e < 113) {                                                  // half subnormal
        m |= 0x800000u;
        const int shift = 126 - e;
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((uint32_t)(e - 112) << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

float h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {                                                    // subnormal: normalise
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            m &= 0x3ffu;
            x = sign | ((uint32_t)(113 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

// Round half to even, as __float2int_rn / cvt.rni does (default FE_TONEAREST).
inline int rint_even(float v) { return (int)std::nearbyint(v); }

template <class F>
void parallel_for(long n, int nthreads, F&& fn) {
    if (nthreads <= 1 || n <= 1) {
        for (long i = 0; i < n; i++) fn(i);
        return;
    }
    nthreads = (int)std::min<long>(nthreads, n);
    std::vector<std::thread> th;
    th.reserve(nthreads);
    for (int t = 0; t < nthreads; t++)
        th.emplace_back([&, t] {
            for (long i = t; i < n; i += nthreads) fn(i);
        });
    for (auto& x : th) x.join();
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- fp16 helpers
void ora_f32_to_f16(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = f2h(in[i]);
}
void ora_f16_to_f32(const uint16_t* in, float* out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = h2f(in[i]);
}

// ---------------------------------------------------------------- attention generators
// Page-table layout of Batch (01_decode_attention.cu:341-350): sequence b gets
// ceil(L_b/16) pages, last-page length L - (np-1)*16. Returns the page count.
int ora_batch_layout(const int* lens, int B, int* indptr, int* last) {
    indptr[0] = 0;
    for (int b = 0; b < B; b++) {
        const int np = ceil_div(lens[b], PAGE);
        indptr[b + 1] = indptr[b] + np;
        last[b] = lens[b] - (np - 1) * PAGE;
    }
    return indptr[B];
}

// Batch(lens, Hq, Hkv, seed, fill) (01_decode_attention.cu:341-366): identity page ids
// shuffled by mt19937(seed), then q, k, v drawn U(-1,1) from the same engine, in that
// order. q is always B*Hq*128; k/v (num_pages*16*Hkv*128) are only written if fill.
void ora_batch_generate(const int* lens, int B, int Hq, int Hkv, unsigned seed, int fill,
                        int* indptr, int* indices, int* last, uint16_t* q, uint16_t* k,
                        uint16_t* v) {
    const int num_pages = ora_batch_layout(lens, B, indptr, last);
    std::iota(indices, indices + num_pages, 0);
    std::mt19937 rng(seed);
    std::shuffle(indices, indices + num_pages, rng);
    const size_t qn = (size_t)B * Hq * HEAD_DIM;
    const size_t kvn = (size_t)num_pages * PAGE * Hkv * HEAD_DIM;
    if (fill) {
        std::uniform_real_distribution<float> U(-1.f, 1.f);
        for (size_t i = 0; i < qn; i++) q[i] = f2h(U(rng));
        for (size_t i = 0; i < kvn; i++) k[i] = f2h(U(rng));
        for (size_t i = 0; i < kvn; i++) v[i] = f2h(U(rng));
    } else if (q) {
        std::memset(q, 0, qn * 2);
    }
}

// Pages used by make_shared_prefix_batch: the Lp/16 shared pages once, plus every
// sequence's private pages (01_decode_attention.cu:720-722).
int ora_shared_prefix_num_pages(int Lp, const int* suffix, int B) {
    const int pp = Lp / PAGE;
    int total = pp;
    for (int b = 0; b < B; b++) total += ceil_div(Lp + suffix[b], PAGE) - pp;
    return total;
}

// make_shared_prefix_batch (01_decode_attention.cu:716-742): lengths Lp + suffix[b];
// a permutation of all pages from mt19937(seed+1); every sequence's first Lp/16 pages are
// perm[0..pp), private pages take perm[pp..] in sequence order; then q, k, v U(-1,1) from
// that same engine when fill.
void ora_shared_prefix_generate(int Lp, const int* suffix, int B, int Hq, int Hkv,
                                unsigned seed, int fill, int* indptr, int* indices,
                                int* last, uint16_t* q, uint16_t* k, uint16_t* v) {
    std::vector<int> lens(B);
    for (int b = 0; b < B; b++) lens[b] = Lp + suffix[b];
    ora_batch_layout(lens.data(), B, indptr, last);
    const int pp = Lp / PAGE;
    const int total = ora_shared_prefix_num_pages(Lp, suffix, B);
    std::vector<int> perm(total);
    std::iota(perm.begin(), perm.end(), 0);
    std::mt19937 rng(seed + 1);
    std::shuffle(perm.begin(), perm.end(), rng);
    int next = pp;
    for (int b = 0; b < B; b++)
        for (int i = 0; i < indptr[b + 1] - indptr[b]; i++)
            indices[indptr[b] + i] = (i < pp) ? perm[i] : perm[next++];
    const size_t qn = (size_t)B * Hq * HEAD_DIM;
    const size_t kvn = (size_t)total * PAGE * Hkv * HEAD_DIM;
    if (fill) {
        std::uniform_real_distribution<float> U(-1.f, 1.f);
        for (size_t i = 0; i < qn; i++) q[i] = f2h(U(rng));
        for (size_t i = 0; i < kvn; i++) k[i] = f2h(U(rng));
        for (size_t i = 0; i < kvn; i++) v[i] = f2h(U(rng));
    } else if (q) {
        std::memset(q, 0, qn * 2);
    }
}

// ---------------------------------------------------------------- attention reference
// cpu_reference (01_decode_attention.cu:371-400): fp64 softmax attention straight through
// the page table; output accumulated in fp32 in key order exactly as the reference does,
// lse = m + log(den) in natural log. rows = (b, h) pairs; `row_list` (optional) restricts
// the computation to the listed b*Hq+h rows (other rows are left untouched). Threads split
// rows; each row is computed identically to the single-threaded loop.
void ora_attention_ref(int B, int Hq, int Hkv, const int* indptr, const int* indices,
                       const int* lens, const uint16_t* q, const uint16_t* k,
                       const uint16_t* v, float* out, float* lse, const int* row_list,
                       int n_rows, int nthreads) {
    const int G = Hq / Hkv;
    const double scale = 1.0 / std::sqrt((double)HEAD_DIM);
    const long nr = row_list ? n_rows : (long)B * Hq;
    parallel_for(nr, nthreads, [&](long i) {
        const int row = row_list ? row_list[i] : (int)i;
        const int b = row / Hq, h = row % Hq, kvh = h / G, L = lens[b];
        const uint16_t* qv = q + (size_t)row * HEAD_DIM;
        float qf[HEAD_DIM];
        for (int d = 0; d < HEAD_DIM; d++) qf[d] = h2f(qv[d]);
        std::vector<double> s(L);
        double m = -1e300;
        for (int key = 0; key < L; key++) {
            const int page = indices[indptr[b] + key / PAGE];
            const size_t off = (((size_t)page * PAGE + key % PAGE) * Hkv + kvh) * HEAD_DIM;
            double acc = 0;
            for (int d = 0; d < HEAD_DIM; d++) acc += (double)qf[d] * h2f(k[off + d]);
            s[key] = acc * scale;
            m = std::max(m, s[key]);
        }
        double den = 0;
        for (int key = 0; key < L; key++) {
            s[key] = std::exp(s[key] - m);
            den += s[key];
        }
        float* o = out + (size_t)row * HEAD_DIM;
        for (int d = 0; d < HEAD_DIM; d++) o[d] = 0.f;
        for (int key = 0; key < L; key++) {
            const int page = indices[indptr[b] + key / PAGE];
            const size_t off = (((size_t)page * PAGE + key % PAGE) * Hkv + kvh) * HEAD_DIM;
            for (int d = 0; d < HEAD_DIM; d++) o[d] += (float)(s[key] / den * h2f(v[off + d]));
        }
        lse[row] = (float)(m + std::log(den));
    });
}

// ---------------------------------------------------------------- planners (host math)
// plan_chunks (01_decode_attention.cu:292-312), with the occupancy-derived slot count
// passed in (`wave_slots` = SMs x resident blocks per SM) instead of queried.
void ora_plan_chunks(int B, int Hkv, int max_len, int force_chunks, int wave_slots,
                     int* num_chunks, int* chunk_tokens) {
    int chunks;
    if (force_chunks > 0) {
        chunks = force_chunks;
    } else {
        const int want = std::max(1, wave_slots / (B * Hkv));
        const int cap = std::max(1, ceil_div(max_len, 256));
        chunks = std::min(want, cap);
    }
    const int tokens = ceil_div(ceil_div(max_len, chunks), 32) * 32;
    *chunk_tokens = tokens;
    *num_chunks = ceil_div(max_len, tokens);
}

// shared_prefix_pages (01_decode_attention.cu:636-646): the longest run of physical pages
// every sequence starts with, each sequence keeping at least one private page; B<2 -> 0.
int ora_shared_prefix_pages(const int* indptr, const int* indices, int B) {
    if (B < 2) return 0;
    for (int P = 0;; P++) {
        for (int b = 0; b < B; b++)
            if (P >= indptr[b + 1] - indptr[b] - 1) return P;
        const int pg = indices[indptr[0] + P];
        for (int b = 1; b < B; b++)
            if (indices[indptr[b] + P] != pg) return P;
    }
}

// ---------------------------------------------------------------- MoE generators
// make_logits (common/moe.cuh:142-151): mt19937(seed), N(0,1) floats; a per-expert bias
// of 0.8*N(0,1) drawn first (disable >= 0 -> that bias is -1e4), then logits
// N(0,1) + bias, row-major [T][E].
//
// msvc_pair_order: the reference's published results (results/moe_decode_counts.txt) come
// from an MSVC build (build.ps1). Both standard libraries draw normals with the polar
// method, two values per accepted uniform pair, but MSVC returns the pair in the opposite
// order from libstdc++. With msvc_pair_order != 0 the i-th draw is libstdc++'s draw i^1,
// which reproduces that build's stream exactly.
void ora_make_logits(int T, int E, unsigned seed, int disable, int msvc_pair_order,
                     float* lg) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> N01(0.f, 1.f);
    const size_t n = (size_t)E + (size_t)T * E;
    std::vector<float> draws(n + (n & 1));
    for (auto& x : draws) x = N01(rng);
    if (msvc_pair_order)
        for (size_t i = 0; i + 1 < draws.size(); i += 2) std::swap(draws[i], draws[i + 1]);
    std::vector<float> bias(E);
    for (int e = 0; e < E; e++) bias[e] = 0.8f * draws[e];
    if (disable >= 0) bias[disable] = -1e4f;
    for (int t = 0; t < T; t++)
        for (int e = 0; e < E; e++)
            lg[(size_t)t * E + e] = draws[(size_t)E + (size_t)t * E + e] + bias[e];
}

// Config-4/5 generator (north-star extension; no reference counterpart): n values
// N(mean, std) from mt19937(seed) with std::normal_distribution<float>, rounded to fp16
// when out16 != nullptr, else written as fp32 to out32.
void ora_normal(size_t n, unsigned seed, float mean, float stddev, uint16_t* out16,
                float* out32) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> N(mean, stddev);
    for (size_t i = 0; i < n; i++) {
        const float x = N(rng);
        if (out16) out16[i] = f2h(x);
        else out32[i] = x;
    }
}

// init_uniform (common/moe.cuh:131-138): the reference's hash-based device generator of
// U(-scale, scale) fp16 values, element i from a 32-bit integer hash of (i, seed). Restated
// on the host so the MoE tests use exactly the reference test's X and W.
void ora_init_uniform(uint16_t* p, size_t n, uint32_t seed, float scale) {
    for (size_t i = 0; i < n; i++) {
        uint32_t x = (uint32_t)(i ^ (i >> 32)) * 2654435761u;
        x ^= seed;
        x ^= x >> 16;
        x *= 0x7feb352du;
        x ^= x >> 15;
        x *= 0x846ca68bu;
        x ^= x >> 16;
        const float u = (float)(x >> 8) * (1.0f / 16777216.0f);
        p[i] = f2h((2.f * u - 1.f) * scale);
    }
}

// ---------------------------------------------------------------- MoE routing
// Routing of the fp64 MoE reference (02_moe_grouped_gemm.cu:273-290): p = softmax(logits)
// in fp64, k rounds of argmax with ties to the lower expert id, weights p_i / sum of the
// chosen p. ids/wts are [T][k].
void ora_route(const float* logits, int T, int E, int k, int* ids, double* wts) {
    std::vector<double> p(E);
    std::vector<char> used(E);
    for (int t = 0; t < T; t++) {
        const float* lg = logits + (size_t)t * E;
        double mx = -1e300, s = 0;
        for (int e = 0; e < E; e++) mx = std::max(mx, (double)lg[e]);
        for (int e = 0; e < E; e++) { p[e] = std::exp(lg[e] - mx); s += p[e]; }
        std::fill(used.begin(), used.end(), 0);
        std::vector<double> sw(k);
        double tot = 0;
        for (int r = 0; r < k; r++) {
            int bi = -1;
            for (int e = 0; e < E; e++)
                if (!used[e] && (bi < 0 || p[e] > p[bi])) bi = e;
            used[bi] = 1;
            ids[(size_t)t * k + r] = bi;
            sw[r] = p[bi] / s;
            tot += sw[r];
        }
        for (int r = 0; r < k; r++) wts[(size_t)t * k + r] = sw[r] / tot;
    }
}

// Deterministic permute (north-star requirement; the reference's moe_permute
// (common/moe.cuh:80-93) assigns slots with atomicAdd, so its order is not fixed):
// counts[E] histogram (common/moe.cuh:74-77), offsets[E+1] exclusive scan
// (03_moe_wq_decode.cu:271-276), tiles[E+1] = exclusive scan of ceil(n_e/bm)
// (02_moe_grouped_gemm.cu:71-82) when tiles != nullptr, and the stable slot
// inv_perm[i] = offsets[e] + #{i' < i : ids[i'] == e} (rank by (expert, token, slot)).
void ora_permute(const int* ids, int A, int E, int bm, int* counts, int* offsets,
                 int* tiles, int* inv_perm) {
    for (int e = 0; e < E; e++) counts[e] = 0;
    for (int i = 0; i < A; i++) counts[ids[i]]++;
    int o = 0, tl = 0;
    for (int e = 0; e < E; e++) {
        offsets[e] = o;
        if (tiles) tiles[e] = tl;
        o += counts[e];
        if (tiles) tl += ceil_div(counts[e], bm);
    }
    offsets[E] = o;
    if (tiles) tiles[E] = tl;
    std::vector<int> cur(E, 0);
    for (int i = 0; i < A; i++) inv_perm[i] = offsets[ids[i]] + cur[ids[i]]++;
}

// ---------------------------------------------------------------- quantizers
// Symmetric group quantizer of pack_weights<BITS> (03_moe_wq_decode.cu:65-84), per
// (expert, group of 128 along K, column): s = fp16(max|w| / QMAX) (1 if all zero),
// q = clamp(rn(w / s), -QMAX, QMAX) with the ROUNDED scale, stored offset-binary
// (q + 8 for int4, q + 128 for int8). group = 128, or group = d for per-channel (config 5,
// same rule as quant_weight_sym 07_int8_gemm.cu:66-83). W is fp16 [E][d][f]; codes are
// uint8 [E][d][f]; scales fp16 [E][d/group][f].
void ora_quant_sym(const uint16_t* W, int E, int d, int f, int bits, int group,
                   uint8_t* codes, uint16_t* scales, int nthreads) {
    const int qmax = bits == 8 ? 127 : 7, bias = bits == 8 ? 128 : 8, ngr = d / group;
    parallel_for((long)E * ngr, nthreads, [&](long eg) {
        const int e = (int)(eg / ngr), g = (int)(eg % ngr);
        const uint16_t* We = W + (size_t)e * d * f;
        for (int c = 0; c < f; c++) {
            float m = 0.f;
            for (int kk = g * group; kk < (g + 1) * group; kk++)
                m = std::max(m, std::fabs(h2f(We[(size_t)kk * f + c])));
            const uint16_t hs = f2h(m > 0.f ? m / (float)qmax : 1.f);
            scales[((size_t)e * ngr + g) * f + c] = hs;
            const float s = h2f(hs);
            for (int kk = g * group; kk < (g + 1) * group; kk++) {
                int q = rint_even(h2f(We[(size_t)kk * f + c]) / s);
                q = std::max(-qmax, std::min(qmax, q));
                codes[((size_t)e * d + kk) * f + c] = (uint8_t)(q + bias);
            }
        }
    });
}

// Asymmetric int4 group quantizer (north-star extension, config 4; follows the
// zero-point rule of quant_act_asym 07_int8_gemm.cu:86-110 and the rounded-scale rule of
// 03_moe_wq_decode.cu:70-72): per (expert, group of 128 along K, column)
// mn = min(w,0), mx = max(w,0), s = fp16((mx-mn)/15) (1 if mx == mn),
// z = clamp(rn(-mn/s), 0, 15), q = clamp(rn(w/s) + z, 0, 15). Dequant (q - z) * s.
// codes uint8 [E][d][f] hold q; scales fp16 and zeros uint8 [E][d/128][f].
void ora_quant_asym4(const uint16_t* W, int E, int d, int f, uint8_t* codes,
                     uint16_t* scales, uint8_t* zeros, int nthreads) {
    const int ngr = d / GS;
    parallel_for((long)E * ngr, nthreads, [&](long eg) {
        const int e = (int)(eg / ngr), g = (int)(eg % ngr);
        const uint16_t* We = W + (size_t)e * d * f;
        for (int c = 0; c < f; c++) {
            float mn = 0.f, mx = 0.f;
            for (int kk = g * GS; kk < (g + 1) * GS; kk++) {
                const float w = h2f(We[(size_t)kk * f + c]);
                mn = std::min(mn, w);
                mx = std::max(mx, w);
            }
            const uint16_t hs = f2h(mx > mn ? (mx - mn) / 15.f : 1.f);
            const float s = h2f(hs);
            const int z = std::max(0, std::min(15, rint_even(-mn / s)));
            scales[((size_t)e * ngr + g) * f + c] = hs;
            zeros[((size_t)e * ngr + g) * f + c] = (uint8_t)z;
            for (int kk = g * GS; kk < (g + 1) * GS; kk++) {
                const int q = std::max(0, std::min(15, rint_even(h2f(We[(size_t)kk * f + c]) / s) + z));
                codes[((size_t)e * d + kk) * f + c] = (uint8_t)q;
            }
        }
    });
}

// Dequantized weight host_weight (03_moe_wq_decode.cu:336-348) generalised with a zero
// point: w = (float)(q - z) * s, exact in fp32. zeros == nullptr means the symmetric bias
// (8 for int4, 128 for int8). Output fp32 [E][d][f].
void ora_dequant(const uint8_t* codes, const uint16_t* scales, const uint8_t* zeros, int E,
                 int d, int f, int bits, int group, float* Wdq) {
    const int ngr = d / group, bias = bits == 8 ? 128 : 8;
    for (int e = 0; e < E; e++)
        for (int kk = 0; kk < d; kk++) {
            const size_t srow = ((size_t)e * ngr + kk / group) * f;
            for (int c = 0; c < f; c++) {
                const int z = zeros ? zeros[srow + c] : bias;
                const int q = codes[((size_t)e * d + kk) * f + c];
                Wdq[((size_t)e * d + kk) * f + c] = (float)(q - z) * h2f(scales[srow + c]);
            }
        }
}

// ---------------------------------------------------------------- MoE GEMM references
// Expert GEMM reference (03_moe_wq_decode.cu:471-479): for every expert e and row
// r in [offsets[e], offsets[e+1]): Y[r][c] = (float) sum_k (double)X[r][k] * W[e][k][c],
// W given dequantized in fp32 [E][d][f]; X fp16 [A][d].
void ora_expert_gemm(const uint16_t* X, const float* W, const int* offsets, int E, int d,
                     int f, float* Y, int nthreads) {
    const int A = offsets[E];
    std::vector<int> row_e(A);
    for (int e = 0; e < E; e++)
        for (int r = offsets[e]; r < offsets[e + 1]; r++) row_e[r] = e;
    parallel_for(A, nthreads, [&](long r) {
        std::vector<double> xr(d);
        for (int kk = 0; kk < d; kk++) xr[kk] = h2f(X[(size_t)r * d + kk]);
        const float* We = W + (size_t)row_e[r] * d * f;
        std::vector<double> acc(f, 0.0);
        for (int kk = 0; kk < d; kk++) {
            const double x = xr[kk];
            const float* wr = We + (size_t)kk * f;
            for (int c = 0; c < f; c++) acc[c] += x * wr[c];
        }
        for (int c = 0; c < f; c++) Y[(size_t)r * f + c] = (float)acc[c];
    });
}

// Full SwiGLU MoE decode layer (north-star extension of MoeDecode, 03_moe_wq_decode.cu:
// 350-391 plus moe_combine common/moe.cuh:97-119): per assignment (t, j) with expert
// e = ids[t][j]: g = x_t Wg_e, u = x_t Wu_e in fp64; h = fp16(silu(g) * u);
// y = h Wd_e in fp64; out[t] = sum_j wts[t][j] * y_j in fp64 (fixed j order), stored fp32.
// Weights are the dequantized fp32 tensors Wg/Wu [E][d][F], Wd [E][F][d]. h_out (optional)
// receives the fp16 intermediate [T*k][F] in (t, j) order.
void ora_moe_layer(const uint16_t* X, int T, int d, int F, int E, int k, const int* ids,
                   const double* wts, const float* Wg, const float* Wu, const float* Wd,
                   float* out, uint16_t* h_out, int nthreads) {
    parallel_for(T, nthreads, [&](long t) {
        std::vector<double> x(d), o(d, 0.0), g(F), u(F), y(d);
        std::vector<double> h(F);
        for (int kk = 0; kk < d; kk++) x[kk] = h2f(X[(size_t)t * d + kk]);
        for (int j = 0; j < k; j++) {
            const int e = ids[(size_t)t * k + j];
            std::fill(g.begin(), g.end(), 0.0);
            std::fill(u.begin(), u.end(), 0.0);
            const float* wg = Wg + (size_t)e * d * F;
            const float* wu = Wu + (size_t)e * d * F;
            for (int kk = 0; kk < d; kk++) {
                const double xv = x[kk];
                for (int c = 0; c < F; c++) {
                    g[c] += xv * wg[(size_t)kk * F + c];
                    u[c] += xv * wu[(size_t)kk * F + c];
                }
            }
            for (int c = 0; c < F; c++) {
                const double sg = g[c] / (1.0 + std::exp(-g[c]));
                const uint16_t hh = f2h((float)(sg * u[c]));
                if (h_out) h_out[((size_t)t * k + j) * F + c] = hh;
                h[c] = h2f(hh);
            }
            std::fill(y.begin(), y.end(), 0.0);
            const float* wd = Wd + (size_t)e * F * d;
            for (int c = 0; c < F; c++) {
                const double hv = h[c];
                for (int n = 0; n < d; n++) y[n] += hv * wd[(size_t)c * d + n];
            }
            const double w = wts[(size_t)t * k + j];
            for (int n = 0; n < d; n++) o[n] += w * y[n];
        }
        for (int n = 0; n < d; n++) out[(size_t)t * d + n] = (float)o[n];
    });
}

// Weighted combine of the reference (common/moe.cuh:97-119), restated in fp64:
// out[t][c] = sum_{j<k} wts[t][j] * Y[inv_perm[t*k+j]][c].
void ora_combine(const float* Y, const int* inv_perm, const double* wts, int T, int k, int f,
                 float* out) {
    for (int t = 0; t < T; t++)
        for (int c = 0; c < f; c++) {
            double acc = 0;
            for (int j = 0; j < k; j++)
                acc += wts[(size_t)t * k + j] * Y[(size_t)inv_perm[(size_t)t * k + j] * f + c];
            out[(size_t)t * f + c] = (float)acc;
        }
}

}  // extern "C"
