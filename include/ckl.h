/* ckl.h -- C ABI of the B200-native (sm_100a) decode layer.
 *
 * Drop-in boundary for the hot path of qilem/cuda-kernel-lab: paged split-KV GQA decode
 * attention with its log-sum-exp merge, the shared-prefix cascade path, and the
 * weight-only W4A16/W8A16 MoE expert layer. The reference exposes this path as C++ free
 * functions and structs inside its .cu files; every entry point below names the
 * reference function it replaces (file:line, relative to the reference project root).
 *
 * Conventions
 *   - All tensors are device pointers owned by the caller; fp16 tensors are passed as
 *     void* (IEEE binary16), fp32 as float*, indices as int32.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Calls are asynchronous on
 *     it and never synchronise the host, except where a comment says "host".
 *   - The library never allocates device memory inside a call: every scratch buffer is a
 *     caller-provided workspace whose size a *_workspace_size() query returns. (The
 *     reference grows a hidden cudaMalloc'd Workspace: 01_decode_attention.cu:314-331.)
 *   - Errors are returned as ckl_status; nothing exits or aborts (the reference calls
 *     exit(1): common/bench.cuh:21-29). ckl_last_error_string() describes the last
 *     failure on the calling host thread.
 *   - Layouts are the reference's: q [B,Hq,128]; K/V pages [num_pages,16,Hkv,128] (NHD);
 *     FlashInfer-style CSR page table kv_indptr[B+1], kv_indices[nnz],
 *     kv_last_page_len[B] (1..16); out [B,Hq,128] fp16; lse [B,Hq] fp32 natural log.
 */
#ifndef CKL_H_
#define CKL_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CKL_API __attribute__((visibility("default")))
#else
#define CKL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum ckl_status {
    CKL_OK = 0,
    CKL_INVALID_ARG = 1,
    CKL_UNSUPPORTED_SHAPE = 2,
    CKL_CUDA_ERROR = 3,
    CKL_NCCL_ERROR = 4,
    CKL_TIMEOUT = 5,
    CKL_WORKSPACE_TOO_SMALL = 6
} ckl_status;

/* Head size and page size of the path (01_decode_attention.cu:45-46). */
#define CKL_HEAD_DIM 128
#define CKL_PAGE_SIZE 16

/* Description of the last failed call on this host thread ("" if none). */
CKL_API const char* ckl_last_error_string(void);

/* Library version string. */
CKL_API const char* ckl_version(void);

/* Reads and clears the device-side error word that bounded waits inside the kernels set
 * when they give up (host; synchronises the current device). Returns CKL_TIMEOUT if a
 * kernel launched since the last call timed out waiting on a barrier, CKL_INVALID_ARG if a
 * device-side bound given by the caller was exceeded (ckl_moe_ep_layer_ex's T_max), else
 * CKL_OK. */
CKL_API ckl_status ckl_check_device_error(void);

/* Upper bound, in nanoseconds, on any single spin-wait inside the library's kernels
 * (default 1e9; the CKL_SPIN_TIMEOUT_NS environment variable overrides it at load). */
CKL_API void ckl_set_spin_timeout_ns(uint64_t ns);

/* ======================================================================================
 * Paged split-KV decode attention
 * ==================================================================================== */

/* Launch descriptor; mirrors DecodeParams field for field (01_decode_attention.cu:51-65),
 * plus num_pages (the page count of k_cache/v_cache, bounds of the TMA descriptors: a page
 * id outside [0, num_pages) reads zeros instead of faulting). */
typedef struct ckl_decode_params {
    const void* q;                 /* [B, Hq, 128] fp16 */
    const void* k_cache;           /* [num_pages, 16, Hkv, 128] fp16, 16-byte aligned */
    const void* v_cache;           /* same layout as k_cache */
    const int* kv_indptr;          /* [B+1] */
    const int* kv_indices;         /* [kv_indptr[B]] physical page ids */
    const int* kv_last_page_len;   /* [B], 1..16 */
    float* part_o;                 /* [B*Hq, part_stride, 128] normalised partial outputs */
    float* part_lse;               /* [B*Hq, part_stride] */
    int B, Hq, Hkv, num_chunks, chunk_tokens;
    int kv_start;                  /* tokens skipped at the start of every sequence */
    int chunk_base;                /* this launch writes slots [chunk_base, +num_chunks) */
    int part_stride;               /* partial slots per (sequence, q head) */
    float sm_scale;
    int num_pages;
} ckl_decode_params;

/* Split heuristic of plan_chunks (01_decode_attention.cu:292-312): about one wave of
 * resident CTAs on the current device (SMs x resident CTAs per SM of the partial kernel),
 * never chunks shorter than 256 tokens, chunk_tokens a multiple of 32; force_chunks > 0
 * overrides. G = Hq/Hkv. Host only. */
CKL_API ckl_status ckl_decode_plan(int G, int B, int Hkv, int max_len, int force_chunks,
                           int* num_chunks, int* chunk_tokens);

/* Bytes of workspace ckl_decode_attention needs for these params (0 when the launch is a
 * single chunk and writes out/lse directly; SIZE_MAX for shapes the launch rejects, e.g.
 * part_stride > 65535). */
CKL_API size_t ckl_decode_workspace_size(const ckl_decode_params* p);

/* One launch of the partial kernel (decode_partial<G,V>, 01_decode_attention.cu:77-236):
 * for every (chunk, sequence, kv head) the online-softmax attention of its G query heads
 * over keys [kv_start + chunk*chunk_tokens, +chunk_tokens), written as normalised
 * (part_o, part_lse) into slot chunk_base + chunk. Requires chunk_tokens and kv_start to
 * be multiples of 16. Empty chunks write o = 0, lse = -inf. */
CKL_API ckl_status ckl_decode_partial(const ckl_decode_params* p, void* stream);

/* LSE merge of partial slots (merge_states, 01_decode_attention.cu:239-255):
 * m = max lse_i, w_i = exp(lse_i - m), out = sum w_i o_i / sum w_i (fp16),
 * lse = m + log(sum w_i); rows with no keys give out = 0, lse = -inf. rows = B*Hq. */
CKL_API ckl_status ckl_merge_states(const float* part_o, const float* part_lse, void* out,
                            float* lse, int rows, int num_slots, void* stream);

/* decode_attention (01_decode_attention.cu:316-331): partial + merge, with part_o /
 * part_lse carved from `workspace` (p->part_o / p->part_lse are ignored). A single-chunk
 * launch (num_chunks == 1, chunk_base == 0, part_stride == 1) writes out/lse directly
 * from the partial kernel and needs no workspace. */
CKL_API ckl_status ckl_decode_attention(const ckl_decode_params* p, void* out, float* lse,
                                void* workspace, size_t workspace_bytes, void* stream);

/* ckl_decode_attention with flags (no reference counterpart: the reference launches its
 * kernels in plain stream order). ckl_decode_attention may start behind the stream's
 * previous kernel but reads nothing until that kernel has finished. With
 * CKL_DECODE_CACHE_READY the caller vouches that the page table and every KV page except
 * each sequence's last one were written before the previous kernel began (the usual decode
 * step: the kernel before attention writes q and appends the new token to the last page);
 * the call then reads the page table and starts streaming the first pages while that
 * kernel finishes. q, the last pages and every write still wait for it. Same results as
 * ckl_decode_attention. Unknown flag bits: CKL_INVALID_ARG. */
#define CKL_DECODE_CACHE_READY 1u
CKL_API ckl_status ckl_decode_attention_ex(const ckl_decode_params* p, void* out, float* lse,
                                           void* workspace, size_t workspace_bytes,
                                           unsigned flags, void* stream);

/* Balanced split (no reference counterpart: the reference lists it as not done,
 * README.md:54). The pages of all (sequence, kv head) units are divided exactly evenly over
 * one wave of persistent CTAs (SMs x resident CTAs per SM), with a partial wherever a CTA's
 * run of pages crosses a unit boundary and an LSE merge after -- no idle tail wave and one
 * pipeline ramp per CTA. Computed on the device from the page table (no host plan).
 * Requires kv_start == 0; num_chunks / chunk_tokens / chunk_base / part_stride / part_o /
 * part_lse are ignored. Same results as ckl_decode_attention up to the fp32 summation
 * order of the split. */
CKL_API size_t ckl_decode_balanced_workspace_size(const ckl_decode_params* p);
CKL_API ckl_status ckl_decode_attention_balanced(const ckl_decode_params* p, void* out, float* lse,
                                                 void* workspace, size_t workspace_bytes,
                                                 void* stream);

/* Size of the scratch built into the library for ckl_decode_attention_noalloc. */
#define CKL_NOALLOC_SCRATCH_BYTES (16u << 20)

/* No counterpart in the reference. ckl_decode_attention for callers that cannot allocate
 * device memory -- e.g. a plugin whose host process has already reserved the GPU's memory
 * in its own pool, or a decode loop that may not call cudaMalloc/cudaFree because they can
 * synchronise the device. Instead of a caller workspace it uses a scratch array compiled
 * into the library: CKL_NOALLOC_SCRATCH_BYTES (16 MiB) on every GPU that loads the
 * library, kept until the process exits. Inputs and outputs are still the caller's.
 *   - Limit: ckl_decode_workspace_size(p) must be <= CKL_NOALLOC_SCRATCH_BYTES (about
 *     32,500 partial rows B*Hq*num_chunks); larger launches return CKL_WORKSPACE_TOO_SMALL.
 *     chunk_base must be 0 and part_stride == num_chunks.
 *   - The first call on a device looks up the scratch's device address (and may load the
 *     library's device code); make that first call before any stream capture. A failed
 *     lookup is retried by the next call. The address kept is the primary context's: it
 *     does not survive cudaDeviceReset.
 *   - All calls on a device share the one scratch and it keeps the last call's contents
 *     (each call rewrites every slot it reads). Calls that overlap on the GPU -- two
 *     streams, or two host threads -- race on it: serialise them.
 *   - Allocates nothing: no cudaMalloc, cudaFree or other allocating call. */
CKL_API ckl_status ckl_decode_attention_noalloc(const ckl_decode_params* p, void* out,
                                                float* lse, void* stream);

/* Host-side validation of a page table (host arrays): indptr non-decreasing from 0,
 * every index in [0, num_pages), last_page_len in [1,16] for non-empty sequences. */
CKL_API ckl_status ckl_validate_page_table(const int* h_indptr, const int* h_indices,
                                   const int* h_last_page_len, int B, int num_pages);

/* ======================================================================================
 * Shared-prefix (cascade) decode
 * ==================================================================================== */

/* Cascade launch plan (CascadePlan, 01_decode_attention.cu:656-662). */
typedef struct ckl_cascade_plan_t {
    int use;                      /* 0: no usable shared prefix; `suffix` is then the plain
                                     split-KV plan and ckl_cascade_decode runs it */
    int prefix_pages;             /* pages every sequence starts with */
    int prefix_len;               /* prefix_pages * 16 tokens */
    int prefix_chunks;            /* prefix partials occupy slots [0, prefix_chunks) */
    int prefix_chunk_tokens;
    int qtiles;                   /* ceil(B*G / 128) stacked-query tiles per kv head */
    const int* prefix_page_ids;   /* device: kv_indices + kv_indptr[0] */
    ckl_decode_params suffix;     /* kv_start = prefix_len, chunk_base = prefix_chunks,
                                     part_stride = prefix_chunks + suffix chunks */
} ckl_cascade_plan_t;

/* shared_prefix_pages (01_decode_attention.cu:636-646): the longest run of physical pages
 * every sequence starts with, each sequence keeping at least one private page; B < 2 -> 0.
 * Host arrays. */
CKL_API int ckl_shared_prefix_pages(const int* h_indptr, const int* h_indices, int B);

/* plan_cascade (01_decode_attention.cu:666-701): detects the shared prefix from the host
 * copy of the page table; use = 0 when it is shorter than min_prefix tokens (the reference
 * default is 256). Prefix chunks fill about one wave of prefix CTAs. Host only. */
CKL_API ckl_status ckl_cascade_plan(const ckl_decode_params* base, const int* h_indptr,
                                    const int* h_indices, const int* h_lens, int min_prefix,
                                    ckl_cascade_plan_t* plan);

/* Workspace bytes of ckl_cascade_decode (partials of all prefix and suffix slots). */
CKL_API size_t ckl_cascade_workspace_size(const ckl_cascade_plan_t* plan);

/* The prefix kernel alone (cascade_prefix, 01_decode_attention.cu:486-632): attention of
 * all B*G query rows of each kv head over the shared prefix, each page read once per kv
 * head, written as partial slots [0, prefix_chunks) of part_o / part_lse (laid out with
 * plan->suffix.part_stride slots per row). */
CKL_API ckl_status ckl_cascade_prefix(const ckl_cascade_plan_t* plan, float* part_o,
                                      float* part_lse, void* stream);

/* cascade_decode (01_decode_attention.cu:703-712): prefix kernel, suffix partial kernel
 * from kv_start = prefix_len, and one LSE merge over all slots. */
CKL_API ckl_status ckl_cascade_decode(const ckl_cascade_plan_t* plan, void* out, float* lse,
                                      void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------------------------------------------
 * Prefix-tree cascade. No reference counterpart: the reference lists "a prefix tree where
 * only a subset shares the prefix" as not done (README.md:73) and its cascade needs every
 * sequence of the batch to share one prefix (shared_prefix_pages, 01:636-646). Here any
 * group of >= 2 sequences whose page lists start with the same physical pages shares a tree
 * node, nodes nest (a system prompt shared by all, a document shared by some), and each node
 * is read once per kv head for all of its members' query heads.
 * ------------------------------------------------------------------------------------ */

/* Host only. The compressed trie of the batch's page lists, each sequence keeping its last
 * page private. A node is a run of pages [first, end) that the sequences at positions
 * [m0, m1) of perm share (>= 2 of them), begins where its nearest kept ancestor ends, and is
 * kept when it holds >= min_pages pages (runs that are shorter fall to the node's children
 * or its members' private suffixes). Writes:
 *   perm[B]            sequences in trie order (every node's members are contiguous),
 *   nodes[5 * n]       {first page, end page, m0, m1, parent node or -1}, parents first;
 *                      room for max(B - 1, 1) nodes,
 *   start_pages[B]     pages of sequence b covered by its nodes (its private suffix begins
 *                      there; 0 when it is in no node).
 * Returns n, or -1 for bad arguments. */
CKL_API int ckl_prefix_tree(const int* h_indptr, const int* h_indices, int B, int min_pages,
                            int* perm, int* nodes, int* start_pages);

typedef struct ckl_cascade_tree_plan_t {
    int use;              /* 0: no node kept; `suffix` is then the plain split-KV plan */
    int nodes;            /* tree nodes kept */
    int items;            /* prefix work items per kv head (node, page chunk, query tile) */
    int chunk_pages;      /* pages per prefix work item, at most */
    int max_path_slots;   /* prefix partial slots of the sequence with the most */
    int reserved;
    size_t table_bytes;   /* bytes of the device tables ckl_cascade_tree_decode reads */
    ckl_decode_params suffix;   /* the private suffixes: per-sequence start and first slot
                                   come from the tables (kv_start = chunk_base = 0 here);
                                   part_stride = max_path_slots + num_chunks */
} ckl_cascade_tree_plan_t;

/* Host only. Plans the tree cascade from host copies of the page table (h_lens = sequence
 * lengths in tokens) and writes its device tables into the HOST buffer `tables`
 * (table_bytes bytes), which the caller copies to device memory (16-byte aligned) before
 * ckl_cascade_tree_decode. Nodes are kept from min_prefix tokens. When `tables` is NULL or
 * smaller than plan->table_bytes the plan is filled and CKL_WORKSPACE_TOO_SMALL returned.
 * Prefix work items fill about one wave, >= 16 pages each. */
CKL_API ckl_status ckl_cascade_tree_plan(const ckl_decode_params* base, const int* h_indptr,
                                         const int* h_indices, const int* h_lens,
                                         int min_prefix, ckl_cascade_tree_plan_t* plan,
                                         void* tables, size_t table_bytes);

CKL_API size_t ckl_cascade_tree_workspace_size(const ckl_cascade_tree_plan_t* plan);

/* The tree's prefix kernel alone: every node's attention for its members' query heads,
 * written as their prefix slots of part_o / part_lse (plan->suffix.part_stride slots per
 * row). */
CKL_API ckl_status ckl_cascade_tree_prefix(const ckl_cascade_tree_plan_t* plan,
                                           const void* d_tables, float* part_o,
                                           float* part_lse, void* stream);

/* Prefix kernel over every node's work items, the suffix partial kernel from each
 * sequence's own start, and one LSE merge of each sequence's own slots. d_tables is the
 * plan's tables in device memory. Results equal ckl_decode_attention's up to the fp32
 * summation order of the split. */
CKL_API ckl_status ckl_cascade_tree_decode(const ckl_cascade_tree_plan_t* plan,
                                           const void* d_tables, void* out, float* lse,
                                           void* workspace, size_t workspace_bytes,
                                           void* stream);

/* ======================================================================================
 * Weight-only quantised MoE decode layer (W4A16 / W8A16 / fp16 experts)
 * ==================================================================================== */

/* Packed expert weights (QuantWeights, 03_moe_wq_decode.cu:281-333). A weight matrix is
 * W[e][k][n], e < E experts, k < K (the reduction dim, the reference's d) and n < N (the
 * output dim, the reference's f), fp16 row-major like the reference's [E][d][f].
 *   packed  device, ckl_moe_packed_bytes(bits, E, K, N, group) bytes: 16-column strips of
 *           per-group records holding each lane's mma.sync A fragments and the group's
 *           scales/zeros (layout documented in csrc/moe_common.cuh)
 *   scales  device fp16 [E][K/group][N] (the reference's Sc layout, 03:71); unused at 16 bits
 *   zeros   device uint32 [E][K/group][N/8], 4-bit zero point of column n in nibble n%8
 *           (asymmetric int4 only; symmetric codes are offset-binary, zero 8 or 128)
 * bits 4: group 128 (symmetric as the reference, or asym = 1 with zero points);
 * bits 8: symmetric, group 128 (the reference) or group = K (per output channel);
 * bits 16: fp16 weights (group ignored). Requires E <= 256, K % 128 == 0, N % 8 == 0. */
typedef struct ckl_moe_weights {
    int bits;
    int E, K, N;
    int group;
    int asym;
    void* packed;
    void* scales;
    void* zeros;
} ckl_moe_weights;

/* Sizes of the three buffers of ckl_moe_weights (bytes; fp16 elements; uint32 words). */
CKL_API size_t ckl_moe_packed_bytes(int bits, int E, int K, int N, int group);
CKL_API size_t ckl_moe_scale_count(int E, int K, int N, int group);
CKL_API size_t ckl_moe_zero_words(int E, int K, int N, int group);

/* pack_weights<BITS> (03_moe_wq_decode.cu:48-87): quantises fp16 W [E][K][N] (device) into
 * the caller-allocated buffers of *w. Symmetric: s = fp16(max|w| / qmax), q = clamp(rn(w/s))
 * with the rounded scale (03:70-81). Asymmetric int4 (north-star extension):
 * s = fp16((max(w,0) - min(w,0)) / 15), z = clamp(rn(-min(w,0)/s), 0, 15),
 * q = clamp(rn(w/s) + z, 0, 15). */
CKL_API ckl_status ckl_moe_pack_weights(const void* W, ckl_moe_weights* w, void* stream);

/* Imports weights the reference has already packed (QuantWeights' P and Sc,
 * 03_moe_wq_decode.cu:281-299, written by pack_weights<BITS> 03:49-87): P (device) holds
 * uint32 words in widx order (03:43-45) -- word ((e*(K/4) + k/4)*(N/CPT) + cw)*4 + k%4 has
 * columns cw*CPT .. cw*CPT+CPT-1 (CPT = 32/bits) at bit offsets bits*c, offset-binary codes
 * (q + 8 int4, q + 128 int8) or two fp16 values at 16 bits; Sc (device) the fp16 scales
 * [E][K/128][N]. *w is caller-allocated as for ckl_moe_pack_weights with asym = 0 and
 * group 128 (bits 4 and 8): the codes are re-laid into the packed records on the device
 * (nothing is re-quantised) and Sc is copied into w->scales (which may be Sc itself).
 * The result is bit-identical to ckl_moe_pack_weights on the weights the reference
 * quantised. Asynchronous on `stream`. */
CKL_API ckl_status ckl_moe_import_reference_packed(const uint32_t* P, const void* Sc,
                                                   ckl_moe_weights* w, void* stream);

/* The dequantised weights the GEMM uses, fp32 [E][K][N]: (q - z) * s exactly
 * (host_weight, 03_moe_wq_decode.cu:336-348). */
CKL_API ckl_status ckl_moe_dequant_weights(const ckl_moe_weights* w, float* W_out, void* stream);

/* Workspace of ckl_moe_expert_gemm(_ex) for A permuted rows (split-K partials; 0 when the
 * launch does not split K). swiglu = 1 for a gate/up pair. */
CKL_API size_t ckl_moe_gemm_workspace_size(const ckl_moe_weights* w, int A, int swiglu,
                                           int force_ksplit);

/* QuantWeights::run (03_moe_wq_decode.cu:318-332): Yp[r] = Xp[r] . dequant(W_e) for every
 * expert e and row r in [offsets[e], offsets[e+1]); Xp fp16 [A][K], Yp fp16 [A][N]. The
 * grid is an upper bound of min(E, A) expert slots resolved on the device from offsets:
 * no host sync. force_ksplit > 0 overrides the K split (pick_ksplit 03:306-315). */
CKL_API ckl_status ckl_moe_expert_gemm(const void* Xp, void* Yp, const int* offsets, int A,
                                       const ckl_moe_weights* w, int force_ksplit,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* Extended form: rows gathered from X through row_src[A] (NULL: X is already permuted);
 * with `up` != NULL the gate/up pair is fused: Y = fp16(silu(X.Wg) * (X.Wu)) (the SwiGLU
 * intermediate, north-star extension); y_f32 = 1 writes fp32 Y. */
CKL_API ckl_status ckl_moe_expert_gemm_ex(const void* X, const int* row_src, const int* offsets,
                                          int A, const ckl_moe_weights* gate,
                                          const ckl_moe_weights* up, void* Y, int y_f32,
                                          int force_ksplit, void* workspace,
                                          size_t workspace_bytes, void* stream);

/* MoeDecode::route_and_permute (03_moe_wq_decode.cu:382-389): router_topk (common/moe.cuh:
 * 23-72: softmax top-k, ties to the lower id, weights renormalised over the chosen k),
 * counts (moe_count), offsets[E+1] (moe_scan_offsets), optional tile offsets
 * tiles[E+1] = exclusive scan of ceil(count/bm) (moe_scan, 02_moe_grouped_gemm.cu:71-82),
 * inv_perm[T*k], and when Xp != NULL the permuted rows Xp[inv_perm[i]] = X[i/k]. The slot
 * order is the stable rank by (expert, token, slot) -- deterministic, unlike the
 * reference's atomicAdd. logits fp32 [T][E]; E <= 256, k <= 8, T*k <= 4096. */
CKL_API ckl_status ckl_moe_route_permute(const float* logits, const void* X, int T, int E, int k,
                                         int d, int* ids, float* wts, int* counts, int* offsets,
                                         int* inv_perm, void* Xp, int bm, int* tiles,
                                         void* stream);

/* moe_combine (common/moe.cuh:97-119): out[t] = sum_{j<k} wts[t][j] * Yp[inv_perm[t*k+j]]
 * accumulated in fp32 in fixed j order, written fp16 [T][f]. Yp fp16 (y_f32 = 0) or fp32. */
CKL_API ckl_status ckl_moe_combine(const void* Yp, int y_f32, const int* inv_perm,
                                   const float* wts, void* out, int T, int k, int f,
                                   void* stream);

/* moe_grouped_gemm (02_moe_grouped_gemm.cu:86-186), the dense path for batches with tens of
 * tokens or more per expert: Yp[r] = Xp[r] . W[e] for the rows r in [offsets[e],
 * offsets[e+1]) of every expert, fp16 in, fp32 accumulation, fp16 out. Xp [A][d] sorted by
 * expert (ckl_moe_route_permute), W fp16 [E][d][f] row-major (the reference's layout),
 * offsets [E+1] device. tcgen05 tensor cores, one persistent launch, device-side schedule (no
 * host sync). d % 64 == 0, f % 128 == 0, E <= 256.
 * workspace: ckl_moe_grouped_gemm_workspace_size() bytes (16-byte aligned) whose first 1024
 * bytes are zero before the first launch; every launch that completes leaves them zero (they
 * are the flags of the k-split work items, the rest holds their fp32 partial tiles). One
 * workspace serves one launch at a time; after a CKL_TIMEOUT (ckl_check_device_error) zero it
 * again. */
CKL_API size_t ckl_moe_grouped_gemm_workspace_size(void);
CKL_API ckl_status ckl_moe_grouped_gemm(const void* Xp, const void* W, void* Yp, const int* offsets,
                                        int A, int E, int d, int f, void* workspace,
                                        size_t workspace_bytes, void* stream);

/* Stable on-disk format of packed expert weights (no reference counterpart: the reference
 * quantises at start-up, 03_moe_wq_decode.cu:286-299). A 64-byte little-endian header
 * (magic "CKLMOEW1", version 1, bits, E, K, N, group, asym, CRC-32 of the payload, the
 * three section sizes; layout in csrc/moe_io.cu) followed by the packed codes, scales and
 * zero points exactly as in device memory. save: device -> file; file_info: the header's
 * shape into *w (buffer pointers set to NULL) so the caller can size the buffers
 * (ckl_moe_packed_bytes ...); load: file -> the caller's device buffers, after checking
 * the shape against *w and the checksum. Host functions: they synchronise `stream`. */
CKL_API ckl_status ckl_moe_weights_save(const char* path, const ckl_moe_weights* w, void* stream);
CKL_API ckl_status ckl_moe_weights_file_info(const char* path, ckl_moe_weights* w);
CKL_API ckl_status ckl_moe_weights_load(const char* path, ckl_moe_weights* w, void* stream);

/* Workspace of ckl_moe_layer. */
CKL_API size_t ckl_moe_layer_workspace_size(int T, int k, const ckl_moe_weights* gate,
                                            const ckl_moe_weights* down);

/* The MoE decode layer (MoeDecode route_and_permute + expert GEMM + combine,
 * 03_moe_wq_decode.cu:350-391, with a SwiGLU expert per the north star): routing, fused
 * gate/up GEMM with h = fp16(silu(x Wg) * (x Wu)), down GEMM, fixed-order combine.
 * gate/up are [E][d][F], down is [E][F][d]; X fp16 [T][d]; out fp16 [T][d]. ids_out /
 * wts_out (optional, [T][k]) receive the routing. No host sync. */
CKL_API ckl_status ckl_moe_layer(const float* logits, const void* X, int T, int k,
                                 const ckl_moe_weights* gate, const ckl_moe_weights* up,
                                 const ckl_moe_weights* down, void* out, int* ids_out,
                                 float* wts_out, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* ======================================================================================
 * Head-parallel decode attention with a fused gather (north star: attention partitioned by
 * KV head, "no collective except a final gather"; the reference is single-GPU)
 * ==================================================================================== */

/* ckl_decode_attention for one KV-head shard: p describes this rank's heads (Hq, Hkv, its
 * q [B,Hq,128], K/V pages [num_pages,16,Hkv,128] holding only its heads; the page table is
 * the replicated one), and the rows of (b, h) are written to out_full[b][head_offset + h]
 * and lse_full[b][head_offset + h] of a [B][Hq_total] output -- which may be another GPU's
 * buffer mapped into this process (CUDA IPC): the kernel that produces a row stores it
 * over NVLink, so the gather needs no copy or collective of its own. */
CKL_API ckl_status ckl_decode_attention_gather(const ckl_decode_params* p, void* out_full,
                                               float* lse_full, int Hq_total, int head_offset,
                                               void* workspace, size_t workspace_bytes,
                                               void* stream);

/* A group of ranks with a small peer-mapped flag window each (CKL_PEER_WINDOW_BYTES,
 * allocated with ckl_ep_window_alloc and mapped with ckl_ep_window_open). */
#define CKL_PEER_WINDOW_BYTES 256
typedef struct ckl_peer_group {
    int rank, world;
    void* windows[8];    /* windows[i] = rank i's flag window as mapped here */
} ckl_peer_group;

/* Completion of a gather into `root`: every rank calls ckl_gather_signal after the calls
 * that write into the root's buffers (stream order); the root calls ckl_gather_wait before
 * it reads them. Epoch flags, bounded wait (CKL_TIMEOUT via ckl_check_device_error). Every
 * rank signals once per root wait. */
CKL_API ckl_status ckl_gather_signal(const ckl_peer_group* g, int root, void* stream);
CKL_API ckl_status ckl_gather_wait(const ckl_peer_group* g, void* stream);

/* Barrier of the group on the GPUs (no reference counterpart: the reference runs on one
 * GPU): no rank's later kernels on `stream` run before every rank has reached its barrier
 * call in stream order. For a double-buffered gather, where the root must have read a
 * buffer back before any rank writes it again. Epoch flags in the same windows, bounded
 * wait (CKL_TIMEOUT via ckl_check_device_error); every rank calls it the same number of
 * times. */
CKL_API ckl_status ckl_peer_barrier(const ckl_peer_group* g, void* stream);

/* ======================================================================================
 * Expert-parallel MoE layer over NVLink peer memory (north star: "expert-parallel with a
 * token all-to-all for dispatch and combine"; the reference is single-GPU and has no
 * counterpart -- its layer is MoeDecode, 03_moe_wq_decode.cu:350-391)
 * ==================================================================================== */

#define CKL_EP_MAX_RANKS 8
#define CKL_IPC_HANDLE_BYTES 64

/* Rank r owns experts [r*E/world, (r+1)*E/world). Every rank has a communication window
 * (one device allocation of ckl_moe_ep_window_bytes) that every other rank maps:
 *   dispatch: each rank routes its own T tokens and writes the token row of every
 *             (token, slot) assignment into the owner's window, in slab `rank`, at the
 *             assignment's position among this rank's rows for that owner (expert order);
 *   experts:  the owner runs the gate/up and down GEMMs over the rows it received
 *             (its local experts, packed like any ckl_moe_weights with E = E/world);
 *   combine:  every rank reads its assignments' outputs back from the owners' windows and
 *             sums them in fixed slot order (as ckl_moe_combine).
 * Ranks are kept in step by epoch flags in the windows (release/acquire at system scope)
 * with bounded waits; a wait that gives up records CKL_TIMEOUT (ckl_check_device_error). */
typedef struct ckl_moe_ep_comm {
    int rank, world;       /* world <= CKL_EP_MAX_RANKS, E % world == 0 */
    int T_cap;             /* most tokens any rank passes in one call */
    int k, E, d;           /* top-k, total experts, d_model (row width) */
    void* windows[CKL_EP_MAX_RANKS];   /* windows[i] = rank i's window as mapped here
                                          (windows[rank] = this rank's own) */
} ckl_moe_ep_comm;

/* Bytes of one rank's window for this configuration. */
CKL_API size_t ckl_moe_ep_window_bytes(int world, int T_cap, int k, int E, int d);

/* Window allocation helpers (CUDA IPC; the caller owns the memory): alloc zeroes a window
 * on the current device and returns its IPC handle (CKL_IPC_HANDLE_BYTES bytes) for the
 * other ranks (alloc returns after the window is zeroed); open maps a peer's handle;
 * close unmaps; free releases an own window. Every rank must have allocated its window
 * before any rank's first ckl_moe_ep_layer (a host barrier after alloc), and every peer
 * must have closed its mapping before the owner frees it (a host barrier between). */
CKL_API ckl_status ckl_ep_window_alloc(size_t bytes, void** window, void* ipc_handle);
CKL_API ckl_status ckl_ep_window_open(const void* ipc_handle, void** window);
CKL_API ckl_status ckl_ep_window_close(void* window);
CKL_API ckl_status ckl_ep_window_free(void* window);

/* Workspace of ckl_moe_ep_layer on this rank (gate/down: this rank's local experts). */
CKL_API size_t ckl_moe_ep_workspace_size(const ckl_moe_ep_comm* comm, const ckl_moe_weights* gate,
                                         const ckl_moe_weights* down);

/* One expert-parallel SwiGLU MoE layer. Every rank calls it the same number of times, with
 * its own T (0 <= T <= T_cap) tokens: logits fp32 [T][E], X fp16 [T][d], out fp16 [T][d];
 * gate/up [E/world][d][F] and down [E/world][F][d] are this rank's experts. ids_out /
 * wts_out (optional, [T][k]) receive the routing. Asynchronous, no host sync; the result
 * equals ckl_moe_layer over all E experts up to the split-K summation order. */
CKL_API ckl_status ckl_moe_ep_layer(const ckl_moe_ep_comm* comm, const float* logits,
                                    const void* X, int T, const ckl_moe_weights* gate,
                                    const ckl_moe_weights* up, const ckl_moe_weights* down,
                                    void* out, int* ids_out, float* wts_out, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* ckl_moe_ep_layer with T_max, an upper bound of T on every rank for this call (0 < T_max <=
 * T_cap; 0 = T_cap). It bounds the rows a rank can receive (world * T_max * min(k, E/world)),
 * which sizes the expert GEMMs' grids: with small batches most of the T_cap-sized grid
 * would be CTAs that find no expert and exit. A rank that receives more rows than the bound
 * processes none of them and records CKL_INVALID_ARG (ckl_check_device_error). */
CKL_API ckl_status ckl_moe_ep_layer_ex(const ckl_moe_ep_comm* comm, int T_max, const float* logits,
                                       const void* X, int T, const ckl_moe_weights* gate,
                                       const ckl_moe_weights* up, const ckl_moe_weights* down,
                                       void* out, int* ids_out, float* wts_out, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* ======================================================================================
 * Measurement
 * ==================================================================================== */

/* Achievable-bandwidth probe (stream_read, 01_decode_attention.cu:257-265): reads
 * `bytes` (a multiple of 16) once with 16-byte loads, grid = SMs x 16 x 256 threads. */
CKL_API ckl_status ckl_stream_read(const void* buf, size_t bytes, unsigned* sink, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CKL_H_ */
