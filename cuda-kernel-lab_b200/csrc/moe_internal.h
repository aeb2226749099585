// moe_internal.h -- host functions shared by the MoE sources (moe_gemm.cu, moe_layer.cu,
// moe_ep.cu); one declaration, so that the three agree on every signature.
#pragma once

#include "ckl_internal.h"

namespace ckl {
namespace moe {

// Expert GEMM over rows grouped by expert (offsets), optionally gathering X rows (row_src),
// scattering Y rows (row_dst) and fusing SwiGLU (w1 = up). max_rows bounds one expert's
// rows. dep: 0 normal launch; 1 launched dependent on the kernel that produced offsets
// (waits first); 2 dependent on the kernel that produced only X (prefetches weights first).
// a_rows (device, optional): rows in use.
ckl_status expert_gemm(const void* X, const int* row_src, const int* offsets, int A, int max_rows,
                       const ckl_moe_weights* w0, const ckl_moe_weights* w1, void* Y, int y_f32,
                       int force_ksplit, void* workspace, size_t workspace_bytes, void* stream,
                       int dep = 0, const int* row_dst = nullptr, const int* a_rows = nullptr);

// Routing of T tokens: ids, wts, counts, offsets, inv_perm and row_src (the token of each
// expert-sorted row).
ckl_status route_tokens(const float* logits, int T, int E, int k, int* ids, float* wts,
                        int* counts, int* offsets, int* inv_perm, int* row_src, cudaStream_t s);

}  // namespace moe
}  // namespace ckl
