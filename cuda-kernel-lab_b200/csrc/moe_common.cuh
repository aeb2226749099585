// moe_common.cuh -- the packed expert-weight format shared by the packer, the dequantiser
// and the tensor-core expert GEMM.
//
// Weights W[e][k][n] (k = reduction dim K, n = output dim N, the reference's [E][d][f]) are
// stored as strips of 16 output columns ("column tiles"). A strip holds, for every 16-wide
// step of K, exactly the A-operand fragment of one mma.m16n8k16 per lane: rows of A are the
// 16 columns of the tile (swap-AB: weights are the M operand, tokens the N operand), so
// lane (g = lane/4, t = lane%4) owns columns g and g+8 at four k positions. Within each
// 32-wide block of K the k order is permuted so that lane t's four positions of step s are
// the physical k = 8t + 4s + {0,1,2,3}: one 16-byte load of an activation row then feeds
// the B operand of two consecutive MMAs.
//
//   bits 4  (4 bytes per lane per k16 step): one uint32, nibble j:
//           j=0: (k0, g)  j=4: (k1, g)  j=1: (k0, g+8)  j=5: (k1, g+8)
//           j=2: (k2, g)  j=6: (k3, g)  j=3: (k2, g+8)  j=7: (k3, g+8)
//           (k0..k3 = 8t+4s+0..3), so ((w >> 8i) & 0x000F000F) / (& 0x00F000F0) decode the
//           pairs (a0, a2) / (a1, a3) with the fp16 magic number 0x6400 (= 1024.0).
//   bits 8  (8 bytes): uint32 word0 bytes (k0,g) (k0,g+8) (k1,g) (k1,g+8), word1 the same
//           for k2, k3 -- (w & 0x00FF00FF) and ((w >> 8) & 0x00FF00FF) give a0/a1 (a2/a3).
//   bits 16 (16 bytes): the four half2 registers a0..a3 themselves.
//
// Memory order: one record per (16-column tile, 128-wide k group). A record starts with
// the group's fragments: [8 k16 steps grouped in 16-byte lane chunks][32 lanes][16 B], i.e.
// every 512 contiguous bytes hold one 16-byte chunk per lane (1 KB of int4 per record).
// Grouped formats (int4, int8 with group 128) append the group's quantisation parameters
// for the tile's 16 columns -- 16 fp16 scales, then 16 4-bit zero points (column c in nibble
// c of 8 bytes), then 8 bytes of padding. The records of the 4 tiles of a 64-column quad
// are adjacent for each group, and a quad's groups follow one another:
// [e][quad][group][tile in quad][record], so one bulk copy per (quad, group) brings a
// CTA's codes and parameters. N is padded to a multiple of 64 with zero columns.
//
// The same scales (and zeros) are also kept in the reference's layout for interchange:
// fp16 Sc[(e * (K/group) + grp) * N + n] (03_moe_wq_decode.cu:71) and, for asymmetric int4,
// 4 bits per column, 8 columns per uint32: Z[(e * (K/group) + grp) * (N/8) + n/8], nibble
// n%8. Symmetric codes are offset-binary (q + 8 for int4, q + 128 for int8), i.e. an
// implicit zero point (the embedded zeros of symmetric int4 are 8).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace ckl {
namespace moe {

constexpr int KGROUP_STAGE = 128;   // k per pipeline stage (and the int4 quantisation group)

__host__ __device__ constexpr int bytes_per_lane(int bits) { return bits == 4 ? 4 : bits == 8 ? 8 : 16; }

// Whether group parameters are embedded in the strip records (int4, or int8 with group 128).
__host__ __device__ constexpr bool embeds_params(int bits, int group) {
    return bits == 4 || (bits == 8 && group == KGROUP_STAGE);
}
constexpr int PARAM_BYTES = 48;   // 16 fp16 scales + 8 bytes of zero nibbles + 8 bytes pad

// Bytes of the fragments of one 128-k group of one strip, and of its whole record.
__host__ __device__ constexpr int group_code_bytes(int bits) { return 256 * bytes_per_lane(bits); }
__host__ __device__ constexpr int record_bytes(int bits, int group) {
    return group_code_bytes(bits) + (embeds_params(bits, group) ? PARAM_BYTES : 0);
}

// Column quads (64 columns = 4 tiles of 16) of an N-wide matrix.
__host__ __device__ inline int num_quads(int N) { return (N + 63) / 64; }

// Byte offset of the 4-record block of (expert e, quad, group grp).
__host__ __device__ inline size_t block_offset(int bits, int group, int K, int N, int e, int quad,
                                               int grp) {
    const int ngroups = K / KGROUP_STAGE;
    return (((size_t)e * num_quads(N) + quad) * ngroups + grp) * 4 * (size_t)record_bytes(bits, group);
}

// Total packed bytes of E experts.
__host__ __device__ inline size_t packed_bytes(int bits, int group, int E, int K, int N) {
    return (size_t)E * num_quads(N) * (K / KGROUP_STAGE) * 4 * (size_t)record_bytes(bits, group);
}

// Byte offset, inside a group record, of the bytes lane `lane` owns for k16 step `ks`
// (0..7 within the group).
__host__ __device__ inline int frag_offset(int bits, int ks, int lane) {
    const int bpl = bytes_per_lane(bits);
    const int steps_per_chunk = 16 / bpl;   // k16 steps per 16-byte lane chunk
    return ((ks / steps_per_chunk) * 32 + lane) * 16 + (ks % steps_per_chunk) * bpl;
}

// Physical (k, column-in-tile) of element `j` of lane `lane`'s fragment at k16 step `ks`.
// j indexes the A registers' halves: a0 = {0,1}, a1 = {2,3}, a2 = {4,5}, a3 = {6,7}.
__host__ __device__ inline void frag_coord(int ks, int lane, int j, int* k, int* col) {
    const int g = lane >> 2, t = lane & 3;
    const int blk = ks >> 1, s = ks & 1;
    const int reg = j >> 1, hi = j & 1;          // register a0..a3, low/high half
    const int kq = (reg >= 2 ? 2 : 0) + hi;      // which of the four k positions
    *k = blk * 32 + 8 * t + 4 * s + kq;
    *col = g + ((reg & 1) ? 8 : 0);
}

}  // namespace moe
}  // namespace ckl
