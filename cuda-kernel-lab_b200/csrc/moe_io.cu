// moe_io.cu -- stable on-disk format of packed expert weights.
//
// The reference packs its weights on the device at start-up (QuantWeights,
// 03_moe_wq_decode.cu:286-299) and keeps no file format. A serving process loads weights
// far more often than it quantises them, so the packed buffers of ckl_moe_weights are
// written once and read back as they are:
//
//   offset  size  field (little-endian)
//   0       8     magic "CKLMOEW1"
//   8       4     format version (1)
//   12      4     bits (4, 8, 16)
//   16      4     E
//   20      4     K
//   24      4     N
//   28      4     group (128 or K; K for bits 16)
//   32      4     asym (0 or 1)
//   36      4     CRC-32 (IEEE, reflected 0xEDB88320) of the payload
//   40      8     packed bytes
//   48      8     scale count (fp16 elements; 0 for bits 16)
//   56      8     zero-point words (uint32; 0 unless asym)
//   64      ...   payload: packed codes, scales, zero points
//
// The packed layout itself is described in moe_common.cuh; version 1 is that layout.

#include <cstdio>
#include <cstring>
#include <vector>

#include "ckl_internal.h"

namespace ckl {
namespace moeio {

constexpr char MAGIC[8] = {'C', 'K', 'L', 'M', 'O', 'E', 'W', '1'};
constexpr uint32_t VERSION = 1;
constexpr size_t HEADER = 64;

struct Header {
    char magic[8];
    uint32_t version;
    int32_t bits, E, K, N, group, asym;
    uint32_t crc;
    uint64_t packed, scales, zeros;
};
static_assert(sizeof(Header) == HEADER, "header layout");

uint32_t crc32_update(uint32_t crc, const uint8_t* p, size_t n) {
    static uint32_t table[256];
    static bool init = false;
    if (!init) {
        for (uint32_t i = 0; i < 256; i++) {
            uint32_t c = i;
            for (int k = 0; k < 8; k++) c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
            table[i] = c;
        }
        init = true;
    }
    crc = ~crc;
    for (size_t i = 0; i < n; i++) crc = table[(crc ^ p[i]) & 0xFF] ^ (crc >> 8);
    return ~crc;
}

// Byte sizes of the three buffers for a weights description.
void sizes(const ckl_moe_weights* w, uint64_t* packed, uint64_t* scales, uint64_t* zeros) {
    const int group = w->bits == 16 ? w->K : w->group;
    *packed = ckl_moe_packed_bytes(w->bits, w->E, w->K, w->N, group);
    *scales = w->bits == 16 ? 0 : ckl_moe_scale_count(w->E, w->K, w->N, group);
    *zeros = w->asym ? ckl_moe_zero_words(w->E, w->K, w->N, group) : 0;
}

ckl_status read_header(FILE* f, const char* path, Header* h) {
    if (fread(h, 1, HEADER, f) != HEADER) return fail(CKL_INVALID_ARG, "%s: short header", path);
    if (memcmp(h->magic, MAGIC, 8) != 0) return fail(CKL_INVALID_ARG, "%s: not a packed-weights file", path);
    if (h->version != VERSION)
        return fail(CKL_UNSUPPORTED_SHAPE, "%s: format version %u (this library reads %u)", path, h->version,
                    VERSION);
    ckl_moe_weights w{};
    w.bits = h->bits; w.E = h->E; w.K = h->K; w.N = h->N; w.group = h->group; w.asym = h->asym;
    uint64_t p, s, z;
    sizes(&w, &p, &s, &z);
    if (p == 0 || p != h->packed || s != h->scales || z != h->zeros)
        return fail(CKL_INVALID_ARG, "%s: section sizes do not match the shape", path);
    return CKL_OK;
}

}  // namespace moeio
}  // namespace ckl

using namespace ckl;
using namespace ckl::moeio;

extern "C" {

ckl_status ckl_moe_weights_save(const char* path, const ckl_moe_weights* w, void* stream) {
    if (!path || !w || !w->packed) return fail(CKL_INVALID_ARG, "moe_weights_save: NULL argument");
    Header h{};
    memcpy(h.magic, MAGIC, 8);
    h.version = VERSION;
    h.bits = w->bits; h.E = w->E; h.K = w->K; h.N = w->N;
    h.group = w->bits == 16 ? w->K : w->group;
    h.asym = w->asym;
    sizes(w, &h.packed, &h.scales, &h.zeros);
    if (h.packed == 0) return fail(CKL_INVALID_ARG, "moe_weights_save: bad shape");
    if ((h.scales && !w->scales) || (h.zeros && !w->zeros))
        return fail(CKL_INVALID_ARG, "moe_weights_save: NULL scales/zeros");
    std::vector<uint8_t> buf(h.packed + h.scales * 2 + h.zeros * 4);
    const cudaStream_t s = (cudaStream_t)stream;
    CKL_CUDA_TRY(cudaMemcpyAsync(buf.data(), w->packed, h.packed, cudaMemcpyDeviceToHost, s));
    if (h.scales)
        CKL_CUDA_TRY(cudaMemcpyAsync(buf.data() + h.packed, w->scales, h.scales * 2, cudaMemcpyDeviceToHost, s));
    if (h.zeros)
        CKL_CUDA_TRY(cudaMemcpyAsync(buf.data() + h.packed + h.scales * 2, w->zeros, h.zeros * 4,
                                     cudaMemcpyDeviceToHost, s));
    CKL_CUDA_TRY(cudaStreamSynchronize(s));
    h.crc = crc32_update(0, buf.data(), buf.size());
    FILE* f = fopen(path, "wb");
    if (!f) return fail(CKL_INVALID_ARG, "moe_weights_save: cannot create %s", path);
    const bool ok = fwrite(&h, 1, HEADER, f) == HEADER && fwrite(buf.data(), 1, buf.size(), f) == buf.size();
    if (fclose(f) != 0 || !ok) return fail(CKL_INVALID_ARG, "moe_weights_save: write to %s failed", path);
    return CKL_OK;
}

ckl_status ckl_moe_weights_file_info(const char* path, ckl_moe_weights* w) {
    if (!path || !w) return fail(CKL_INVALID_ARG, "moe_weights_file_info: NULL argument");
    FILE* f = fopen(path, "rb");
    if (!f) return fail(CKL_INVALID_ARG, "moe_weights_file_info: cannot open %s", path);
    Header h;
    const ckl_status st = read_header(f, path, &h);
    fclose(f);
    if (st != CKL_OK) return st;
    memset(w, 0, sizeof(*w));
    w->bits = h.bits; w->E = h.E; w->K = h.K; w->N = h.N; w->group = h.group; w->asym = h.asym;
    return CKL_OK;
}

ckl_status ckl_moe_weights_load(const char* path, ckl_moe_weights* w, void* stream) {
    if (!path || !w || !w->packed) return fail(CKL_INVALID_ARG, "moe_weights_load: NULL argument");
    FILE* f = fopen(path, "rb");
    if (!f) return fail(CKL_INVALID_ARG, "moe_weights_load: cannot open %s", path);
    Header h;
    ckl_status st = read_header(f, path, &h);
    if (st != CKL_OK) {
        fclose(f);
        return st;
    }
    if (w->bits != h.bits || w->E != h.E || w->K != h.K || w->N != h.N || w->asym != h.asym ||
        (h.bits != 16 && w->group != h.group)) {
        fclose(f);
        return fail(CKL_INVALID_ARG, "moe_weights_load: %s holds bits=%d E=%d K=%d N=%d group=%d asym=%d",
                    path, h.bits, h.E, h.K, h.N, h.group, h.asym);
    }
    if ((h.scales && !w->scales) || (h.zeros && !w->zeros)) {
        fclose(f);
        return fail(CKL_INVALID_ARG, "moe_weights_load: NULL scales/zeros");
    }
    std::vector<uint8_t> buf(h.packed + h.scales * 2 + h.zeros * 4);
    const bool ok = fread(buf.data(), 1, buf.size(), f) == buf.size();
    fclose(f);
    if (!ok) return fail(CKL_INVALID_ARG, "moe_weights_load: %s is truncated", path);
    if (crc32_update(0, buf.data(), buf.size()) != h.crc)
        return fail(CKL_INVALID_ARG, "moe_weights_load: %s fails its checksum", path);
    const cudaStream_t s = (cudaStream_t)stream;
    CKL_CUDA_TRY(cudaMemcpyAsync(w->packed, buf.data(), h.packed, cudaMemcpyHostToDevice, s));
    if (h.scales)
        CKL_CUDA_TRY(cudaMemcpyAsync(w->scales, buf.data() + h.packed, h.scales * 2, cudaMemcpyHostToDevice, s));
    if (h.zeros)
        CKL_CUDA_TRY(cudaMemcpyAsync(w->zeros, buf.data() + h.packed + h.scales * 2, h.zeros * 4,
                                     cudaMemcpyHostToDevice, s));
    CKL_CUDA_TRY(cudaStreamSynchronize(s));      // the host buffer goes away on return
    return CKL_OK;
}

}  // extern "C"
