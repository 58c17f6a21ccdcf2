// C-ABI plumbing of libkush_sm100.so: error reporting, version, record size and the decode kernel selection.
#include <stdarg.h>
#include <stdio.h>

#include "kush_common.cuh"

namespace kush {

static thread_local char g_err[512] = "";

int set_error(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return status;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(KUSH_ERR_CUDA, "%s: CUDA error %d (%s)", what, int(e), cudaGetErrorString(e));
    return KUSH_OK;
}

// decode launchers (kush_decode_simt.cu, kush_decode_mma.cu)
int launch_decode_simt_any(int D, int bits, int P, int dtype, int G, const void* q, void* out, const void* cache,
                           int64_t block_stride, int64_t head_stride, const void* tail_k, const int32_t* tail_idx,
                           const int32_t* block_table, const int32_t* seq_lens, int64_t max_pages, int32_t hkv,
                           float scale, int32_t n_splits, float* part_ml, float* part_o, int32_t n_seqs, int rot,
                           const int32_t* order, cudaStream_t stream);
int decode_mma_supported(int D, int bits, int P, int dtype, int G);
int launch_decode_mma(int D, int bits, int P, int dtype, int G, const void* q, void* out, const void* cache,
                      int64_t block_stride, int64_t head_stride, const void* tail_k, const int32_t* tail_idx,
                      const int32_t* block_table, const int32_t* seq_lens, int64_t max_pages, int32_t hkv, float scale,
                      int32_t n_splits, float* part_ml, float* part_o, int32_t n_seqs, int rot, const int32_t* order,
                      int32_t* counters, cudaStream_t stream);

}  // namespace kush

extern "C" int kush_sm100_combine(int32_t head_dim, int32_t dtype, int32_t group, void* out, const float* part_ml,
                                  const float* part_o, int32_t n_splits, int32_t hkv, int32_t n_seqs, void* stream);
extern "C" int kush_sm100_combine_rotated(int32_t head_dim, int32_t dtype, int32_t group, void* out,
                                          const float* part_ml, const float* part_o, int32_t n_splits, int32_t hkv,
                                          int32_t n_seqs, void* stream);

using namespace kush;

extern "C" const char* kush_sm100_last_error(void) { return g_err; }

extern "C" const char* kush_sm100_version(void) { return "kushkash_b200 0.1.0 (sm_100a)"; }

extern "C" int64_t kush_sm100_record_bytes(int32_t head_dim, int32_t bits, int32_t page) {
    if ((head_dim != 64 && head_dim != 128 && head_dim != 256) || (bits != 4 && bits != 8) || (page != 16 && page != 32))
        return 0;
    const int64_t dc = bits == 8 ? head_dim : head_dim / 2;
    return 2 * int64_t(page) * dc + 4 * int64_t(head_dim) + 4 * int64_t(page);
}

extern "C" int kush_sm100_decode_tensor_cores(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype,
                                              int32_t group) {
    if (kush_sm100_record_bytes(head_dim, bits, page) == 0 || dtype < KUSH_F16 || dtype > KUSH_F32 || group < 1)
        return KUSH_ERR_UNSUPPORTED;
    return decode_mma_supported(head_dim, bits, page, dtype, group) ? 1 : 0;
}

static int decode_any(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, int32_t group,
                                 const void* q, void* out, const void* cache, int64_t block_stride, int64_t head_stride,
                                 const void* tail_k, const int32_t* tail_idx, const int32_t* block_table,
                                 const int32_t* seq_lens, int64_t max_pages, int32_t hkv, float scale, int32_t n_splits,
                                 float* part_ml, float* part_o, int32_t n_seqs, int rot, const int32_t* order,
                                 void* stream, int32_t* counters = nullptr) {
    if (n_seqs < 0 || hkv < 1 || group < 1 || n_splits < 1)
        return set_error(KUSH_ERR_ARG, "kush_sm100_decode: n_seqs %d hkv %d group %d n_splits %d", n_seqs, hkv, group,
                         n_splits);
    if (n_seqs == 0) return KUSH_OK;
    if (!q || !out || !cache || !tail_k || !tail_idx || !block_table || !seq_lens)
        return set_error(KUSH_ERR_ARG, "kush_sm100_decode: null pointer");
    if (n_splits > 1 && (!part_ml || !part_o))
        return set_error(KUSH_ERR_ARG, "kush_sm100_decode: n_splits %d needs part_ml and part_o", n_splits);
    if (n_splits > 65535) return set_error(KUSH_ERR_ARG, "kush_sm100_decode: n_splits %d > 65535", n_splits);
    if (!aligned16(cache) || (block_stride & 15) || (head_stride & 15))
        return set_error(KUSH_ERR_ARG, "kush_sm100_decode: records must be 16-byte aligned (cache %p, strides %lld %lld)",
                         cache, (long long)block_stride, (long long)head_stride);
    if (!aligned16(tail_k) || !aligned16(q) || !aligned16(out))
        return set_error(KUSH_ERR_ARG, "kush_sm100_decode: q, out and tail_k must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (decode_mma_supported(head_dim, bits, page, dtype, group))
        return launch_decode_mma(head_dim, bits, page, dtype, group, q, out, cache, block_stride, head_stride, tail_k,
                                 tail_idx, block_table, seq_lens, max_pages, hkv, scale, n_splits, part_ml, part_o,
                                 n_seqs, rot, order, n_splits > 1 ? counters : nullptr, st);
    g_err[0] = 0;
    int rc = launch_decode_simt_any(head_dim, bits, page, dtype, group, q, out, cache, block_stride, head_stride, tail_k,
                                    tail_idx, block_table, seq_lens, max_pages, hkv, scale, n_splits, part_ml, part_o,
                                    n_seqs, rot, order, st);
    if (rc == KUSH_ERR_UNSUPPORTED && g_err[0] == 0)
        return set_error(rc, "kush_sm100_decode: unsupported head_dim %d / bits %d / page %d / dtype %d", head_dim, bits,
                         page, dtype);
    if (rc == KUSH_OK && counters && n_splits > 1)     // the CUDA-core decode: its combine as a second launch
        rc = rot ? kush_sm100_combine_rotated(head_dim, dtype, group, out, part_ml, part_o, n_splits, hkv, n_seqs, stream)
                 : kush_sm100_combine(head_dim, dtype, group, out, part_ml, part_o, n_splits, hkv, n_seqs, stream);
    return rc;
}

extern "C" int kush_sm100_decode(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, int32_t group,
                                 const void* q, void* out, const void* cache, int64_t block_stride, int64_t head_stride,
                                 const void* tail_k, const int32_t* tail_idx, const int32_t* block_table,
                                 const int32_t* seq_lens, int64_t max_pages, int32_t hkv, float scale, int32_t n_splits,
                                 float* part_ml, float* part_o, int32_t n_seqs, void* stream) {
    return decode_any(head_dim, bits, page, dtype, group, q, out, cache, block_stride, head_stride, tail_k, tail_idx,
                      block_table, seq_lens, max_pages, hkv, scale, n_splits, part_ml, part_o, n_seqs, 0, nullptr,
                      stream);
}

extern "C" int kush_sm100_decode_rotated(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, int32_t group,
                                         const void* q, void* out, const void* cache, int64_t block_stride,
                                         int64_t head_stride, const void* tail_k, const int32_t* tail_idx,
                                         const int32_t* block_table, const int32_t* seq_lens, int64_t max_pages,
                                         int32_t hkv, float scale, int32_t n_splits, float* part_ml, float* part_o,
                                         int32_t n_seqs, void* stream) {
    return decode_any(head_dim, bits, page, dtype, group, q, out, cache, block_stride, head_stride, tail_k, tail_idx,
                      block_table, seq_lens, max_pages, hkv, scale, n_splits, part_ml, part_o, n_seqs, 1, nullptr,
                      stream);
}

extern "C" int kush_sm100_decode_ex(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, int32_t group,
                                    const void* q, void* out, const void* cache, int64_t block_stride,
                                    int64_t head_stride, const void* tail_k, const int32_t* tail_idx,
                                    const int32_t* block_table, const int32_t* seq_lens, int64_t max_pages,
                                    int32_t hkv, float scale, int32_t n_splits, float* part_ml, float* part_o,
                                    int32_t n_seqs, int32_t flags, const int32_t* order, void* stream) {
    if (flags & ~KUSH_DECODE_ROTATE) return set_error(KUSH_ERR_ARG, "kush_sm100_decode_ex: unknown flags %d", flags);
    return decode_any(head_dim, bits, page, dtype, group, q, out, cache, block_stride, head_stride, tail_k, tail_idx,
                      block_table, seq_lens, max_pages, hkv, scale, n_splits, part_ml, part_o, n_seqs,
                      (flags & KUSH_DECODE_ROTATE) ? 1 : 0, order, stream);
}

extern "C" int kush_sm100_decode_fused_combine(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype,
                                               int32_t group, const void* q, void* out, const void* cache,
                                               int64_t block_stride, int64_t head_stride, const void* tail_k,
                                               const int32_t* tail_idx, const int32_t* block_table,
                                               const int32_t* seq_lens, int64_t max_pages, int32_t hkv, float scale,
                                               int32_t n_splits, float* part_ml, float* part_o, int32_t* counters,
                                               int32_t n_seqs, int32_t flags, const int32_t* order, void* stream) {
    if (flags & ~KUSH_DECODE_ROTATE)
        return set_error(KUSH_ERR_ARG, "kush_sm100_decode_fused_combine: unknown flags %d", flags);
    if (n_splits > 1 && !counters) return set_error(KUSH_ERR_ARG, "kush_sm100_decode_fused_combine: null counters");
    return decode_any(head_dim, bits, page, dtype, group, q, out, cache, block_stride, head_stride, tail_k, tail_idx,
                      block_table, seq_lens, max_pages, hkv, scale, n_splits, part_ml, part_o, n_seqs,
                      (flags & KUSH_DECODE_ROTATE) ? 1 : 0, order, stream, counters);
}
