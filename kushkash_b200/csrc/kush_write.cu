// Quantize-on-write kernels: decode appends and ragged (prefill / chunked prefill) writes into page records.
// Bit-exact with the reference quantizer (kushkash/kush/quant.mojo:25-50) through kush_common.cuh's qparams/qcode.
//
// Work split on the GPU: a V token row is one warp (per-token range = warp min/max, lane holds dims lane + 32i);
// a K page is one thread per channel (int8) or per channel pair (int4: dims j and j + D/2 share a byte), reading
// the page column-wise.  The decode append reads its one row per head straight from global memory; the bulk write
// stages a page's rows in shared memory with 16-byte loads and writes the assembled record with 16-byte stores.
#include <stdio.h>

#include "kush_common.cuh"

namespace kush {

// one warp: V token row src[0:D] -> row t of the record (per-token range: the row's final encoding)
// (kushkash/kush/gpu.mojo:163-188 _quantize_v_row)
template <int D, int BITS, int P, class IN>
__device__ __forceinline__ void quantize_v_row(const IN* __restrict__ src, uint8_t* __restrict__ rec, int t, int lane) {
    using F = Fmt<D, BITS, P>;
    constexpr int R = D / WARP;
    float x[R];
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < R; i++) {
        x[i] = to_f32(src[lane + WARP * i]);
        mn = fminf(mn, x[i]);
        mx = fmaxf(mx, x[i]);
    }
    float s, b, inv;
    qparams<BITS>(warp_min(mn), warp_max(mx), s, b, inv);
    if (lane == 0) {
        h_store(rec + F::OFF_VS, t, s);
        h_store(rec + F::OFF_VB, t, b);
    }
    uint8_t* vc = rec + F::OFF_VQ + t * F::DC;
    if constexpr (BITS == 8) {
#pragma unroll
        for (int i = 0; i < R; i++) vc[lane + WARP * i] = uint8_t(qcode<8>(x[i], b, inv));
    } else {
#pragma unroll
        for (int i = 0; i < R / 2; i++)                    // byte j = lane + 32i holds dims j and j + D/2 = x[i + R/2]
            vc[lane + WARP * i] = pack4(qcode<4>(x[i], b, inv), qcode<4>(x[i + R / 2], b, inv));
    }
}

// K of one page by the threads of a block (kushkash/kush/gpu.mojo:121-160 _quantize_k_page): per-channel range
// over the P tokens; token row t < split comes from ka + t*sa (the tail), the rest from kb + (t - split)*skb.
template <int D, int BITS, int P, class IN>
__device__ __forceinline__ void quantize_k_page(const IN* __restrict__ ka, int64_t sa, const IN* __restrict__ kb,
                                                int64_t skb, int split, uint8_t* __restrict__ rec) {
    using F = Fmt<D, BITS, P>;
    constexpr int NCH = BITS == 8 ? D : D / 2;             // threads with work: channel (int8) or channel pair (int4)
    for (int c = threadIdx.x; c < NCH; c += blockDim.x) {
        constexpr int NC = BITS == 8 ? 1 : 2;
        float bias[NC], inv[NC];
#pragma unroll
        for (int e = 0; e < NC; e++) {
            const int d = c + e * (D / 2);
            float mn = INFINITY, mx = -INFINITY;
#pragma unroll 4
            for (int t = 0; t < P; t++) {
                float x = to_f32(t < split ? ka[t * sa + d] : kb[(t - split) * skb + d]);
                mn = fminf(mn, x);
                mx = fmaxf(mx, x);
            }
            float s;
            qparams<BITS>(mn, mx, s, bias[e], inv[e]);
            h_store(rec + F::OFF_KS, d, s);
            h_store(rec + F::OFF_KB, d, bias[e]);
        }
#pragma unroll 4
        for (int t = 0; t < P; t++) {
            const IN* row = t < split ? ka + t * sa : kb + (t - split) * skb;
            if constexpr (BITS == 8) {
                rec[t * F::DC + c] = uint8_t(qcode<8>(to_f32(row[c]), bias[0], inv[0]));
            } else {
                rec[t * F::DC + c] = pack4(qcode<4>(to_f32(row[c]), bias[0], inv[0]),
                                           qcode<4>(to_f32(row[c + D / 2]), bias[1], inv[1]));
            }
        }
    }
}

__device__ __forceinline__ uint8_t* rec_at(uint8_t* cache, int64_t blk, int h, int64_t block_stride, int64_t head_stride) {
    return cache + blk * block_stride + int64_t(h) * head_stride;
}

// grid (S), block D: one token per sequence (kushkash/kush/gpu.mojo:207-238 kush_append)
template <int D, int BITS, int P, class IN>
__global__ void __launch_bounds__(D) append_kernel(const IN* __restrict__ k_new, const IN* __restrict__ v_new,
                                                   int64_t k_stride, int64_t v_stride, int32_t* seq_lens, int pos_offset,
                                                   int advance, const int32_t* __restrict__ tail_idx, uint8_t* cache,
                                                   int64_t block_stride, int64_t head_stride, IN* tail_k,
                                                   const int32_t* __restrict__ block_table, int64_t max_pages, int H) {
    const int s = blockIdx.x, d = threadIdx.x, lane = d % WARP, w = d / WARP;
    constexpr int NW = D / WARP;
    const int64_t pos = int64_t(seq_lens[s]) + pos_offset;
    if (pos < 0) return;                                   // padding row
    const int slot = int(pos % P);
    const int64_t tb = int64_t(tail_idx[s]) * H * P * D;
    const int64_t blk = block_table[s * max_pages + pos / P];
    for (int h = 0; h < H; h++) tail_k[tb + (int64_t(h) * P + slot) * D + d] = k_new[s * k_stride + h * D + d];
    for (int h = w; h < H; h += NW)
        quantize_v_row<D, BITS, P, IN>(v_new + s * v_stride + h * D, rec_at(cache, blk, h, block_stride, head_stride), slot, lane);
    __syncthreads();                                       // tail rows visible to the page quantizer; seq_lens read
    if (slot == P - 1) {
        for (int h = 0; h < H; h++) {
            const IN* t0 = tail_k + tb + int64_t(h) * P * D;
            quantize_k_page<D, BITS, P, IN>(t0, D, t0, D, P, rec_at(cache, blk, h, block_stride, head_stride));
        }
    }
    if (advance && d == 0) seq_lens[s] = int32_t(pos + 1);
}

// Copy `rows` rows of D elements (row r at src + r * stride) into shared memory dst (rows packed), all threads of the
// block; 16-byte loads when every row start is 16-byte aligned, else element loads.
template <int D, class IN>
__device__ __forceinline__ void stage_rows(IN* dst, const IN* src, int64_t stride, int rows, bool vec) {
    if (rows <= 0) return;
    if (vec) {
        constexpr int CPR = D * int(sizeof(IN)) / 16;              // 16-byte chunks per row
        for (int c = threadIdx.x; c < rows * CPR; c += blockDim.x) {
            const int r = c / CPR, k = c % CPR;
            reinterpret_cast<uint4*>(dst + r * D)[k] = reinterpret_cast<const uint4*>(src + r * stride)[k];
        }
    } else {
        for (int c = threadIdx.x; c < rows * D; c += blockDim.x) dst[c] = src[(c / D) * stride + c % D];
    }
}

// Copy bytes [lo, hi) of a record assembled in shared memory to its place in global memory (16-byte stores for
// the 16-byte-aligned middle when the record is 16-byte aligned, 2-byte stores otherwise and at the edges: every
// range here starts and ends on an fp16 boundary).
__device__ __forceinline__ void store_range(uint8_t* dst, const uint8_t* src, int lo, int hi, bool vec) {
    const int a = (lo + 15) & ~15, b = hi & ~15;
    if (a >= b || !vec) {
        for (int i = lo + 2 * int(threadIdx.x); i < hi; i += 2 * blockDim.x)
            *reinterpret_cast<uint16_t*>(dst + i) = *reinterpret_cast<const uint16_t*>(src + i);
        return;
    }
    for (int i = lo + 2 * int(threadIdx.x); i < a; i += 2 * blockDim.x)
        *reinterpret_cast<uint16_t*>(dst + i) = *reinterpret_cast<const uint16_t*>(src + i);
    for (int i = a + 16 * int(threadIdx.x); i < b; i += 16 * blockDim.x)
        *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(src + i);
    for (int i = b + 2 * int(threadIdx.x); i < hi; i += 2 * blockDim.x)
        *reinterpret_cast<uint16_t*>(dst + i) = *reinterpret_cast<const uint16_t*>(src + i);
}

// grid (n_jobs, H), block D: ragged writes (kushkash/kush/gpu.mojo:241-276 kush_write); mode 0 / 1 as the
// reference, mode 2 = both in one launch: the tail stash of a sequence's last, partial page is done by the CTA that
// quantizes the sequence's first page from the old tail (after it has staged those rows), or by the last page's own
// CTA when no page reads the old tail.
// The page's new V rows and (for a page now complete) its K rows are first staged in shared memory with 16-byte
// loads; V rows are quantized by warps (one row per warp at a time), K channels by threads; the record bytes are
// assembled in shared memory and written back with 16-byte stores.  Same arithmetic as the per-token helpers above.
template <int D, int BITS, int P, class IN>
__global__ void __launch_bounds__(D) write_kernel(const IN* __restrict__ k_new, const IN* __restrict__ v_new,
                                                  int64_t k_stride, int64_t v_stride,
                                                  const int32_t* __restrict__ qsl, const int32_t* __restrict__ seq_lens,
                                                  const int32_t* __restrict__ tail_idx, const int32_t* __restrict__ job_seq,
                                                  const int32_t* __restrict__ job_page, int mode, uint8_t* cache,
                                                  int64_t block_stride, int64_t head_stride, IN* tail_k,
                                                  const int32_t* __restrict__ block_table, int64_t max_pages, int H,
                                                  int vec) {
    using F = Fmt<D, BITS, P>;
    constexpr int NW = D / WARP, R = D / WARP;
    extern __shared__ __align__(16) uint8_t wsm[];
    IN* ks_in = reinterpret_cast<IN*>(wsm);                         // [P][D] K rows of the page (complete pages)
    IN* vs_in = ks_in + P * D;                                      // [P][D] new V rows (row t - ps)
    uint8_t* rs = reinterpret_cast<uint8_t*>(vs_in + P * D);        // [RB] the record, assembled
    const int j = blockIdx.x, h = blockIdx.y, d = threadIdx.x, lane = d % WARP, w = d / WARP;
    const int64_t s = job_seq[j];
    const int64_t ps = int64_t(job_page[j]) * P;
    const int64_t q0 = qsl[s];
    const int64_t total = seq_lens[s];
    const int64_t ctx = total - (int64_t(qsl[s + 1]) - q0);
    const int64_t tb = (int64_t(tail_idx[s]) * H + h) * P * D;
    const bool complete = ps + P <= total;

    // mode 1 work for page pstart: copy its new K rows into the tail
    auto stash = [&](int64_t pstart) {
        for (int64_t t = max(pstart, ctx); t < total; t++)
            tail_k[tb + (t - pstart) * D + d] = k_new[(q0 + t - ctx) * k_stride + h * D + d];
    };

    if (mode == 1) {
        if (!complete) stash(ps);
        return;
    }
    uint8_t* rec = rec_at(cache, block_table[s * max_pages + ps / P], h, block_stride, head_stride);
    const int r0 = int(max(ps, ctx) - ps), r1 = int(min(ps + P, total) - ps);    // new rows [r0, r1) of the page
    const int split = complete ? int(max(int64_t(0), min(int64_t(P), ctx - ps))) : 0;
    // 1. stage inputs
    const bool vin = vec & 1;
    stage_rows<D, IN>(vs_in + r0 * D, v_new + (q0 + ps + r0 - ctx) * v_stride + h * D, v_stride, r1 - r0, vin);
    if (complete) {
        stage_rows<D, IN>(ks_in, tail_k + tb, D, split, vin);
        stage_rows<D, IN>(ks_in + split * D, k_new + (q0 + ps + split - ctx) * k_stride + h * D, k_stride, P - split, vin);
    }
    __syncthreads();
    // mode 2: the old tail rows are staged; the stash of the sequence's last partial page may now overwrite them
    if (mode == 2) {
        const int64_t first = (ctx / P) * P, last = ((total - 1) / P) * P;
        const bool last_partial = total % P != 0 && total > ctx;
        const bool first_reads_tail = ctx % P != 0 && first + P <= total;
        if (last_partial && ((first_reads_tail && last != first) ? ps == first : ps == last)) stash(last);
    }
    // 2. V rows: per-token range, warp w takes rows r0 + w, r0 + w + NW, ...
    for (int r = r0 + w; r < r1; r += NW) {
        float x[R];
        float mn = INFINITY, mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < R; i++) {
            x[i] = to_f32(vs_in[r * D + lane + WARP * i]);
            mn = fminf(mn, x[i]);
            mx = fmaxf(mx, x[i]);
        }
        float sc, b, inv;
        qparams<BITS>(warp_min(mn), warp_max(mx), sc, b, inv);
        if (lane == 0) {
            h_store(rs + F::OFF_VS, r, sc);
            h_store(rs + F::OFF_VB, r, b);
        }
        uint8_t* vc = rs + F::OFF_VQ + r * F::DC;
        if constexpr (BITS == 8) {
#pragma unroll
            for (int i = 0; i < R; i++) vc[lane + WARP * i] = uint8_t(qcode<8>(x[i], b, inv));
        } else {
#pragma unroll
            for (int i = 0; i < R / 2; i++)
                vc[lane + WARP * i] = pack4(qcode<4>(x[i], b, inv), qcode<4>(x[i + R / 2], b, inv));
        }
    }
    // 3. K page (complete pages): per-channel range over the P staged rows, thread = channel (int4: channel pair)
    if (complete) {
        constexpr int NCH = BITS == 8 ? D : D / 2;
        for (int c = d; c < NCH; c += blockDim.x) {
            constexpr int NC = BITS == 8 ? 1 : 2;
            float bias[NC], inv[NC];
#pragma unroll
            for (int e = 0; e < NC; e++) {
                const int ch = c + e * (D / 2);
                float mn = INFINITY, mx = -INFINITY;
#pragma unroll
                for (int t = 0; t < P; t++) {
                    const float x = to_f32(ks_in[t * D + ch]);
                    mn = fminf(mn, x);
                    mx = fmaxf(mx, x);
                }
                float sc;
                qparams<BITS>(mn, mx, sc, bias[e], inv[e]);
                h_store(rs + F::OFF_KS, ch, sc);
                h_store(rs + F::OFF_KB, ch, bias[e]);
            }
#pragma unroll
            for (int t = 0; t < P; t++) {
                if constexpr (BITS == 8) {
                    rs[t * F::DC + c] = uint8_t(qcode<8>(to_f32(ks_in[t * D + c]), bias[0], inv[0]));
                } else {
                    rs[t * F::DC + c] = pack4(qcode<4>(to_f32(ks_in[t * D + c]), bias[0], inv[0]),
                                              qcode<4>(to_f32(ks_in[t * D + c + D / 2]), bias[1], inv[1]));
                }
            }
        }
    }
    __syncthreads();
    // 4. write back: V code rows and V scale / bias entries of the new rows; the K part of a complete page
    const bool vout = vec & 2;
    if (r1 > r0) {
        store_range(rec, rs, F::OFF_VQ + r0 * F::DC, F::OFF_VQ + r1 * F::DC, vout);
        store_range(rec, rs, F::OFF_VS + 2 * r0, F::OFF_VS + 2 * r1, vout);
        store_range(rec, rs, F::OFF_VB + 2 * r0, F::OFF_VB + 2 * r1, vout);
    }
    if (complete) {
        store_range(rec, rs, 0, P * F::DC, vout);
        store_range(rec, rs, F::OFF_KS, F::OFF_VS, vout);
    }
}

template <int D, int BITS, int P, class IN>
int launch_append(const void* k_new, const void* v_new, int64_t k_stride, int64_t v_stride, int32_t* seq_lens,
                  int32_t pos_offset, int32_t advance, const int32_t* tail_idx, void* cache, int64_t block_stride,
                  int64_t head_stride, void* tail_k, const int32_t* block_table, int64_t max_pages, int32_t hkv,
                  int32_t n_seqs, cudaStream_t stream) {
    append_kernel<D, BITS, P, IN><<<n_seqs, D, 0, stream>>>(
        static_cast<const IN*>(k_new), static_cast<const IN*>(v_new), k_stride, v_stride, seq_lens, pos_offset, advance,
        tail_idx, static_cast<uint8_t*>(cache), block_stride, head_stride, static_cast<IN*>(tail_k), block_table,
        max_pages, hkv);
    return check_launch("kush_sm100_append");
}

template <int D, int BITS, int P, class IN>
int launch_write(const void* k_new, const void* v_new, int64_t k_stride, int64_t v_stride, const int32_t* qsl,
                 const int32_t* seq_lens, const int32_t* tail_idx, const int32_t* job_seq, const int32_t* job_page,
                 int32_t mode, void* cache, int64_t block_stride, int64_t head_stride, void* tail_k,
                 const int32_t* block_table, int64_t max_pages, int32_t hkv, int32_t n_jobs, cudaStream_t stream) {
    dim3 grid(n_jobs, hkv);
    const size_t smem = 2 * sizeof(IN) * P * D + Fmt<D, BITS, P>::RB;
    auto kern = write_kernel<D, BITS, P, IN>;
    static unsigned long long attr_set = 0;             // one bit per device: the attribute is per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && !(attr_set >> (dev & 63) & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return set_error(KUSH_ERR_CUDA, "write: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        attr_set |= 1ull << (dev & 63);
    }
    // 16-byte staging loads need every row start 16-byte aligned (head stride D is; bases and row strides must be)
    const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    const int vin = al(k_new) && al(v_new) && al(tail_k) && (k_stride * int64_t(sizeof(IN))) % 16 == 0 &&
                    (v_stride * int64_t(sizeof(IN))) % 16 == 0;
    const int vout = al(cache) && block_stride % 16 == 0 && head_stride % 16 == 0;     // 16-byte record stores
    const int vec = vin | (vout << 1);
    kern<<<grid, D, smem, stream>>>(
        static_cast<const IN*>(k_new), static_cast<const IN*>(v_new), k_stride, v_stride, qsl, seq_lens, tail_idx,
        job_seq, job_page, mode, static_cast<uint8_t*>(cache), block_stride, head_stride, static_cast<IN*>(tail_k),
        block_table, max_pages, hkv, vec);
    return check_launch("kush_sm100_write");
}

}  // namespace kush

using namespace kush;

extern "C" int kush_sm100_append(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, const void* k_new,
                                 const void* v_new, int64_t k_stride, int64_t v_stride, int32_t* seq_lens,
                                 int32_t pos_offset, int32_t advance, const int32_t* tail_idx, void* cache,
                                 int64_t block_stride, int64_t head_stride, void* tail_k, const int32_t* block_table,
                                 int64_t max_pages, int32_t hkv, int32_t n_seqs, void* stream) {
    if (n_seqs < 0 || hkv < 1) return set_error(KUSH_ERR_ARG, "kush_sm100_append: n_seqs %d, hkv %d", n_seqs, hkv);
    if (n_seqs == 0) return KUSH_OK;
    if (!k_new || !v_new || !seq_lens || !tail_idx || !cache || !tail_k || !block_table)
        return set_error(KUSH_ERR_ARG, "kush_sm100_append: null pointer");
    int rc = dispatch_fmt(head_dim, bits, page, dtype, [&](auto D, auto B, auto P, auto in) {
        return launch_append<D.value, B.value, P.value, decltype(in)>(
            k_new, v_new, k_stride, v_stride, seq_lens, pos_offset, advance, tail_idx, cache, block_stride, head_stride,
            tail_k, block_table, max_pages, hkv, n_seqs, static_cast<cudaStream_t>(stream));
    });
    if (rc == KUSH_ERR_UNSUPPORTED)
        return set_error(rc, "kush_sm100_append: unsupported head_dim %d / bits %d / page %d / dtype %d", head_dim, bits,
                         page, dtype);
    return rc;
}

extern "C" int kush_sm100_write(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, const void* k_new,
                                const void* v_new, int64_t k_stride, int64_t v_stride, const int32_t* query_start_loc,
                                const int32_t* seq_lens, const int32_t* tail_idx, const int32_t* job_seq,
                                const int32_t* job_page, int32_t mode, void* cache, int64_t block_stride,
                                int64_t head_stride, void* tail_k, const int32_t* block_table, int64_t max_pages,
                                int32_t hkv, int32_t n_jobs, void* stream) {
    if (n_jobs < 0 || hkv < 1 || mode < 0 || mode > 2)
        return set_error(KUSH_ERR_ARG, "kush_sm100_write: n_jobs %d, hkv %d, mode %d", n_jobs, hkv, mode);
    if (n_jobs == 0) return KUSH_OK;
    if (!k_new || !v_new || !query_start_loc || !seq_lens || !tail_idx || !job_seq || !job_page || !cache || !tail_k ||
        !block_table)
        return set_error(KUSH_ERR_ARG, "kush_sm100_write: null pointer");
    int rc = dispatch_fmt(head_dim, bits, page, dtype, [&](auto D, auto B, auto P, auto in) {
        return launch_write<D.value, B.value, P.value, decltype(in)>(
            k_new, v_new, k_stride, v_stride, query_start_loc, seq_lens, tail_idx, job_seq, job_page, mode, cache,
            block_stride, head_stride, tail_k, block_table, max_pages, hkv, n_jobs, static_cast<cudaStream_t>(stream));
    });
    if (rc == KUSH_ERR_UNSUPPORTED)
        return set_error(rc, "kush_sm100_write: unsupported head_dim %d / bits %d / page %d / dtype %d", head_dim, bits,
                         page, dtype);
    return rc;
}
