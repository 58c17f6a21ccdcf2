// Quantize-on-write kernels: decode appends and ragged (prefill / chunked prefill) writes into page records.
// Bit-exact with the reference quantizer (kushkash/kush/quant.mojo:25-50) through kush_common.cuh's qparams/qcode.
//
// Work split on the GPU: a V token row is one warp (per-token range = warp min/max, lane holds dims lane + 32i);
// a K page is one thread per channel (int8) or per channel pair (int4: dims j and j + D/2 share a byte), reading
// the page column-wise.  The decode append reads its one row per head straight from global memory; the bulk write
// stages a page's rows in shared memory with 16-byte loads and writes the assembled record with 16-byte stores.
#include <stdio.h>

#include <atomic>

#include "kush_async.cuh"
#include "kush_common.cuh"

namespace kush {

// one warp: V token row x (lane l holding dims l + 32 i) -> row t of the record (per-token range: the row's final
// encoding) (kushkash/kush/gpu.mojo:163-188 _quantize_v_row)
template <int D, int BITS, int P>
__device__ __forceinline__ void quantize_v_vals(const float (&x)[D / WARP], uint8_t* __restrict__ rec, int t, int lane) {
    using F = Fmt<D, BITS, P>;
    constexpr int R = D / WARP;
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < R; i++) {
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

// one warp: V token row src[0:D] -> row t of the record
template <int D, int BITS, int P, class IN>
__device__ __forceinline__ void quantize_v_row(const IN* __restrict__ src, uint8_t* __restrict__ rec, int t, int lane) {
    float x[D / WARP];
#pragma unroll
    for (int i = 0; i < D / WARP; i++) x[i] = to_f32(src[lane + WARP * i]);
    quantize_v_vals<D, BITS, P>(x, rec, t, lane);
}

// K of one page by the threads of a block (kushkash/kush/gpu.mojo:121-160 _quantize_k_page): per-channel range
// over the P tokens; token row t < split comes from ka + t*sa (the tail), the rest from kb + (t - split)*skb.
// Thread `tid` of `nth` takes channels tid, tid + nth, ...
template <int D, int BITS, int P, class IN>
__device__ __forceinline__ void quantize_k_page(const IN* __restrict__ ka, int64_t sa, const IN* __restrict__ kb,
                                                int64_t skb, int split, uint8_t* __restrict__ rec, int tid, int nth) {
    using F = Fmt<D, BITS, P>;
    constexpr int NCH = BITS == 8 ? D : D / 2;             // threads with work: channel (int8) or channel pair (int4)
    for (int c = tid; c < NCH; c += nth) {
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
                                                   const int32_t* __restrict__ block_table, int64_t max_pages, int H,
                                                   int rot) {
    pdl_wait();                                       // previous kernel on the stream done
    pdl_trigger();                                    // the decode after it may launch (it waits for this grid)
    const int s = blockIdx.x, d = threadIdx.x, lane = d % WARP, w = d / WARP;
    constexpr int NW = D / WARP, R = D / WARP;
    const int64_t pos = int64_t(seq_lens[s]) + pos_offset;
    if (pos < 0) return;                                   // padding row
    const int slot = int(pos % P);
    const int64_t tb = int64_t(tail_idx[s]) * H * P * D;
    const int64_t blk = block_table[s * max_pages + pos / P];
    if (rot) {
        // rotated rows (canonical FWHT, rounded to IN: what kush_sm100_fwht would have handed over), one warp per head
        for (int h = w; h < H; h += NW) {
            float x[R];
#pragma unroll
            for (int i = 0; i < R; i++) x[i] = to_f32(k_new[s * k_stride + h * D + lane + WARP * i]);
            fwht_warp<D>(x, lane);
#pragma unroll
            for (int i = 0; i < R; i++) tail_k[tb + (int64_t(h) * P + slot) * D + lane + WARP * i] = from_f32<IN>(x[i]);
#pragma unroll
            for (int i = 0; i < R; i++) x[i] = to_f32(v_new[s * v_stride + h * D + lane + WARP * i]);
            fwht_warp<D>(x, lane);
#pragma unroll
            for (int i = 0; i < R; i++) x[i] = to_f32(from_f32<IN>(x[i]));
            quantize_v_vals<D, BITS, P>(x, rec_at(cache, blk, h, block_stride, head_stride), slot, lane);
        }
    } else {
        for (int h = 0; h < H; h++) tail_k[tb + (int64_t(h) * P + slot) * D + d] = k_new[s * k_stride + h * D + d];
        for (int h = w; h < H; h += NW)
            quantize_v_row<D, BITS, P, IN>(v_new + s * v_stride + h * D, rec_at(cache, blk, h, block_stride, head_stride),
                                           slot, lane);
    }
    __syncthreads();                                       // tail rows visible to the page quantizer; seq_lens read
    if (slot == P - 1) {
        // each head's P tail rows into shared memory first, every load in flight at once (read from global memory
        // inside the quantizer's row loops, they cost a round trip every few rows: ~25 us for 4 heads at page 32)
        __shared__ __align__(16) IN krows[P * D];
        const bool vec = (reinterpret_cast<uintptr_t>(tail_k) & 15) == 0;
        for (int h = 0; h < H; h++) {
            const IN* t0 = tail_k + tb + int64_t(h) * P * D;
            if (vec) {
                for (int c = threadIdx.x; c < P * D * int(sizeof(IN)) / 16; c += blockDim.x)
                    reinterpret_cast<uint4*>(krows)[c] = reinterpret_cast<const uint4*>(t0)[c];
            } else {
                for (int c = threadIdx.x; c < P * D; c += blockDim.x) krows[c] = t0[c];
            }
            __syncthreads();
            quantize_k_page<D, BITS, P, IN>(krows, D, krows, D, P, rec_at(cache, blk, h, block_stride, head_stride),
                                            threadIdx.x, blockDim.x);
            __syncthreads();                                // krows is reused by the next head
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
    if (job_seq[j] < 0) return;                                     // a padding job (kush_sm100_write_jobs)
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

// ------------------------------------------------------------------ streaming bulk write (fp16 / bf16 inputs)
// The ragged write again, as a persistent kernel: every warp owns a stream of (job, kv head) items (item = job * H +
// head; warp g of the grid takes items g, g + W, g + 2W, ...) and a ring of NS shared-memory slots.  An item whose
// page is entirely new and complete (every page of a prefill chunk but its first and last) is a "full" item: its P
// K rows and P V rows are brought into a slot by 2P one-row bulk copies (cp.async.bulk, mbarrier completion, no
// multicast), issued NS - 1 items ahead, and encoded from there with packed arithmetic straight into the record
// (16-bit min / max on the raw inputs, fp32x2 code arithmetic, byte packing with IMAD / PRMT, 4 to 16-byte stores).
// Other items (a page that continues the old tail, a sequence's last partial page, mode 1) take the warp-level
// version of the per-token path above.  Job metadata (sequence, page, offsets, block id) is prefetched 32 items at a
// time, one item per lane.
//
// Scale arithmetic, bit-exact with qparams: (mx - mn) / (2^BITS - 1) by Markstein's correction step (q0 = d * R,
// r = fma(-q0, L, d), q = fma(r, R, q0) with R = RN(1 / L): the correctly rounded quotient when q0 is within an ulp
// and nothing under- or overflows; other d take the IEEE divide), and 1 / s for the fp16 scale s by the hardware
// reciprocal approximation plus one Newton step.  kush_sm100_selfcheck verifies both exhaustively against IEEE
// division: every fp32 d of the Markstein range, every fp16 s.
__device__ int g_write_error = 0;              // set when a bounded wait of the streaming write gave up

template <class IN> struct Pair16;
template <> struct Pair16<__nv_bfloat16> {
    static __device__ __forceinline__ float lo(uint32_t w) { return __uint_as_float(w << 16); }
    static __device__ __forceinline__ float hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
    // hi(w) if up else lo(w), one PRMT
    static __device__ __forceinline__ float half(uint32_t w, bool up) { return __uint_as_float(prmt(w, 0, up ? 0x3244 : 0x1044)); }
    static __device__ __forceinline__ uint32_t min2(uint32_t a, uint32_t b) {
        uint32_t r;
        asm("min.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
        return r;
    }
    static __device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b) {
        uint32_t r;
        asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
        return r;
    }
};
template <> struct Pair16<__half> {
    static __device__ __forceinline__ float lo(uint32_t w) { return __half2float(__ushort_as_half(uint16_t(w))); }
    static __device__ __forceinline__ float hi(uint32_t w) { return __half2float(__ushort_as_half(uint16_t(w >> 16))); }
    static __device__ __forceinline__ float half(uint32_t w, bool up) { return __half2float(__ushort_as_half(uint16_t(up ? w >> 16 : w))); }
    static __device__ __forceinline__ uint32_t min2(uint32_t a, uint32_t b) {
        uint32_t r;
        asm("min.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
        return r;
    }
    static __device__ __forceinline__ uint32_t max2(uint32_t a, uint32_t b) {
        uint32_t r;
        asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
        return r;
    }
};

// (mx - mn) / (2^BITS - 1), correctly rounded (Markstein), IEEE divide outside [2^-100, 2^100]
template <int BITS>
__device__ __forceinline__ float div_levels(float d) {
    constexpr float L = float((1 << BITS) - 1);
    constexpr float R = 1.0f / L;
    const float q0 = __fmul_rn(d, R);
    float q = __fmaf_rn(__fmaf_rn(-q0, L, d), R, q0);
    if (!(d <= 0x1p100f && (d >= 0x1p-100f || d == 0.0f))) q = __fdiv_rn(d, L);
    return q;
}

// qparams' `s > 0 ? 1 / s : 0` for an fp16-representable s: the hardware reciprocal approximation and one
// Newton-Raphson step (e = 1 - s r, r' = r + r e), 0 unless s > 0 and finite; RN(1 / s) for every fp16 s (checked
// exhaustively by kush_sm100_selfcheck).
__device__ __forceinline__ float rcp_nr(float s) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(s));
    r = __fmaf_rn(r, __fmaf_rn(-s, r, 1.0f), r);
    return (s > 0.0f && s <= 65504.0f) ? r : 0.0f;
}

// fp32x2 arithmetic of the scale and code paths (PTX with explicit rounding).  One measured hazard on sm_100a: a
// packed multiply whose result feeds a packed add directly could come out rounded once, as by one fused
// multiply-add, even with -fmad=false; the magic add after the code multiply is therefore two scalar __fadd_rn.
__device__ __forceinline__ uint64_t f2_bits(float2 a) {
    return uint64_t(__float_as_uint(a.x)) | uint64_t(__float_as_uint(a.y)) << 32;
}
__device__ __forceinline__ float2 bits_f2(uint64_t r) {
    return make_float2(__uint_as_float(uint32_t(r)), __uint_as_float(uint32_t(r >> 32)));
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return bits_f2(r);
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
    return bits_f2(r);
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
    return bits_f2(r);
}

// div_levels for two values at once (the form the write kernel uses)
template <int BITS>
__device__ __forceinline__ float2 div_levels2(float2 d) {
    constexpr float L = float((1 << BITS) - 1), R = 1.0f / L;
    const float2 q0 = mul2_rn(d, make_float2(R, R));
    float2 q = fma2_rn(fma2_rn(q0, make_float2(-L, -L), d), make_float2(R, R), q0);
    if (!(d.x <= 0x1p100f && (d.x >= 0x1p-100f || d.x == 0.0f))) q.x = __fdiv_rn(d.x, L);
    if (!(d.y <= 0x1p100f && (d.y >= 0x1p-100f || d.y == 0.0f))) q.y = __fdiv_rn(d.y, L);
    return q;
}

// qparams for two ranges at once (x: first, y: second), fp32x2 arithmetic; also returns the fp16 scales and biases
// as half2 bits and whether any value of either range can need qcode's clamp: the code of a value is monotone in
// it, so when the codes of both ends (mn, mx) are inside the code range, every code is.
template <int BITS>
__device__ __forceinline__ bool qparams2(float2 mn, float2 mx, uint32_t& sh2, uint32_t& bh2,
                                         float2& b, float2& inv) {
    constexpr float HALFF = float(1 << (BITS - 1));
    constexpr float LO = -HALFF - 0.5f, HI = HALFF - 0.5f;          // round(y) in range <=> LO <= y < HI
    const float2 m1 = make_float2(-1.0f, -1.0f);
    const float2 d = fma2_rn(mn, m1, mx);                       // mx - mn
    const float2 q = div_levels2<BITS>(d);
    const __half2 s16 = __floats2half2_rn(q.x, q.y);
    const float2 s = __half22float2(s16);
    const float2 bp = fma2_rn(s, make_float2(HALFF, HALFF), mn);   // mn + s * HALF (the product is exact)
    const __half2 b16 = __floats2half2_rn(bp.x, bp.y);
    b = __half22float2(b16);
    inv = make_float2(rcp_nr(s.x), rcp_nr(s.y));
    sh2 = *reinterpret_cast<const uint32_t*>(&s16);
    bh2 = *reinterpret_cast<const uint32_t*>(&b16);
    const float2 ylo = mul2_rn(fma2_rn(b, m1, mn), inv), yhi = mul2_rn(fma2_rn(b, m1, mx), inv);
    return !(ylo.x >= LO && ylo.y >= LO && yhi.x < HI && yhi.y < HI);
}

// codes of a pair of values (x.x, x.y) against their (bias, 1 / scale) pairs: float bits whose low byte is the code
// (int8: two's complement; int4: code + 8), by qcode's round-half-even magic add; CL: with qcode's clamp (taken
// before the rounding: rounding is monotone and the bounds are integers, so the codes are the same)
template <int BITS, bool CL>
__device__ __forceinline__ uint2 code_bits(float2 x, float2 b, float2 iv) {
    constexpr float LO = -float(1 << (BITS - 1)), HI = float((1 << (BITS - 1)) - 1);
    constexpr float MAGIC = BITS == 4 ? 12582920.0f : 12582912.0f;       // 1.5 * 2^23 (+ 8)
    float2 y = mul2_rn(fma2_rn(b, make_float2(-1.0f, -1.0f), x), iv);
    if constexpr (CL) {
        y.x = fminf(fmaxf(y.x, LO), HI);
        y.y = fminf(fmaxf(y.y, LO), HI);
    }
    return make_uint2(__float_as_uint(__fadd_rn(y.x, MAGIC)), __float_as_uint(__fadd_rn(y.y, MAGIC)));
}

template <class IN> __device__ __forceinline__ float2 f2_of(uint32_t w) {
    return make_float2(Pair16<IN>::lo(w), Pair16<IN>::hi(w));
}

// int4: two code bytes (bits 0-15, each still XOR 0x88) of lo dims (a.lo, a.hi) and hi dims (b.lo, b.hi)
template <class IN, bool CL>
__device__ __forceinline__ uint32_t unit4(uint32_t a, uint32_t b, float2 b0, float2 iv0, float2 b1, float2 iv1) {
    const float2 fa = f2_of<IN>(a), fb = f2_of<IN>(b);
    const uint2 e0 = code_bits<4, CL>(make_float2(fa.x, fb.x), b0, iv0);
    const uint2 e1 = code_bits<4, CL>(make_float2(fa.y, fb.y), b1, iv1);
    return prmt(e0.y * 16u + e0.x, e1.y * 16u + e1.x, 0x0040);          // low byte: (lo + 8) | (hi + 8) << 4
}
// int8: two code bytes (bits 0-15) of dims (a.lo, a.hi)
template <class IN, bool CL>
__device__ __forceinline__ uint32_t unit8(uint32_t a, float2 b, float2 iv) {
    const uint2 e = code_bits<8, CL>(f2_of<IN>(a), b, iv);
    return prmt(e.x, e.y, 0x0040);
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// qparams for one range, scalar (bit-exact as qparams2); returns whether a code of the range can need the clamp
template <int BITS>
__device__ __forceinline__ bool qparams1(float mn, float mx, uint16_t& sh, uint16_t& bh, float& b,
                                         float& inv) {
    constexpr float HALFF = float(1 << (BITS - 1));
    constexpr float LO = -HALFF - 0.5f, HI = HALFF - 0.5f;
    const __half s16 = __float2half_rn(div_levels<BITS>(__fsub_rn(mx, mn)));
    const float s = __half2float(s16);
    const __half b16 = __float2half_rn(__fmaf_rn(s, HALFF, mn));       // mn + s * HALF (the product is exact)
    b = __half2float(b16);
    inv = rcp_nr(s);
    sh = __half_as_ushort(s16);
    bh = __half_as_ushort(b16);
    const float ylo = __fmul_rn(__fsub_rn(mn, b), inv), yhi = __fmul_rn(__fsub_rn(mx, b), inv);
    return !(ylo >= LO && yhi < HI);
}

// Streaming-write geometry.  An item is one page of one kv head.  P = 16: one warp encodes the item's V rows and
// K page from one ring slot.  P = 32: two warps take the item, warp 0 its V rows and warp 1 its K page, each from
// its own ring of slots holding only the rows it encodes (no slot is shared, so the two never wait on each other).
template <int D, int BITS, int P, class IN>
struct WS {
    using F = Fmt<D, BITS, P>;
    static constexpr int G = P / 16;                                // warps per item
    static constexpr int ROWB = 2 * D;                              // bytes of an input row
    static constexpr int RSTR = ROWB + 16;                          // slot row stride (skews banks across rows)
    // K: lane = KC code bytes of a row (int4: KC lo dims + KC hi dims; int8: KC dims), LW lanes per token set, TS
    // token sets of TPS rows (ranges combined across sets by shuffles)
    static constexpr int DC = F::DC;
    static constexpr int KC = DC / 32 > 4 ? DC / 32 : 4;
    static constexpr int LW = DC / KC, TS = 32 / LW, TPS = P / TS;
    // slot: K rows (the rows of token set k shifted by k KGAP bytes: the sets read in one shared-memory wavefront
    // then hit disjoint banks) unless the warp encodes V only, then the V rows from VOFF unless it encodes K only
    static constexpr int KGAP = 8 * LW;
    static constexpr int KBYTES = P * RSTR + (TS - 1) * KGAP;
    static constexpr int VOFF = G == 1 ? KBYTES : 0;
    static constexpr int STAGE = G == 1 ? KBYTES + P * RSTR : (KBYTES > P * RSTR ? KBYTES : P * RSTR);
    static constexpr int NS = 2;                                    // ring slots per warp
    static constexpr int NW = 4 * NS * STAGE <= 73728 ? 4 : 2;      // warps per CTA
    static constexpr int NST = NW / G;                              // item streams per CTA
    static constexpr int OFF_BAR = 0;                               // full[NW][NS]
    static constexpr int OFF_STAGE = 128;
    static constexpr int SMEM = OFF_STAGE + NW * NS * STAGE;
    // V: GL lanes per row, VPL values per lane (int4: VPL/2 lo dims + the matching hi dims), RPP rows per pass
    static constexpr int GL = D / 64 > 2 ? D / 64 : 2;
    static constexpr int VPL = D / GL, VW = VPL / 2, RPP = 32 / GL, VPASS = P / RPP;
    static constexpr int NU = KC / 2;                               // 2-byte code units per row per lane
    static constexpr int KWD = BITS == 4 ? KC : KC / 2;             // input words per row per lane
    static constexpr int NPR = BITS == 4 ? 2 * NU : NU;             // channel pairs per lane
    static constexpr bool KREG = TPS * KWD <= 32;                   // keep the K words in registers between passes
    __host__ __device__ static constexpr int kpos(int t) { return t * RSTR + (t / TPS) * KGAP; }
    static_assert(P == 16 * G && NW % G == 0 && P % RPP == 0 && NW * NS * 8 <= OFF_STAGE && VOFF % 16 == 0 &&
                      STAGE >= P * ROWB && STAGE % 16 == 0,
                  "geometry");
};

// the VW words of V row `row` this lane encodes: int4: lo dims [j VPL/2, (j+1) VPL/2), then the same hi dims;
// int8: dims [j VPL, (j+1) VPL)
template <int D, int BITS, int P, class IN>
__device__ __forceinline__ void v_words(const uint8_t* row, int j, uint32_t (&w)[WS<D, BITS, P, IN>::VW]) {
    using C = WS<D, BITS, P, IN>;
    constexpr int NQ = C::VW / 4;                                   // 16-byte loads
#pragma unroll
    for (int q = 0; q < NQ; q++) {
        int off;
        if constexpr (BITS == 4) off = q < NQ / 2 ? j * C::VPL + 16 * q : D + j * C::VPL + 16 * (q - NQ / 2);
        else off = 2 * j * C::VPL + 16 * q;
        const uint4 a = lds128(row + off);
        w[4 * q] = a.x;
        w[4 * q + 1] = a.y;
        w[4 * q + 2] = a.z;
        w[4 * q + 3] = a.w;
    }
}

template <int D, int BITS, int P, class IN, bool CL>
__device__ __forceinline__ void v_encode(const uint32_t (&w)[WS<D, BITS, P, IN>::VW], float bias, float inv,
                                         uint8_t* dst) {
    constexpr int VW = WS<D, BITS, P, IN>::VW;
    const float2 b = make_float2(bias, bias), iv = make_float2(inv, inv);
    if constexpr (BITS == 4) {
        constexpr int NO = VW / 4;                                  // output words (VW/2 units of 2 bytes)
        uint32_t o[NO];
#pragma unroll
        for (int k = 0; k < NO; k++)
            o[k] = prmt(unit4<IN, CL>(w[2 * k], w[VW / 2 + 2 * k], b, iv, b, iv),
                        unit4<IN, CL>(w[2 * k + 1], w[VW / 2 + 2 * k + 1], b, iv, b, iv), 0x5410) ^ 0x88888888u;
#pragma unroll
        for (int k = 0; k < NO; k += 4) *reinterpret_cast<uint4*>(dst + 4 * k) = make_uint4(o[k], o[k + 1], o[k + 2], o[k + 3]);
    } else {
        constexpr int NO = VW / 2;
        uint32_t o[NO];
#pragma unroll
        for (int k = 0; k < NO; k++) o[k] = prmt(unit8<IN, CL>(w[2 * k], b, iv), unit8<IN, CL>(w[2 * k + 1], b, iv), 0x5410);
#pragma unroll
        for (int k = 0; k < NO; k += 4) *reinterpret_cast<uint4*>(dst + 4 * k) = make_uint4(o[k], o[k + 1], o[k + 2], o[k + 3]);
    }
}

// pairwise min / max tree over n words
template <class IN, int N>
__device__ __forceinline__ void range_tree(const uint32_t (&w)[N], uint32_t& m, uint32_t& M) {
    using PR = Pair16<IN>;
    uint32_t a[N / 2], b[N / 2];
#pragma unroll
    for (int i = 0; i < N / 2; i++) {
        a[i] = PR::min2(w[2 * i], w[2 * i + 1]);
        b[i] = PR::max2(w[2 * i], w[2 * i + 1]);
    }
#pragma unroll
    for (int s = 1; s < N / 2; s <<= 1)
#pragma unroll
        for (int i = 0; i + s < N / 2; i += 2 * s) {
            a[i] = PR::min2(a[i], a[i + s]);
            b[i] = PR::max2(b[i], b[i + s]);
        }
    m = a[0];
    M = b[0];
}

// the V rows of a full page from the slot: row pass RPP + lane / GL, lane part j = lane % GL
template <int D, int BITS, int P, class IN>
__device__ __forceinline__ void ws_v_rows(const uint8_t* vbuf, uint8_t* rec, int lane) {
    using C = WS<D, BITS, P, IN>;
    using F = typename C::F;
    using PR = Pair16<IN>;
    const int j = lane % C::GL;
#pragma unroll 1
    for (int pass = 0; pass < C::VPASS; pass++) {
        const int r = pass * C::RPP + lane / C::GL;
        uint32_t w[C::VW];
        v_words<D, BITS, P, IN>(vbuf + r * C::RSTR, j, w);
        uint32_t m, M;
        range_tree<IN, C::VW>(w, m, M);
        const uint32_t nM = M ^ 0x80008000u;                        // -max: both ranges reduce as one min
        uint32_t mm = PR::min2(prmt(m, nM, 0x5410), prmt(m, nM, 0x7632));       // (min, -max)
#pragma unroll
        for (int o = C::GL / 2; o; o >>= 1) mm = PR::min2(mm, __shfl_xor_sync(0xffffffffu, mm, o));
        uint16_t sh, bh;
        float b, inv;
        const bool need = qparams1<BITS>(PR::lo(mm), -PR::hi(mm), sh, bh, b, inv);
        if (j == 0) {
            reinterpret_cast<uint16_t*>(rec + F::OFF_VS)[r] = sh;
            reinterpret_cast<uint16_t*>(rec + F::OFF_VB)[r] = bh;
        }
        uint8_t* dst = rec + F::OFF_VQ + r * F::DC + j * (F::DC / C::GL);
        if (__any_sync(0xffffffffu, need)) v_encode<D, BITS, P, IN, true>(w, b, inv, dst);
        else v_encode<D, BITS, P, IN, false>(w, b, inv, dst);
    }
}

// this lane's K input words of row t: int4: KC/2 words of lo dims [e0, e0 + KC), then the same of hi dims;
// int8: KC/2 words of dims [e0, e0 + KC); e0 = the lane's first code byte
template <int D, int BITS, int P, class IN>
__device__ __forceinline__ void ws_k_words(const uint8_t* kbuf, int t, int e0, uint32_t (&w)[WS<D, BITS, P, IN>::KWD]) {
    using C = WS<D, BITS, P, IN>;
    const uint8_t* row = kbuf + C::kpos(t) + 2 * e0;
    if constexpr (C::KC == 4) {
        const uint2 a = *reinterpret_cast<const uint2*>(row);
        w[0] = a.x;
        w[1] = a.y;
        if constexpr (BITS == 4) {
            const uint2 b = *reinterpret_cast<const uint2*>(row + D);
            w[2] = b.x;
            w[3] = b.y;
        }
    } else {                                                         // int8, KC = 8
        const uint4 a = lds128(row);
        w[0] = a.x;
        w[1] = a.y;
        w[2] = a.z;
        w[3] = a.w;
    }
}

template <int D, int BITS, int P, class IN, bool CL>
__device__ __forceinline__ void k_encode(const uint32_t (&w)[WS<D, BITS, P, IN>::KWD], const float2 (&b)[WS<D, BITS, P, IN>::NPR],
                                         const float2 (&iv)[WS<D, BITS, P, IN>::NPR], uint8_t* dst) {
    using C = WS<D, BITS, P, IN>;
    constexpr int NU = C::NU;
    uint32_t u16[NU];
#pragma unroll
    for (int u = 0; u < NU; u++) {
        if constexpr (BITS == 4) u16[u] = unit4<IN, CL>(w[u], w[NU + u], b[2 * u], iv[2 * u], b[2 * u + 1], iv[2 * u + 1]);
        else u16[u] = unit8<IN, CL>(w[u], b[u], iv[u]);
    }
    if constexpr (NU == 2) {
        uint32_t o = prmt(u16[0], u16[1], 0x5410);
        if constexpr (BITS == 4) o ^= 0x88888888u;
        *reinterpret_cast<uint32_t*>(dst) = o;
    } else {
        *reinterpret_cast<uint2*>(dst) = make_uint2(prmt(u16[0], u16[1], 0x5410), prmt(u16[2], u16[3], 0x5410));
    }
}

// The K page of a full page from the slot, in three phases (ranges, scale parameters, codes) so that a caller can
// interleave them with the V rows' phases.
template <int D, int BITS, int P, class IN>
struct KPage {
    using C = WS<D, BITS, P, IN>;
    using F = typename C::F;
    using PR = Pair16<IN>;
    static constexpr int KWD = C::KWD, NU = C::NU, NPR = C::NPR;
    static constexpr int TR = C::KREG ? C::TPS : 1;                  // rows whose words stay in registers
    static constexpr int OWN = NPR >= C::TS ? NPR / C::TS : 1;       // channel pairs whose scales a lane computes
    const uint8_t* kbuf;
    int lane, t0, e0;
    uint32_t kw[TR][KWD], mn[KWD], mx[KWD];
    float2 b[NPR], iv[NPR];
    bool need;

    __device__ __forceinline__ KPage(const uint8_t* kb, int lane_) : kbuf(kb), lane(lane_), need(false) {
        t0 = (lane / C::LW) * C::TPS;
        e0 = (lane % C::LW) * C::KC;                                 // first code byte of the lane
    }

    // per-channel (min, max) over the P rows: in-lane over the set's TPS rows, then across the TS sets
    __device__ __forceinline__ void ranges() {
        ws_k_words<D, BITS, P, IN>(kbuf, t0, e0, kw[0]);
#pragma unroll
        for (int i = 0; i < KWD; i++) mn[i] = mx[i] = kw[0][i];
#pragma unroll
        for (int t = 1; t < C::TPS; t++) {
            uint32_t w[KWD];
            ws_k_words<D, BITS, P, IN>(kbuf, t0 + t, e0, w);
#pragma unroll
            for (int i = 0; i < KWD; i++) {
                if constexpr (C::KREG) kw[t < TR ? t : 0][i] = w[i];
                mn[i] = PR::min2(mn[i], w[i]);
                mx[i] = PR::max2(mx[i], w[i]);
            }
        }
#pragma unroll
        for (int o = C::LW; o < 32; o <<= 1)
#pragma unroll
            for (int i = 0; i < KWD; i++) {
                mn[i] = PR::min2(mn[i], __shfl_xor_sync(0xffffffffu, mn[i], o));
                mx[i] = PR::max2(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], o));
            }
    }

    // channel pairs: int4 pair q = (lo dim e0 + q, hi dim e0 + q); int8 pair q = (dims e0 + 2q, e0 + 2q + 1).
    // The TS token sets hold the same ranges: set k computes pairs [k OWN, (k + 1) OWN), stores their scales and
    // biases, and every lane takes the other pairs' (bias, 1 / scale) from their owners by shuffles.
    __device__ __forceinline__ void params(uint8_t* rec) {
        const int set = lane / C::LW;
        float2 bo[OWN], ivo[OWN];
        uint32_t sh[OWN], bh[OWN];
#pragma unroll
        for (int o = 0; o < OWN; o++) {
            // the words of pair q = (set OWN + o) % NPR, chosen among the TS candidates by selects (no indexing
            // by a run-time value: every lane runs the same qparams2)
            uint32_t a0 = 0, a1 = 0, m0 = 0, m1 = 0;
            bool up = false;
#pragma unroll
            for (int k = 0; k < C::TS; k++) {
                const int q = (k * OWN + o) % NPR;
                const bool pick = set == k;
                if constexpr (BITS == 4) {           // pair q: unit q / 2, low (q even) or high (q odd) halves
                    a0 = pick ? mn[q / 2] : a0;
                    a1 = pick ? mn[NU + q / 2] : a1;
                    m0 = pick ? mx[q / 2] : m0;
                    m1 = pick ? mx[NU + q / 2] : m1;
                    up = pick ? (q & 1) != 0 : up;
                } else {                             // pair q: both halves of word q
                    a0 = pick ? mn[q] : a0;
                    m0 = pick ? mx[q] : m0;
                }
            }
            float2 lo_, hi_;
            if constexpr (BITS == 4) {
                lo_ = make_float2(PR::half(a0, up), PR::half(a1, up));
                hi_ = make_float2(PR::half(m0, up), PR::half(m1, up));
            } else {
                lo_ = f2_of<IN>(a0);
                hi_ = f2_of<IN>(m0);
            }
            need |= qparams2<BITS>(lo_, hi_, sh[o], bh[o], bo[o], ivo[o]);
        }
        if (set * OWN < NPR) {
            const int q0 = set * OWN;
            if constexpr (BITS == 4) {
                // pair q: ks[e0 + q] = low half, ks[D/2 + e0 + q] = high half
                if constexpr (OWN >= 2) {
#pragma unroll
                    for (int o = 0; o < OWN; o += 2) {
                        const int e = e0 + q0 + o;
                        *reinterpret_cast<uint32_t*>(rec + F::OFF_KS + 2 * e) = prmt(sh[o], sh[o + 1], 0x5410);
                        *reinterpret_cast<uint32_t*>(rec + F::OFF_KS + D + 2 * e) = prmt(sh[o], sh[o + 1], 0x7632);
                        *reinterpret_cast<uint32_t*>(rec + F::OFF_KB + 2 * e) = prmt(bh[o], bh[o + 1], 0x5410);
                        *reinterpret_cast<uint32_t*>(rec + F::OFF_KB + D + 2 * e) = prmt(bh[o], bh[o + 1], 0x7632);
                    }
                } else {
                    const int e = e0 + q0;
                    reinterpret_cast<uint16_t*>(rec + F::OFF_KS)[e] = uint16_t(sh[0]);
                    reinterpret_cast<uint16_t*>(rec + F::OFF_KS)[D / 2 + e] = uint16_t(sh[0] >> 16);
                    reinterpret_cast<uint16_t*>(rec + F::OFF_KB)[e] = uint16_t(bh[0]);
                    reinterpret_cast<uint16_t*>(rec + F::OFF_KB)[D / 2 + e] = uint16_t(bh[0] >> 16);
                }
            } else {
#pragma unroll
                for (int o = 0; o < OWN; o++) {
                    const int e = e0 + 2 * (q0 + o);
                    *reinterpret_cast<uint32_t*>(rec + F::OFF_KS + 2 * e) = sh[o];
                    *reinterpret_cast<uint32_t*>(rec + F::OFF_KB + 2 * e) = bh[o];
                }
            }
        }
#pragma unroll
        for (int q = 0; q < NPR; q++) {
            const int src = lane % C::LW + (q / OWN) * C::LW;
            b[q] = make_float2(__shfl_sync(0xffffffffu, bo[q % OWN].x, src), __shfl_sync(0xffffffffu, bo[q % OWN].y, src));
            iv[q] = make_float2(__shfl_sync(0xffffffffu, ivo[q % OWN].x, src),
                                __shfl_sync(0xffffffffu, ivo[q % OWN].y, src));
        }
    }

    __device__ __forceinline__ void codes(uint8_t* rec) {
        uint8_t* dst = rec + t0 * F::DC + e0;
        const bool cl = __any_sync(0xffffffffu, need);
#pragma unroll
        for (int t = 0; t < C::TPS; t++) {
            uint32_t w[KWD];
            if constexpr (C::KREG) {
#pragma unroll
                for (int i = 0; i < KWD; i++) w[i] = kw[t][i];
            } else {
                ws_k_words<D, BITS, P, IN>(kbuf, t0 + t, e0, w);
            }
            if (cl) k_encode<D, BITS, P, IN, true>(w, b, iv, dst + t * F::DC);
            else k_encode<D, BITS, P, IN, false>(w, b, iv, dst + t * F::DC);
        }
    }
};

// One full page of one kv head from the slot, this warp's share (role 0: V rows, 1: K page; P = 16: both, the
// V and K phases interleaved -- ranges, then every scale parameter (independent chains), then the codes).
template <int D, int BITS, int P, class IN>
__device__ __forceinline__ void ws_item(const uint8_t* buf, uint8_t* rec, int lane, int role) {
    using C = WS<D, BITS, P, IN>;
    using F = typename C::F;
    using PR = Pair16<IN>;
    if constexpr (C::G == 2) {
        if (role == 0) {
            ws_v_rows<D, BITS, P, IN>(buf, rec, lane);
        } else {
            KPage<D, BITS, P, IN> kp(buf, lane);
            kp.ranges();
            kp.params(rec);
            kp.codes(rec);
        }
    } else if constexpr (C::VPASS == 1) {
        KPage<D, BITS, P, IN> kp(buf, lane);
        const int j = lane % C::GL, r = lane / C::GL;
        uint32_t w[C::VW];
        v_words<D, BITS, P, IN>(buf + C::VOFF + r * C::RSTR, j, w);
        uint32_t m, M;
        range_tree<IN, C::VW>(w, m, M);
        const uint32_t nM = M ^ 0x80008000u;                        // -max: both ranges reduce as one min
        uint32_t mm = PR::min2(prmt(m, nM, 0x5410), prmt(m, nM, 0x7632));       // (min, -max)
#pragma unroll
        for (int o = C::GL / 2; o; o >>= 1) mm = PR::min2(mm, __shfl_xor_sync(0xffffffffu, mm, o));
        kp.ranges();
        uint16_t sh, bh;
        float b, inv;
        const bool need = qparams1<BITS>(PR::lo(mm), -PR::hi(mm), sh, bh, b, inv);
        kp.params(rec);
        if (j == 0) {
            reinterpret_cast<uint16_t*>(rec + F::OFF_VS)[r] = sh;
            reinterpret_cast<uint16_t*>(rec + F::OFF_VB)[r] = bh;
        }
        uint8_t* dst = rec + F::OFF_VQ + r * F::DC + j * (F::DC / C::GL);
        if (__any_sync(0xffffffffu, need)) v_encode<D, BITS, P, IN, true>(w, b, inv, dst);
        else v_encode<D, BITS, P, IN, false>(w, b, inv, dst);
        kp.codes(rec);
    } else {
        ws_v_rows<D, BITS, P, IN>(buf + C::VOFF, rec, lane);
        KPage<D, BITS, P, IN> kp(buf, lane);
        kp.ranges();
        kp.params(rec);
        kp.codes(rec);
    }
}

// job metadata of one item, one item per lane (see write_stream_kernel); hf = kv head | full << 30
struct WMeta {
    int row0, hf, blk, s, pg, q0, ctx, total;
};

// one warp: n rows of D 16-bit values (row r at src + r * ss, 16-byte aligned) into shared memory dst (rows packed)
// by 16-byte cp.async copies, all in flight together; cp_async_wait_warp waits for them and publishes them to the warp
template <int D, class IN>
__device__ __forceinline__ void stage_rows_warp(IN* dst, const IN* src, int64_t ss, int n, int lane) {
    constexpr int CPR = D * int(sizeof(IN)) / 16, E = 16 / int(sizeof(IN));
    const uint32_t d0 = smem_u32(dst);
    for (int c = lane; c < n * CPR; c += WARP) {
        const int r = c / CPR, q = c % CPR;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d0 + uint32_t((r * D + q * E) * int(sizeof(IN)))),
                     "l"(src + r * ss + q * E)
                     : "memory");
    }
}

__device__ __forceinline__ void cp_async_wait_warp() {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
}

// one warp: n rows of D 16-bit values from src (row stride ss) to dst (rows packed) in global memory, 16-byte
// accesses, four loads per lane in flight before their stores (src is not written by the kernel)
template <int D, class IN>
__device__ __forceinline__ void copy_rows_warp(IN* dst, const IN* __restrict__ src, int64_t ss, int n, int lane) {
    constexpr int CPR = D * int(sizeof(IN)) / 16, E = 16 / int(sizeof(IN)), B = 4;
    for (int c0 = lane; c0 < n * CPR; c0 += B * WARP) {
        uint4 v[B];
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int c = c0 + b * WARP;
            if (c < n * CPR) v[b] = __ldg(reinterpret_cast<const uint4*>(src + (c / CPR) * ss + (c % CPR) * E));
        }
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int c = c0 + b * WARP;
            if (c < n * CPR) *reinterpret_cast<uint4*>(dst + (c / CPR) * D + (c % CPR) * E) = v[b];
        }
    }
}

template <int D, int BITS, int P, class IN>
__global__ void __launch_bounds__(WS<D, BITS, P, IN>::NW * 32, 3)
    write_stream_kernel(const IN* __restrict__ k_new, const IN* __restrict__ v_new, int64_t k_stride, int64_t v_stride,
                        const int32_t* __restrict__ qsl, const int32_t* __restrict__ seq_lens,
                        const int32_t* __restrict__ tail_idx, const int32_t* __restrict__ job_seq,
                        const int32_t* __restrict__ job_page, int mode, uint8_t* cache, int64_t block_stride,
                        int64_t head_stride, IN* tail_k, const int32_t* __restrict__ block_table, int64_t max_pages,
                        int H, int n_jobs) {
    using C = WS<D, BITS, P, IN>;
    constexpr int FULL = 1 << 30, SKIP = 1 << 29;                    // item flags beside the kv head in hf
    extern __shared__ __align__(128) uint8_t wss[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(wss + C::OFF_BAR);
    const int lane = threadIdx.x % WARP, w = threadIdx.x / WARP;
    const int st = w / C::G, role = w % C::G;                        // item stream of the CTA, role in it
    if (threadIdx.x < C::NW * C::NS) mbar_init(&bars[threadIdx.x], 1);                   // full: the issuing lane
    fence_mbar_init();
    __syncthreads();

    uint8_t* slots = wss + C::OFF_STAGE + w * C::NS * C::STAGE;      // this warp's ring
    const uint32_t bar0 = smem_u32(&bars[w * C::NS]);
    const int64_t n_items = int64_t(n_jobs) * H;
    const int64_t TW = int64_t(gridDim.x) * C::NST;
    const int64_t first = int64_t(blockIdx.x) * C::NST + st;
    const int n_local = first < n_items ? int((n_items - first + TW - 1) / TW) : 0;

    auto load_meta = [&](int batch) {
        WMeta m{0, 0, 0, 0, 0, 0, 0, 0};
        const int64_t it = first + (int64_t(batch) * WARP + lane) * TW;
        if (it < n_items && job_seq[it / H] < 0) {                  // a padding job: no copy, no encode
            m.hf = SKIP;
        } else if (it < n_items) {
            const int64_t j = it / H;
            m.s = job_seq[j];
            m.pg = job_page[j];
            m.q0 = qsl[m.s];
            m.total = seq_lens[m.s];
            m.ctx = m.total - (qsl[m.s + 1] - m.q0);
            m.blk = block_table[int64_t(m.s) * max_pages + m.pg];
            const int ps = m.pg * P;
            m.row0 = m.q0 + ps - m.ctx;
            const bool full = mode != 1 && ps >= m.ctx && ps + P <= m.total;
            m.hf = int(it - j * H) | (full ? FULL : 0);
        }
        return m;
    };
    WMeta cur = load_meta(0), nxt = load_meta(1);
#define KUSH_META(field, use_b, l) __shfl_sync(0xffffffffu, (use_b) ? nxt.field : cur.field, (l))
    // bring the rows of full item i (first input row row0, kv head h) this warp encodes into its slot i % NS:
    // P = 16 K and V rows; P = 32 the V rows (role 0) or the K rows (role 1)
    auto issue = [&](int i, int row0, int h) {
        constexpr int NR = C::G == 1 ? 2 * P : P;
        const uint32_t bar = bar0 + 8u * uint32_t(i % C::NS);
        const uint32_t dst = smem_u32(slots + (i % C::NS) * C::STAGE);
        if (lane == 0)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(uint32_t(NR * C::ROWB))
                         : "memory");
        __syncwarp();
#pragma unroll
        for (int r = lane; r < NR; r += WARP) {
            const bool is_k = C::G == 1 ? r < P : role == 1;
            const int t = C::G == 1 && r >= P ? r - P : r;           // token row of the page
            const IN* src = is_k ? k_new + (int64_t(row0) + t) * k_stride + int64_t(h) * D
                                 : v_new + (int64_t(row0) + t) * v_stride + int64_t(h) * D;
            const uint32_t off = is_k ? C::kpos(t) : C::VOFF + t * C::RSTR;
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                             dst + off),
                         "l"(src), "r"(uint32_t(C::ROWB)), "r"(bar)
                         : "memory");
        }
    };
    // every other item: the per-token path (mode 0 / 1 / 2 as write_kernel) by the role-0 warp of the stream, its
    // slot i % NS as the page's staging rows: [split old tail rows][new rows], loaded by cp.async all at once
    auto general = [&](int i, int l, int h, int blk) {
        const int64_t ps = int64_t(KUSH_META(pg, false, l)) * P, ctx = KUSH_META(ctx, false, l);
        const int64_t total = KUSH_META(total, false, l), q0 = KUSH_META(q0, false, l);
        const int s = KUSH_META(s, false, l);
        const int64_t tb = (int64_t(tail_idx[s]) * H + h) * P * D, hd = int64_t(h) * D;
        const bool complete = ps + P <= total;
        auto stash = [&](int64_t pstart) {
            const int64_t t0 = max(pstart, ctx);
            if (t0 < total)
                copy_rows_warp<D, IN>(tail_k + tb + (t0 - pstart) * D, k_new + (q0 + t0 - ctx) * k_stride + hd, k_stride,
                                      int(total - t0), lane);
        };
        if (mode == 1) {
            if (!complete) stash(ps);
            return;
        }
        uint8_t* rec = rec_at(cache, blk, h, block_stride, head_stride);
        const int r0 = int(max(ps, ctx) - ps), r1 = int(min(ps + P, total) - ps);
        const int split = complete ? int(max(int64_t(0), min(int64_t(P), ctx - ps))) : 0;
        IN* stage = reinterpret_cast<IN*>(slots + (i % C::NS) * C::STAGE);
        stage_rows_warp<D, IN>(stage, tail_k + tb, D, split, lane);                  // old tail rows, before a stash
        stage_rows_warp<D, IN>(stage + split * D, v_new + (q0 + ps + r0 - ctx) * v_stride + hd, v_stride, r1 - r0,
                               lane);
        cp_async_wait_warp();
        if (mode == 2) {
            const int64_t f0 = (ctx / P) * P, last = ((total - 1) / P) * P;
            const bool last_partial = total % P != 0 && total > ctx;
            const bool first_reads_tail = ctx % P != 0 && f0 + P <= total;
            if (last_partial && ((first_reads_tail && last != f0) ? ps == f0 : ps == last)) stash(last);
        }
        for (int r = r0; r < r1; r++) quantize_v_row<D, BITS, P, IN>(stage + (split + r - r0) * D, rec, r, lane);
        if (complete) {
            __syncwarp();                                                            // V rows read: reuse for K
            stage_rows_warp<D, IN>(stage + split * D, k_new + (q0 + ps + split - ctx) * k_stride + hd, k_stride,
                                   P - split, lane);
            cp_async_wait_warp();
            quantize_k_page<D, BITS, P, IN>(stage, D, stage + split * D, D, split, rec, lane, WARP);
        }
        __syncwarp();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the slot may next be filled by a bulk copy
    };

    // full[slot] completes one phase per FULL item of the slot (general items are never issued): phase bit per
    // slot, flipped at each completed wait; the slots with copies in flight are kept for the error path
    uint32_t phase = 0, inflight = 0;
    bool ok = true;
    for (int i = 0; i < C::NS - 1 && i < n_local; i++) {
        const int hf = KUSH_META(hf, false, i);
        if (hf & FULL) {
            issue(i, KUSH_META(row0, false, i), hf & (FULL - 1));
            inflight |= 1u << (i % C::NS);
        }
    }
    for (int i = 0; i < n_local && ok; i++) {
        if (i % WARP == 0 && i) {
            cur = nxt;
            nxt = load_meta(i / WARP + 1);
        }
        const int ia = i + C::NS - 1;                                // the item whose rows start now
        if (ia < n_local) {
            const bool nb = ia / WARP != i / WARP;
            const int hfa = KUSH_META(hf, nb, ia % WARP);
            if (hfa & FULL) {
                issue(ia, KUSH_META(row0, nb, ia % WARP), hfa & (FULL - 1));
                inflight |= 1u << (ia % C::NS);
            }
        }
        const int l = i % WARP;
        const int hf = KUSH_META(hf, false, l), blk = KUSH_META(blk, false, l);
        const int h = hf & (FULL - 1), slot = i % C::NS;
        if (hf & FULL) {
            ok = __all_sync(0xffffffffu, mbar_wait_u32(bar0 + 8u * slot, (phase >> slot) & 1u));
            if (ok) {
                phase ^= 1u << slot;
                inflight &= ~(1u << slot);
                ws_item<D, BITS, P, IN>(slots + slot * C::STAGE, rec_at(cache, blk, h, block_stride, head_stride),
                                        lane, role);
            }
        } else if (role == 0 && !(hf & SKIP)) {
            general(i, l, h, blk);
        }
        __syncwarp();
    }
    if (!ok) {
        // a copy never completed: record it, wait (bounded) for this warp's copies still in flight, stop
        if (lane == 0) atomicExch(&g_write_error, 1);
#pragma unroll
        for (int sl = 0; sl < C::NS; sl++)
            if (inflight >> sl & 1u) mbar_wait_u32(bar0 + 8u * sl, (phase >> sl) & 1u);
    }
#undef KUSH_META
}

template <int D, int BITS, int P, class IN>
int launch_append(const void* k_new, const void* v_new, int64_t k_stride, int64_t v_stride, int32_t* seq_lens,
                  int32_t pos_offset, int32_t advance, const int32_t* tail_idx, void* cache, int64_t block_stride,
                  int64_t head_stride, void* tail_k, const int32_t* block_table, int64_t max_pages, int32_t hkv,
                  int32_t n_seqs, int rot, cudaStream_t stream) {
    launch_pdl(append_kernel<D, BITS, P, IN>, dim3(n_seqs), dim3(D), 0, stream, static_cast<const IN*>(k_new),
               static_cast<const IN*>(v_new), k_stride, v_stride, seq_lens, pos_offset, advance, tail_idx,
               static_cast<uint8_t*>(cache), block_stride, head_stride, static_cast<IN*>(tail_k), block_table,
               max_pages, hkv, rot);
    return check_launch("kush_sm100_append");
}

// the streaming write: grid = resident CTAs of the device (or fewer when there are fewer items than warps)
template <int D, int BITS, int P, class IN>
int launch_write_stream(const void* k_new, const void* v_new, int64_t k_stride, int64_t v_stride, const int32_t* qsl,
                        const int32_t* seq_lens, const int32_t* tail_idx, const int32_t* job_seq,
                        const int32_t* job_page, int32_t mode, void* cache, int64_t block_stride, int64_t head_stride,
                        void* tail_k, const int32_t* block_table, int64_t max_pages, int32_t hkv, int32_t n_jobs,
                        int dev, cudaStream_t stream) {
    using C = WS<D, BITS, P, IN>;
    auto kern = write_stream_kernel<D, BITS, P, IN>;
    static std::atomic<int> resident[64];                // per device: CTAs per SM x SMs, 0 until first use
    const int di = dev & 63;
    int slots = resident[di].load(std::memory_order_relaxed);
    if (slots == 0) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        int per_sm = 0, sms = 0;
        if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, C::NW * WARP, C::SMEM);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return set_error(KUSH_ERR_CUDA, "write: kernel setup: %s", cudaGetErrorString(e));
        if (per_sm < 1) return set_error(KUSH_ERR_CUDA, "write: streaming kernel does not fit on an SM");
        slots = per_sm * sms;
        resident[di].store(slots, std::memory_order_relaxed);
    }
    const int64_t want = (int64_t(n_jobs) * hkv + C::NST - 1) / C::NST;
    const int grid = int(want < slots ? want : slots);
    kern<<<grid, C::NW * WARP, C::SMEM, stream>>>(
        static_cast<const IN*>(k_new), static_cast<const IN*>(v_new), k_stride, v_stride, qsl, seq_lens, tail_idx,
        job_seq, job_page, mode, static_cast<uint8_t*>(cache), block_stride, head_stride, static_cast<IN*>(tail_k),
        block_table, max_pages, hkv, n_jobs);
    return check_launch("kush_sm100_write");
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
    if constexpr (sizeof(IN) == 2) {
        if (vin && vout)
            return launch_write_stream<D, BITS, P, IN>(k_new, v_new, k_stride, v_stride, qsl, seq_lens, tail_idx,
                                                       job_seq, job_page, mode, cache, block_stride, head_stride,
                                                       tail_k, block_table, max_pages, hkv, n_jobs, dev, stream);
    }
    const int vec = vin | (vout << 1);
    kern<<<grid, D, smem, stream>>>(
        static_cast<const IN*>(k_new), static_cast<const IN*>(v_new), k_stride, v_stride, qsl, seq_lens, tail_idx,
        job_seq, job_page, mode, static_cast<uint8_t*>(cache), block_stride, head_stride, static_cast<IN*>(tail_k),
        block_table, max_pages, hkv, vec);
    return check_launch("kush_sm100_write");
}

// Exhaustive check of the scale arithmetic of the streaming write against CUDA's IEEE operations: div_levels and
// the packed div_levels2 (every value through both lanes) for every fp32 d in [2^-100, 2^100] (and 0), BITS 4 and
// 8, against __fdiv_rn; rcp_nr for every fp16 bit pattern against `s > 0 ? __frcp_rn(s) : 0`.  Mismatch counts in
// bad[0..2].
__global__ void __launch_bounds__(256) selfcheck_kernel(unsigned long long* bad) {
    const uint32_t lo = 0x0D800000u, hi = 0x71800000u;          // 2^-100 .. 2^100
    unsigned long long b4 = 0, b8 = 0, br = 0;
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t u = lo + blockIdx.x * blockDim.x + threadIdx.x; u <= hi; u += stride) {
        // d in the first lane of the packed form, its neighbour in the other (every value goes through both lanes)
        const float d = __uint_as_float(u), e = __uint_as_float(u > lo ? u - 1 : hi);
        const float q4 = __fdiv_rn(d, 15.0f), q8 = __fdiv_rn(d, 255.0f);
        const float2 p4 = div_levels2<4>(make_float2(d, e)), p8 = div_levels2<8>(make_float2(e, d));
        b4 += (__float_as_uint(div_levels<4>(d)) != __float_as_uint(q4)) + (__float_as_uint(p4.x) != __float_as_uint(q4)) +
              (__float_as_uint(p4.y) != __float_as_uint(__fdiv_rn(e, 15.0f)));
        b8 += (__float_as_uint(div_levels<8>(d)) != __float_as_uint(q8)) + (__float_as_uint(p8.y) != __float_as_uint(q8)) +
              (__float_as_uint(p8.x) != __float_as_uint(__fdiv_rn(e, 255.0f)));
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        b4 += div_levels<4>(0.0f) != 0.0f || div_levels2<4>(make_float2(0.0f, 0.0f)).x != 0.0f;
        b8 += div_levels<8>(0.0f) != 0.0f || div_levels2<8>(make_float2(0.0f, 0.0f)).y != 0.0f;
    }
    for (uint32_t p = blockIdx.x * blockDim.x + threadIdx.x; p < 65536u; p += stride) {
        const float sv = __half2float(__ushort_as_half(uint16_t(p)));
        const float want = sv > 0.0f ? __frcp_rn(sv) : 0.0f;
        br += __float_as_uint(rcp_nr(sv)) != __float_as_uint(want);
    }
    if (b4) atomicAdd(&bad[0], b4);
    if (b8) atomicAdd(&bad[1], b8);
    if (br) atomicAdd(&bad[2], br);
}

int write_error_flag(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_write_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_write_error, &zero, sizeof(int));
    }
    return v;
}

}  // namespace kush

using namespace kush;

static int append_any(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, const void* k_new,
                      const void* v_new, int64_t k_stride, int64_t v_stride, int32_t* seq_lens, int32_t pos_offset,
                      int32_t advance, const int32_t* tail_idx, void* cache, int64_t block_stride, int64_t head_stride,
                      void* tail_k, const int32_t* block_table, int64_t max_pages, int32_t hkv, int32_t n_seqs, int rot,
                      void* stream, const char* name) {
    if (n_seqs < 0 || hkv < 1) return set_error(KUSH_ERR_ARG, "%s: n_seqs %d, hkv %d", name, n_seqs, hkv);
    if (n_seqs == 0) return KUSH_OK;
    if (!k_new || !v_new || !seq_lens || !tail_idx || !cache || !tail_k || !block_table)
        return set_error(KUSH_ERR_ARG, "%s: null pointer", name);
    int rc = dispatch_fmt(head_dim, bits, page, dtype, [&](auto D, auto B, auto P, auto in) {
        return launch_append<D.value, B.value, P.value, decltype(in)>(
            k_new, v_new, k_stride, v_stride, seq_lens, pos_offset, advance, tail_idx, cache, block_stride, head_stride,
            tail_k, block_table, max_pages, hkv, n_seqs, rot, static_cast<cudaStream_t>(stream));
    });
    if (rc == KUSH_ERR_UNSUPPORTED)
        return set_error(rc, "%s: unsupported head_dim %d / bits %d / page %d / dtype %d", name, head_dim, bits, page,
                         dtype);
    return rc;
}

extern "C" int kush_sm100_append(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, const void* k_new,
                                 const void* v_new, int64_t k_stride, int64_t v_stride, int32_t* seq_lens,
                                 int32_t pos_offset, int32_t advance, const int32_t* tail_idx, void* cache,
                                 int64_t block_stride, int64_t head_stride, void* tail_k, const int32_t* block_table,
                                 int64_t max_pages, int32_t hkv, int32_t n_seqs, void* stream) {
    return append_any(head_dim, bits, page, dtype, k_new, v_new, k_stride, v_stride, seq_lens, pos_offset, advance,
                      tail_idx, cache, block_stride, head_stride, tail_k, block_table, max_pages, hkv, n_seqs, 0, stream,
                      "kush_sm100_append");
}

extern "C" int kush_sm100_append_rotated(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype,
                                         const void* k_new, const void* v_new, int64_t k_stride, int64_t v_stride,
                                         int32_t* seq_lens, int32_t pos_offset, int32_t advance,
                                         const int32_t* tail_idx, void* cache, int64_t block_stride,
                                         int64_t head_stride, void* tail_k, const int32_t* block_table,
                                         int64_t max_pages, int32_t hkv, int32_t n_seqs, void* stream) {
    return append_any(head_dim, bits, page, dtype, k_new, v_new, k_stride, v_stride, seq_lens, pos_offset, advance,
                      tail_idx, cache, block_stride, head_stride, tail_k, block_table, max_pages, hkv, n_seqs, 1, stream,
                      "kush_sm100_append_rotated");
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

extern "C" int kush_sm100_selfcheck(uint64_t* mismatches) {
    if (!mismatches) return set_error(KUSH_ERR_ARG, "kush_sm100_selfcheck: null pointer");
    unsigned long long* d = nullptr;
    cudaError_t e = cudaMalloc(&d, 3 * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(d, 0, 3 * sizeof(unsigned long long));
    if (e == cudaSuccess) {
        int sms = 0;
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        selfcheck_kernel<<<(sms > 0 ? sms : 1) * 8, 256>>>(d);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(mismatches, d, 3 * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    if (d) cudaFree(d);
    if (e != cudaSuccess) return set_error(KUSH_ERR_CUDA, "kush_sm100_selfcheck: %s", cudaGetErrorString(e));
    return KUSH_OK;
}
