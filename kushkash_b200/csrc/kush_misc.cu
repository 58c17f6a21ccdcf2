// Canonical Walsh-Hadamard rotation (fwht_warp, kush_common.cuh) of rows and the packed-prefill unpack, both
// bit-identical to the CPU restatement.
#include "kush_async.cuh"
#include "kush_common.cuh"

namespace kush {

// grid (ceil(rows / 4)), block 128: one warp per row; y may alias x (kushkash/kush/gpu.mojo:95-112 kush_fwht)
template <int D, class IN>
__global__ void __launch_bounds__(128) fwht_kernel(const IN* x, IN* y, int64_t xs, int64_t ys, int64_t rows) {
    constexpr int R = D / WARP;
    const int lane = threadIdx.x % WARP;
    const int64_t r = int64_t(blockIdx.x) * 4 + threadIdx.x / WARP;
    if (r >= rows) return;
    float v[R];
#pragma unroll
    for (int i = 0; i < R; i++) v[i] = to_f32(x[r * xs + lane + WARP * i]);
    fwht_warp<D>(v, lane);
#pragma unroll
    for (int i = 0; i < R; i++) y[r * ys + lane + WARP * i] = from_f32<IN>(v[i]);
}

// grid (n_pages + n_tail + ceil(n_new / 32), Hkv), block 128 (kushkash/kush/gpu.mojo:303-375 kush_unpack).
// Block x < n_pages: history page; < n_pages + n_tail: partial page; else 32 rows of the new chunk.  Element-wise
// loads and stores: the form for records, tail slots or outputs that are not 16-byte aligned (unpack_vec_kernel
// below takes every aligned call).
template <int D, int BITS, int P, class IN>
__global__ void __launch_bounds__(128) unpack_kernel(const uint8_t* __restrict__ cache, int64_t block_stride,
                                                     int64_t head_stride, int H, const int32_t* __restrict__ page_blk,
                                                     const int32_t* __restrict__ page_dst, int n_pages,
                                                     const int32_t* __restrict__ tail_blk,
                                                     const int32_t* __restrict__ tail_info, int n_tail,
                                                     const IN* __restrict__ tail_k, const IN* __restrict__ k_new,
                                                     const IN* __restrict__ v_new, int64_t ks, int64_t vs,
                                                     const int32_t* __restrict__ new_dst, int n_new,
                                                     IN* __restrict__ kp, IN* __restrict__ vp, int rot) {
    using F = Fmt<D, BITS, P>;
    constexpr int R = D / WARP;
    const int b = blockIdx.x, h = blockIdx.y, w = threadIdx.x / WARP, lane = threadIdx.x % WARP;
    const int64_t rs = int64_t(H) * D;
    if (b < n_pages + n_tail) {
        const bool page = b < n_pages;
        const int i = b - n_pages;
        const int32_t blk = page ? page_blk[b] : tail_blk[i];
        if (blk < 0) return;                                   // a padding entry (kush_sm100_unpack_plan)
        const uint8_t* rec = cache + int64_t(blk) * block_stride + int64_t(h) * head_stride;
        const int64_t dst0 = page ? page_dst[b] : tail_info[3 * i];
        const int n = page ? P : tail_info[3 * i + 1];
        float ksv[R], kbv[R];
        if (page) {
#pragma unroll
            for (int j = 0; j < R; j++) {
                ksv[j] = h_load(rec + F::OFF_KS, lane + WARP * j);
                kbv[j] = h_load(rec + F::OFF_KB, lane + WARP * j);
            }
        }
        const IN* tk = page ? nullptr : tail_k + (int64_t(tail_info[3 * i + 2]) * H + h) * P * D;
        for (int t = w; t < n; t += 4) {
            float kx[R], vx[R];
            const float vsc = h_load(rec + F::OFF_VS, t), vbi = h_load(rec + F::OFF_VB, t);
#pragma unroll
            for (int j = 0; j < R; j++) {
                const int d = lane + WARP * j;
                kx[j] = page ? __fmaf_rn(float(code_at<D, BITS>(rec + t * F::DC, d)), ksv[j], kbv[j]) : to_f32(tk[t * D + d]);
                vx[j] = __fmaf_rn(float(code_at<D, BITS>(rec + F::OFF_VQ + t * F::DC, d)), vsc, vbi);
            }
            if (rot) {
                fwht_warp<D>(kx, lane);
                fwht_warp<D>(vx, lane);
            }
            const int64_t o = (dst0 + t) * rs + int64_t(h) * D;
#pragma unroll
            for (int j = 0; j < R; j++) {
                kp[o + lane + WARP * j] = from_f32<IN>(kx[j]);
                vp[o + lane + WARP * j] = from_f32<IN>(vx[j]);
            }
        }
    } else {
        const int j0 = (b - n_pages - n_tail) * 32;
        for (int t = w; t < 32; t += 4) {
            const int j = j0 + t;
            if (j < n_new && new_dst[j] >= 0) {
                const int64_t o = int64_t(new_dst[j]) * rs + int64_t(h) * D;
#pragma unroll
                for (int c = 0; c < R; c++) {
                    kp[o + lane + WARP * c] = k_new[j * ks + int64_t(h) * D + lane + WARP * c];
                    vp[o + lane + WARP * c] = v_new[j * vs + int64_t(h) * D + lane + WARP * c];
                }
            }
        }
    }
}

// ------------------------------------------------------------------ vectorised unpack
// Both reference callers launch the unrotated form (rot=False: kushkash/vllm/backend.py:848,
// kushkash/sglang/backend.py:376); the rotate-back runs on the same layout (fwht_chunk).  One warp per item: a
// (history page, kv head), a (partial page, kv head) or one new row (all kv heads).  Codes are read 8 bytes at a time
// (a chunk: 8 channels for int8; 8 + 8 for int4, byte j holding channel j in its low nibble and channel j + D/2 in its
// high one), dequantized as fma(code, scale, bias) in fp32, rounded once and written with 16-byte stores.  Chunk c
// of a page is token c / NG, bytes 8 (c % NG) .. + 7 (NG = row bytes / 8, which divides 32); lane l takes chunks
// l, l + 32, ..., so its channels -- and its K scales -- stay fixed over the page.
//
// Codes to fp32 without a conversion instruction: a byte u placed under the exponent of 2^23 (PRMT with 0x4B000000)
// is the float 2^23 + u, and subtracting 2^23 + OFFS gives u - OFFS exactly.  The stored codes are two's complement;
// u = code + OFFS is the byte (int8, OFFS 128) or nibble (int4, OFFS 8) with its top bit flipped.

constexpr uint32_t MAGIC_BITS = 0x4B000000u;   // 2^23

template <int OFFS>
__device__ __forceinline__ void deq8(uint32_t u0, uint32_t u1, const float (&s)[8], const float (&b)[8], float (&o)[8]) {
    constexpr float M = 8388608.0f + float(OFFS);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        o[k] = __fmaf_rn(__fsub_rn(__uint_as_float(prmt(u0, MAGIC_BITS, 0x7540u + k)), M), s[k], b[k]);
        o[k + 4] = __fmaf_rn(__fsub_rn(__uint_as_float(prmt(u1, MAGIC_BITS, 0x7540u + k)), M), s[k + 4], b[k + 4]);
    }
}

template <class IN>
__device__ __forceinline__ void store8(IN* dst, const float (&v)[8]) {
    if constexpr (std::is_same_v<IN, float>) {
        reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if constexpr (std::is_same_v<IN, __nv_bfloat16>) {
                const __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
                w[k] = *reinterpret_cast<const uint32_t*>(&p);
            } else {
                const __half2 p = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
                w[k] = *reinterpret_cast<const uint32_t*>(&p);
            }
        }
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__device__ __forceinline__ void halves8(const uint8_t* p, float (&f)[8]) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
        f[2 * k] = x.x;
        f[2 * k + 1] = x.y;
    }
}

// one chunk of codes (8 bytes) of token row `row` into out (channels 8g.. [+ D/2 + 8g..] of the output row)
template <int D, int BITS, class IN>
__device__ __forceinline__ void chunk_out(uint2 w, const float (&s0)[8], const float (&b0)[8], const float (&s1)[8],
                                          const float (&b1)[8], IN* out) {
    float o[8];
    if constexpr (BITS == 4) {
        deq8<8>((w.x & 0x0F0F0F0Fu) ^ 0x08080808u, (w.y & 0x0F0F0F0Fu) ^ 0x08080808u, s0, b0, o);
        store8<IN>(out, o);
        deq8<8>(((w.x >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, ((w.y >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, s1, b1, o);
        store8<IN>(out + D / 2, o);
    } else {
        deq8<128>(w.x ^ 0x80808080u, w.y ^ 0x80808080u, s0, b0, o);
        store8<IN>(out, o);
    }
}

// tokens [0, n) of the record at rec into rows kout + t * rs, vout + t * rs; K from tk ([P, D], n < P) when given
template <int D, int BITS, int P, class IN>
__device__ __forceinline__ void unpack_page_vec(const uint8_t* __restrict__ rec, const IN* __restrict__ tk, int n,
                                                IN* __restrict__ kout, IN* __restrict__ vout, int64_t rs, int lane) {
    using F = Fmt<D, BITS, P>;
    constexpr int NG = F::DC / 8, TPW = WARP / NG, PASSES = P / TPW;
    static_assert(WARP % NG == 0 && P % TPW == 0, "chunk mapping");
    const int g = lane % NG, t0 = lane / NG;
    const int c0 = 8 * g;                                           // first output channel of this lane's chunks
    if (tk == nullptr) {
        float s0[8], b0[8], s1[8], b1[8];
        halves8(rec + F::OFF_KS + 2 * c0, s0);
        halves8(rec + F::OFF_KB + 2 * c0, b0);
        if constexpr (BITS == 4) {
            halves8(rec + F::OFF_KS + 2 * (c0 + D / 2), s1);
            halves8(rec + F::OFF_KB + 2 * (c0 + D / 2), b1);
        }
        uint2 w[PASSES];
#pragma unroll
        for (int i = 0; i < PASSES; i++)
            w[i] = __ldg(reinterpret_cast<const uint2*>(rec + (t0 + TPW * i) * F::DC + c0));
#pragma unroll
        for (int i = 0; i < PASSES; i++) chunk_out<D, BITS, IN>(w[i], s0, b0, s1, b1, kout + (t0 + TPW * i) * rs + c0);
    } else {
        constexpr int E = 16 / int(sizeof(IN)), CPR = D / E;      // elements per 16 bytes, 16-byte chunks per row
        for (int c = lane; c < n * CPR; c += WARP) {
            const int t = c / CPR, q = c % CPR;
            *reinterpret_cast<uint4*>(kout + t * rs + q * E) = __ldg(reinterpret_cast<const uint4*>(tk + t * D + q * E));
        }
    }
    uint2 w[PASSES];
    float vs[PASSES], vb[PASSES];
#pragma unroll
    for (int i = 0; i < PASSES; i++) {
        const int t = t0 + TPW * i;
        if (t < n) {
            w[i] = __ldg(reinterpret_cast<const uint2*>(rec + F::OFF_VQ + t * F::DC + c0));
            vs[i] = h_load(rec + F::OFF_VS, t);
            vb[i] = h_load(rec + F::OFF_VB, t);
        }
    }
#pragma unroll
    for (int i = 0; i < PASSES; i++) {
        const int t = t0 + TPW * i;
        if (t < n) {
            float s[8], b[8];
#pragma unroll
            for (int k = 0; k < 8; k++) s[k] = vs[i], b[k] = vb[i];
            chunk_out<D, BITS, IN>(w[i], s, b, s, b, vout + t * rs + c0);
        }
    }
}

// Rotate-back on the chunk layout.  A token row is held by the NG lanes of one group; a lane holds channels
// c0..c0+7 in lo and, for int4, D/2+c0..D/2+c0+7 in hi (c0 = 8 (lane % NG)).  The canonical butterflies, strides 1, 2,
// ..., D/2 in that order: strides 1-4 inside lo / hi, strides 8 .. (the lanes' span) / 2 between lanes (shuffle xor
// stride / 8), and for int4 stride D/2 between lo and hi; then the separately rounded multiply by fp32 1/sqrt(D).
// Every value goes through the same correctly rounded operations as in fwht_warp, so the results are identical.
template <int D, int BITS>
__device__ __forceinline__ void fwht_chunk(float (&lo)[8], float (&hi)[8], int g) {
    constexpr int NG = (BITS == 8 ? D : D / 2) / 8;
    auto inreg = [](float (&y)[8]) {
#pragma unroll
        for (int h = 1; h < 8; h <<= 1)
#pragma unroll
            for (int k = 0; k < 8; k++)
                if (!(k & h)) {
                    const float a = y[k], b = y[k + h];
                    y[k] = __fadd_rn(a, b);
                    y[k + h] = __fsub_rn(a, b);
                }
    };
    inreg(lo);
    if constexpr (BITS == 4) inreg(hi);
#pragma unroll
    for (int m = 1; m < NG; m <<= 1) {
        const bool upper = g & m;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const float o = __shfl_xor_sync(0xffffffffu, lo[k], m);
            lo[k] = upper ? __fsub_rn(o, lo[k]) : __fadd_rn(lo[k], o);
            if constexpr (BITS == 4) {
                const float oh = __shfl_xor_sync(0xffffffffu, hi[k], m);
                hi[k] = upper ? __fsub_rn(oh, hi[k]) : __fadd_rn(hi[k], oh);
            }
        }
    }
    if constexpr (BITS == 4) {
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const float a = lo[k], b = hi[k];
            lo[k] = __fadd_rn(a, b);
            hi[k] = __fsub_rn(a, b);
        }
    }
    const float sc = D == 64 ? __uint_as_float(0x3E000000u) : D == 128 ? __uint_as_float(0x3DB504F3u)
                                                                        : __uint_as_float(0x3D800000u);
#pragma unroll
    for (int k = 0; k < 8; k++) {
        lo[k] = __fmul_rn(lo[k], sc);
        hi[k] = __fmul_rn(hi[k], sc);
    }
}

template <int BITS>
__device__ __forceinline__ void chunk_vals(uint2 w, const float (&s0)[8], const float (&b0)[8], const float (&s1)[8],
                                           const float (&b1)[8], float (&lo)[8], float (&hi)[8]) {
    if constexpr (BITS == 4) {
        deq8<8>((w.x & 0x0F0F0F0Fu) ^ 0x08080808u, (w.y & 0x0F0F0F0Fu) ^ 0x08080808u, s0, b0, lo);
        deq8<8>(((w.x >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, ((w.y >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, s1, b1, hi);
    } else {
        deq8<128>(w.x ^ 0x80808080u, w.y ^ 0x80808080u, s0, b0, lo);
#pragma unroll
        for (int k = 0; k < 8; k++) hi[k] = 0.0f;
    }
}

template <class IN>
__device__ __forceinline__ void load8(const IN* p, float (&f)[8]) {
#pragma unroll
    for (int k = 0; k < 8; k++) f[k] = to_f32(p[k]);
}

// unpack_page_vec with the rotate-back: every lane computes all P rows (rows n.. of a partial page are in bounds
// and keep the shuffles convergent) and stores rows < n
template <int D, int BITS, int P, class IN>
__device__ __forceinline__ void unpack_page_vec_rot(const uint8_t* __restrict__ rec, const IN* __restrict__ tk, int n,
                                                    IN* __restrict__ kout, IN* __restrict__ vout, int64_t rs,
                                                    int lane) {
    using F = Fmt<D, BITS, P>;
    constexpr int NG = F::DC / 8, TPW = WARP / NG, PASSES = P / TPW;
    const int g = lane % NG, t0 = lane / NG, c0 = 8 * g;
    float s0[8], b0[8], s1[8], b1[8];
    if (tk == nullptr) {
        halves8(rec + F::OFF_KS + 2 * c0, s0);
        halves8(rec + F::OFF_KB + 2 * c0, b0);
        if constexpr (BITS == 4) {
            halves8(rec + F::OFF_KS + 2 * (c0 + D / 2), s1);
            halves8(rec + F::OFF_KB + 2 * (c0 + D / 2), b1);
        }
    }
#pragma unroll 1
    for (int i = 0; i < PASSES; i++) {
        const int t = t0 + TPW * i;
        float lo[8], hi[8];
        if (tk == nullptr) {
            chunk_vals<BITS>(__ldg(reinterpret_cast<const uint2*>(rec + t * F::DC + c0)), s0, b0, s1, b1, lo, hi);
        } else {
            load8(tk + t * D + c0, lo);
            if constexpr (BITS == 4) load8(tk + t * D + D / 2 + c0, hi);
            else
#pragma unroll
                for (int k = 0; k < 8; k++) hi[k] = 0.0f;
        }
        fwht_chunk<D, BITS>(lo, hi, g);
        if (t < n) {
            store8<IN>(kout + t * rs + c0, lo);
            if constexpr (BITS == 4) store8<IN>(kout + t * rs + D / 2 + c0, hi);
        }
    }
#pragma unroll 1
    for (int i = 0; i < PASSES; i++) {
        const int t = t0 + TPW * i;
        float s[8], b[8], lo[8], hi[8];
        const float vsc = h_load(rec + F::OFF_VS, t), vbi = h_load(rec + F::OFF_VB, t);
#pragma unroll
        for (int k = 0; k < 8; k++) s[k] = vsc, b[k] = vbi;
        chunk_vals<BITS>(__ldg(reinterpret_cast<const uint2*>(rec + F::OFF_VQ + t * F::DC + c0)), s, b, s, b, lo, hi);
        fwht_chunk<D, BITS>(lo, hi, g);
        if (t < n) {
            store8<IN>(vout + t * rs + c0, lo);
            if constexpr (BITS == 4) store8<IN>(vout + t * rs + D / 2 + c0, hi);
        }
    }
}

// grid (ceil(warps / 8)), block 256; warps = (n_pages + n_tail) * H + n_new.  Records, tail_k, kp and vp 16-byte
// aligned (the host checks); vec_new: k_new / v_new rows 16-byte aligned, else the new rows are copied by element.
template <int D, int BITS, int P, class IN>
__global__ void __launch_bounds__(256) unpack_vec_kernel(
    const uint8_t* __restrict__ cache, int64_t block_stride, int64_t head_stride, int H,
    const int32_t* __restrict__ page_blk, const int32_t* __restrict__ page_dst, int n_pages,
    const int32_t* __restrict__ tail_blk, const int32_t* __restrict__ tail_info, int n_tail,
    const IN* __restrict__ tail_k, const IN* __restrict__ k_new, const IN* __restrict__ v_new, int64_t ks, int64_t vs,
    const int32_t* __restrict__ new_dst, int n_new, IN* __restrict__ kp, IN* __restrict__ vp, int vec_new, int rot) {
    const int lane = threadIdx.x % WARP;
    const int64_t wi = int64_t(blockIdx.x) * (blockDim.x / WARP) + threadIdx.x / WARP;
    const int64_t rs = int64_t(H) * D;
    const int64_t n_pw = int64_t(n_pages) * H, n_tw = int64_t(n_tail) * H;
    if (wi < n_pw + n_tw) {
        const bool page = wi < n_pw;
        const int64_t it = page ? wi : wi - n_pw;
        const int i = int(it / H), h = int(it % H);
        const int32_t blk = page ? page_blk[i] : tail_blk[i];
        if (blk < 0) return;                                   // a padding entry (kush_sm100_unpack_plan)
        const uint8_t* rec = cache + int64_t(blk) * block_stride + int64_t(h) * head_stride;
        const int64_t dst0 = page ? page_dst[i] : tail_info[3 * i];
        const int n = page ? P : tail_info[3 * i + 1];
        const IN* tk = page ? nullptr : tail_k + (int64_t(tail_info[3 * i + 2]) * H + h) * P * D;
        IN* kout = kp + dst0 * rs + int64_t(h) * D;
        IN* vout = vp + dst0 * rs + int64_t(h) * D;
        if (rot)
            unpack_page_vec_rot<D, BITS, P, IN>(rec, tk, n, kout, vout, rs, lane);
        else
            unpack_page_vec<D, BITS, P, IN>(rec, tk, n, kout, vout, rs, lane);
    } else if (wi < n_pw + n_tw + n_new) {
        const int64_t j = wi - n_pw - n_tw;
        if (new_dst[j] < 0) return;                            // a padding entry
        const int64_t o = int64_t(new_dst[j]) * rs;
        if (vec_new) {
            constexpr int E = 16 / int(sizeof(IN));
            for (int64_t c = lane; c < rs / E; c += WARP) {
                *reinterpret_cast<uint4*>(kp + o + c * E) = __ldg(reinterpret_cast<const uint4*>(k_new + j * ks + c * E));
                *reinterpret_cast<uint4*>(vp + o + c * E) = __ldg(reinterpret_cast<const uint4*>(v_new + j * vs + c * E));
            }
        } else {
            for (int64_t c = lane; c < rs; c += WARP) {
                kp[o + c] = k_new[j * ks + c];
                vp[o + c] = v_new[j * vs + c];
            }
        }
    }
}

}  // namespace kush

using namespace kush;

extern "C" int kush_sm100_fwht(int32_t head_dim, int32_t dtype, const void* x, void* y, int64_t x_stride,
                               int64_t y_stride, int64_t rows, void* stream) {
    if (rows < 0) return set_error(KUSH_ERR_ARG, "kush_sm100_fwht: rows %lld", (long long)rows);
    if (rows == 0) return KUSH_OK;
    if (!x || !y) return set_error(KUSH_ERR_ARG, "kush_sm100_fwht: null pointer");
    int rc = dispatch_dim(head_dim, [&](auto D) {
        return dispatch_dtype(dtype, [&](auto in) {
            using IN = decltype(in);
            const int64_t blocks = (rows + 3) / 4;
            fwht_kernel<D.value, IN><<<unsigned(blocks), 128, 0, static_cast<cudaStream_t>(stream)>>>(
                static_cast<const IN*>(x), static_cast<IN*>(y), x_stride, y_stride, rows);
            return check_launch("kush_sm100_fwht");
        });
    });
    if (rc == KUSH_ERR_UNSUPPORTED)
        return set_error(rc, "kush_sm100_fwht: unsupported head_dim %d / dtype %d", head_dim, dtype);
    return rc;
}

extern "C" int kush_sm100_unpack(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, const void* cache,
                                 int64_t block_stride, int64_t head_stride, int32_t hkv, const int32_t* page_blk,
                                 const int32_t* page_dst, int32_t n_pages, const int32_t* tail_blk,
                                 const int32_t* tail_info, int32_t n_tail, const void* tail_k, const void* k_new,
                                 const void* v_new, int64_t k_stride, int64_t v_stride, const int32_t* new_dst,
                                 int32_t n_new, void* kp, void* vp, int32_t rot, void* stream) {
    if (n_pages < 0 || n_tail < 0 || n_new < 0 || hkv < 1)
        return set_error(KUSH_ERR_ARG, "kush_sm100_unpack: n_pages %d n_tail %d n_new %d hkv %d", n_pages, n_tail, n_new,
                         hkv);
    const int64_t blocks = int64_t(n_pages) + n_tail + (int64_t(n_new) + 31) / 32;
    if (blocks == 0) return KUSH_OK;
    if (!cache || !kp || !vp) return set_error(KUSH_ERR_ARG, "kush_sm100_unpack: null pointer");
    int rc = dispatch_fmt(head_dim, bits, page, dtype, [&](auto D, auto B, auto P, auto in) {
        using IN = decltype(in);
        const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
        const bool vec = a16(cache) && block_stride % 16 == 0 && head_stride % 16 == 0 && a16(kp) && a16(vp) &&
                         (n_tail == 0 || a16(tail_k));
        if (vec) {
            const int64_t es = int64_t(sizeof(IN));
            const int vec_new = n_new > 0 && a16(k_new) && a16(v_new) && (k_stride * es) % 16 == 0 &&
                                (v_stride * es) % 16 == 0;
            const int64_t warps = (int64_t(n_pages) + n_tail) * hkv + n_new;
            unpack_vec_kernel<D.value, B.value, P.value, IN>
                <<<unsigned((warps + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
                    static_cast<const uint8_t*>(cache), block_stride, head_stride, hkv, page_blk, page_dst, n_pages,
                    tail_blk, tail_info, n_tail, static_cast<const IN*>(tail_k), static_cast<const IN*>(k_new),
                    static_cast<const IN*>(v_new), k_stride, v_stride, new_dst, n_new, static_cast<IN*>(kp),
                    static_cast<IN*>(vp), vec_new, rot);
            return check_launch("kush_sm100_unpack");
        }
        dim3 grid(unsigned(blocks), hkv);
        unpack_kernel<D.value, B.value, P.value, IN><<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const uint8_t*>(cache), block_stride, head_stride, hkv, page_blk, page_dst, n_pages, tail_blk,
            tail_info, n_tail, static_cast<const IN*>(tail_k), static_cast<const IN*>(k_new),
            static_cast<const IN*>(v_new), k_stride, v_stride, new_dst, n_new, static_cast<IN*>(kp),
            static_cast<IN*>(vp), rot);
        return check_launch("kush_sm100_unpack");
    });
    if (rc == KUSH_ERR_UNSUPPORTED)
        return set_error(rc, "kush_sm100_unpack: unsupported head_dim %d / bits %d / page %d / dtype %d", head_dim, bits,
                         page, dtype);
    return rc;
}

// ------------------------------------------------------------------ decode launch order
namespace kush {

constexpr int ORDER_KEYS = 4096;          // full-page counts above ORDER_KEYS - 1 share the top key

// grid 1, block 1024: order[0..S) = the sequences by full pages, most first (a counting sort; ties in any order)
__global__ void __launch_bounds__(1024) order_kernel(const int32_t* __restrict__ seq_lens, int S, int P,
                                                     int32_t* __restrict__ order) {
    pdl_wait();
    __shared__ int cnt[ORDER_KEYS];
    __shared__ int warp_tot[32];
    constexpr int PER = ORDER_KEYS / 1024;                 // keys per thread, thread t: keys from the top down
    const int tid = threadIdx.x, lane = tid % WARP, w = tid / WARP;
    for (int i = tid; i < ORDER_KEYS; i += 1024) cnt[i] = 0;
    __syncthreads();
    auto key = [&](int s) { return min(max(seq_lens[s], 0) / P, ORDER_KEYS - 1); };
    for (int s = tid; s < S; s += 1024) atomicAdd(&cnt[key(s)], 1);
    __syncthreads();
    // start of each key in descending key order: exclusive scan over the keys from ORDER_KEYS - 1 down to 0
    int mine[PER], sum = 0;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        mine[j] = cnt[ORDER_KEYS - 1 - (tid * PER + j)];
        sum += mine[j];
    }
    int incl = sum;                                        // inclusive scan of the per-thread sums
#pragma unroll
    for (int o = 1; o < WARP; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == WARP - 1) warp_tot[w] = incl;
    __syncthreads();
    if (w == 0) {
        int t = warp_tot[lane], ti = t;
#pragma unroll
        for (int o = 1; o < WARP; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, ti, o);
            if (lane >= o) ti += v;
        }
        warp_tot[lane] = ti - t;                           // exclusive prefix of the warp totals
    }
    __syncthreads();
    int run = warp_tot[w] + incl - sum;                    // exclusive prefix of this thread's first key
#pragma unroll
    for (int j = 0; j < PER; j++) {
        cnt[ORDER_KEYS - 1 - (tid * PER + j)] = run;
        run += mine[j];
    }
    __syncthreads();
    for (int s = tid; s < S; s += 1024) order[atomicAdd(&cnt[key(s)], 1)] = s;
}

}  // namespace kush

extern "C" int kush_sm100_order_longest_first(const int32_t* seq_lens, int32_t n_seqs, int32_t page, int32_t* order,
                                              void* stream) {
    if (n_seqs < 0 || page < 1) return set_error(KUSH_ERR_ARG, "kush_sm100_order_longest_first: n_seqs %d page %d",
                                                 n_seqs, page);
    if (n_seqs == 0) return KUSH_OK;
    if (!seq_lens || !order) return set_error(KUSH_ERR_ARG, "kush_sm100_order_longest_first: null pointer");
    launch_pdl(order_kernel, dim3(1), dim3(1024), 0, static_cast<cudaStream_t>(stream), seq_lens, int(n_seqs),
               int(page), order);
    return check_launch("kush_sm100_order_longest_first");
}
