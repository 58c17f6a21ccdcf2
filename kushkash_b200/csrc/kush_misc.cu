// Canonical Walsh-Hadamard rotation and the packed-prefill unpack, both bit-identical to the CPU restatement.
//
// A row of D values is held by one warp, lane l holding x[l + 32 i] (i < D/32).  The canonical order
// (kushkash/kush/quant.mojo:90-122): fp32 butterflies over strides 1, 2, ..., D/2 in that order -- strides < 32
// pair lanes (shuffle xor), strides >= 32 pair a lane's own registers -- then one separately rounded multiply by
// fp32 1/sqrt(D).  Adds, subtracts and the multiply are correctly rounded IEEE operations in a fixed order, so the
// result equals the CPU's bit for bit.
#include "kush_common.cuh"

namespace kush {

template <int D>
__device__ __forceinline__ void fwht_warp(float (&y)[D / WARP], int lane) {
    constexpr int R = D / WARP;
#pragma unroll
    for (int h = 1; h < WARP; h <<= 1) {                    // partner lane ^ h holds x[i ^ h]
        const bool upper = lane & h;
#pragma unroll
        for (int i = 0; i < R; i++) {
            const float other = __shfl_xor_sync(0xffffffffu, y[i], h);
            y[i] = upper ? __fsub_rn(other, y[i]) : __fadd_rn(y[i], other);
        }
    }
#pragma unroll
    for (int hr = 1; hr < R; hr <<= 1) {                    // stride 32 * hr: register bit hr
#pragma unroll
        for (int i = 0; i < R; i++) {
            if (!(i & hr)) {
                const float a = y[i], b = y[i + hr];
                y[i] = __fadd_rn(a, b);
                y[i + hr] = __fsub_rn(a, b);
            }
        }
    }
    const float sc = D == 64 ? __uint_as_float(0x3E000000u) : D == 128 ? __uint_as_float(0x3DB504F3u)
                                                                        : __uint_as_float(0x3D800000u);
#pragma unroll
    for (int i = 0; i < R; i++) y[i] = __fmul_rn(y[i], sc);
}

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
// Block x < n_pages: history page; < n_pages + n_tail: partial page; else 32 rows of the new chunk.
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
        const uint8_t* rec = cache + int64_t(page ? page_blk[b] : tail_blk[i]) * block_stride + int64_t(h) * head_stride;
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
            if (j < n_new) {
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
