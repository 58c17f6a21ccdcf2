// Shared definitions of the sm_100a kushkash kernels: the page-record format, the bit-exact quantizer arithmetic,
// dtype helpers, template dispatch and the C-ABI error plumbing.
//
// Page record of one (page, kv head), P tokens, D channels, BITS in {4, 8} (kushkash/kush/quant.mojo:53-87):
//   [ kq: P*DC int8 | vq: P*DC int8 | ks: D fp16 | kb: D fp16 | vs: P fp16 | vb: P fp16 ],  DC = D (int8) or D/2
//   x ~= s * c + b, c in [-2^(BITS-1), 2^(BITS-1) - 1]; K: (s, b) per channel over the page, V: per token.
//   int4 byte j of a row = code of dim j (low nibble) | code of dim j + D/2 (high nibble).
// Record of (block b, kv head h) at cache + b*block_stride + h*head_stride (byte strides).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>
#include <utility>

#include "../../include/kushkash_b200.h"

namespace kush {

constexpr int WARP = 32;

template <int D, int BITS, int P>
struct Fmt {
    static_assert(D == 64 || D == 128 || D == 256, "head_dim must be 64, 128 or 256");
    static_assert(BITS == 4 || BITS == 8, "bits must be 4 or 8");
    static_assert(P == 16 || P == 32, "page must be 16 or 32 tokens");
    static constexpr int DC = BITS == 8 ? D : D / 2;          // bytes per token row
    static constexpr int OFF_VQ = P * DC;
    static constexpr int OFF_KS = 2 * P * DC;
    static constexpr int OFF_KB = OFF_KS + 2 * D;
    static constexpr int OFF_VS = OFF_KS + 4 * D;
    static constexpr int OFF_VB = OFF_VS + 2 * P;
    static constexpr int RB = 2 * P * DC + 4 * D + 4 * P;      // record bytes (a multiple of 16 for D % 64 == 0)
    static constexpr int HALF = 1 << (BITS - 1);
};

// ------------------------------------------------------------------ dtypes
template <class T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <class T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float h_load(const uint8_t* p, int i) {
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ void h_store(uint8_t* p, int i, float v) { reinterpret_cast<__half*>(p)[i] = __float2half_rn(v); }

// ------------------------------------------------------------------ quantizer (quant.mojo:25-50), bit-exact
// Every operation is an explicitly rounded intrinsic so that no contraction can change a rounding: the pages must
// equal the reference's byte for byte.
template <int BITS>
__device__ __forceinline__ void qparams(float mn, float mx, float& s, float& b, float& inv) {
    constexpr float LEVELS = float((1 << BITS) - 1);
    constexpr float HALFF = float(1 << (BITS - 1));
    s = __half2float(__float2half_rn(__fdiv_rn(__fsub_rn(mx, mn), LEVELS)));
    b = __half2float(__float2half_rn(__fadd_rn(mn, __fmul_rn(s, HALFF))));
    inv = s > 0.0f ? __fdiv_rn(1.0f, s) : 0.0f;
}

// round((x - b) * inv) with ties to even (torch.round, as the reference's tests pin), clamped to the code range.
// The rounding is one fp32 add of 1.5 * 2^23: for |y| < 2^22 the sum's ulp is 1, so IEEE round-to-nearest-even of
// the add is round-half-even of y, and the integer sits in the low mantissa bits (no float->int conversion op).
// Larger |y| (only reachable if the inputs are not finite) saturate like the clamp.
template <int BITS>
__device__ __forceinline__ int qcode(float x, float b, float inv) {
    constexpr int HALF = 1 << (BITS - 1);
    const float y = __fmul_rn(__fsub_rn(x, b), inv);
    const float yc = fminf(fmaxf(y, -4194304.0f), 4194304.0f);
    const int r = __float_as_int(__fadd_rn(yc, 12582912.0f)) - 0x4B400000;
    return min(max(r, -HALF), HALF - 1);
}

__device__ __forceinline__ uint8_t pack4(int lo, int hi) { return uint8_t((lo & 0x0F) | ((hi & 0x0F) << 4)); }

// code of dim c of one token row, as an int (int4: dim c < D/2 is the low nibble of byte c, else the high nibble of
// byte c - D/2; two's complement)
template <int D, int BITS>
__device__ __forceinline__ int code_at(const uint8_t* row, int c) {
    if constexpr (BITS == 8) {
        return int(int8_t(row[c]));
    } else {
        int b = int(int8_t(row[c < D / 2 ? c : c - D / 2]));
        return c < D / 2 ? ((b << 28) >> 28) : (b >> 4);
    }
}

// ------------------------------------------------------------------ warp helpers
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
    for (int o = 16; o; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}
__device__ __forceinline__ float warp_min(float x) {
#pragma unroll
    for (int o = 16; o; o >>= 1) x = fminf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// ------------------------------------------------------------------ canonical Walsh-Hadamard rotation of a row
// A row of D values held by one warp, lane l holding y[i] = x[l + 32 i] (i < D/32).  The canonical order
// (kushkash/kush/quant.mojo:90-122): fp32 butterflies over strides 1, 2, ..., D/2 in that order -- strides < 32 pair
// lanes (shuffle xor), strides >= 32 pair a lane's own registers -- then one separately rounded multiply by fp32
// 1/sqrt(D).  Adds, subtracts and the multiply are correctly rounded IEEE operations in a fixed order, so the result
// equals the CPU's bit for bit.
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

// ------------------------------------------------------------------ split-KV page ranges
// The reference gives split z of a sequence with `full` full pages the range [z q, (z+1) q), q = ceil(full /
// n_splits) (kushkash/kush/gpu.mojo:418-424): every sequence in n_splits pieces, however short.  Here the quota is
// one for the batch, q = ceil(max_full / n_splits) over the batch's sequences: a short sequence fills only its first
// ceil(full / q) splits and its other splits have nothing to do (they only mark their partials empty), so the
// splits go to the long sequences of a ragged batch and no CTA is left with a page or two.  With equal lengths the
// ranges are the reference's.  The tail page belongs to the last split with pages (split 0 when there are none).
// Every warp of a CTA computes the same range (the max is a warp reduction over seq_lens).
struct SplitRange {
    int64_t p0, p1;      // full pages [p0, p1)
    bool active;         // this split has pages, or is split 0
    bool last;           // this split takes the tail page
};

__device__ __forceinline__ SplitRange split_range(const int32_t* seq_lens, int n_seqs, int s, int z, int n_splits,
                                                  int P) {
    const uint32_t full = uint32_t(seq_lens[s]) / uint32_t(P);
    if (n_splits == 1) return {0, int64_t(full), true, true};
    uint32_t mx = 0;
    for (int i = threadIdx.x % WARP; i < n_seqs; i += WARP) mx = max(mx, uint32_t(seq_lens[i]));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const uint32_t q = max(1u, (mx / uint32_t(P) + uint32_t(n_splits) - 1) / uint32_t(n_splits));   // pages per split
    const uint32_t p0 = min(full, uint32_t(z) * q), p1 = min(full, p0 + q);
    const bool active = z == 0 || p0 < full;
    return {int64_t(p0), int64_t(p1), active, active && p1 == full};
}

// ------------------------------------------------------------------ split-KV merge
// The combine of one (sequence, kv head, q head) at output dim d (kushkash/kush/gpu.mojo:469-491): ml points at the
// first split's (m, l) (natural-log max, sum; split z at ml[2 z G]), po at the first split's unnormalised output
// for dim d (split z at po[z G D]).  Splits with m = -inf are empty and skipped.  Returns o / L (0 when L = 0).
// CG: read through L2 only (partials that other CTAs of the same launch have just stored).
template <bool CG = false>
__device__ __forceinline__ float merge_splits(const float* __restrict__ ml, const float* __restrict__ po, int n_splits,
                                              int G, int D) {
    auto ld = [](const float* p) { return CG ? __ldcg(p) : *p; };
    float M = -INFINITY;
    for (int z = 0; z < n_splits; z++) M = fmaxf(M, ld(ml + 2 * int64_t(z) * G));
    float L = 0.0f, o = 0.0f;
    for (int z = 0; z < n_splits; z++) {
        const float mz = ld(ml + 2 * int64_t(z) * G);
        if (mz > -INFINITY) {
            const float f = __expf(mz - M);
            L = fmaf(ld(ml + 2 * int64_t(z) * G + 1), f, L);
            o = fmaf(f, ld(po + int64_t(z) * G * D), o);
        }
    }
    return L > 0.0f ? o / L : 0.0f;
}

// ------------------------------------------------------------------ programmatic dependent launch
// The decode-step kernels are launched with programmatic stream serialization (launch_pdl): the next kernel on the
// stream may be launched as the blocks of the running one exit, and it runs pdl_wait() -- which returns when the
// previous grid has completed and its memory is visible -- before it touches memory.  Every kernel launched this way
// starts with pdl_wait(), so the stream order of memory effects is kept; what overlaps is the launch and the block
// dispatch.  Two kernels trigger their dependent early (pdl_trigger() right after their wait, so the next launch's
// blocks are placed while they run and wait in pdl_wait()): the append (the decode after it launches while the short
// append runs: config 2 -5%, config 5 -0.4 to -1.2%, config 4 -0.5%, configs 1 and 3 unchanged) and the decode
// without splits (the next layer's kernels launch behind its last wave: config 5 -2.3%, config 3 -0.2%).  In every
// kernel at block start, the split decodes included, the trigger made config 4's step 2% and config 1's 4% slower,
// the waiting blocks resident beside the issue-bound decode; in the split combine it measured neutral.  Without the
// launch attribute pdl_wait() and pdl_trigger() are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------ host-side dispatch
template <int V> using IC = std::integral_constant<int, V>;

template <class F> int dispatch_page(int page, F&& f) {
    switch (page) {
        case 16: return f(IC<16>{});
        case 32: return f(IC<32>{});
        default: return KUSH_ERR_UNSUPPORTED;
    }
}
template <class F> int dispatch_bits(int bits, F&& f) {
    switch (bits) {
        case 4: return f(IC<4>{});
        case 8: return f(IC<8>{});
        default: return KUSH_ERR_UNSUPPORTED;
    }
}
template <class F> int dispatch_dim(int d, F&& f) {
    switch (d) {
        case 64: return f(IC<64>{});
        case 128: return f(IC<128>{});
        case 256: return f(IC<256>{});
        default: return KUSH_ERR_UNSUPPORTED;
    }
}
template <class F> int dispatch_dtype(int dtype, F&& f) {
    switch (dtype) {
        case KUSH_F16: return f(__half{});
        case KUSH_BF16: return f(__nv_bfloat16{});
        case KUSH_F32: return f(float{});
        default: return KUSH_ERR_UNSUPPORTED;
    }
}
// (head_dim, bits, page, dtype) -> f(IC<D>, IC<BITS>, IC<P>, IN{})
template <class F> int dispatch_fmt(int d, int bits, int page, int dtype, F&& f) {
    return dispatch_dim(d, [&](auto D) {
        return dispatch_bits(bits, [&](auto B) {
            return dispatch_page(page, [&](auto P) { return dispatch_dtype(dtype, [&](auto in) { return f(D, B, P, in); }); });
        });
    });
}

// records the message of the last failed call on this host thread; returns the status to hand back
int set_error(int status, const char* fmt, ...);
// checks the launch that just happened (cudaGetLastError); KUSH_OK or KUSH_ERR_CUDA with the message recorded
int check_launch(const char* what);

// the streaming write's bounded-wait flag (1 if a wait gave up), optionally cleared; -1 on a CUDA error
int write_error_flag(int clear);
int gather_error_flag(int clear);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace kush
