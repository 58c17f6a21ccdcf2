// Fused dequant paged decode attention on the tensor cores (sm_100a), for fp16 / bf16 q and outputs.
//
// Same contract as the reference's kush_decode_tc (kushkash/kush/gpu.mojo:566-807); the algebra differs only in
// where the K scale and bias enter (below), the rest -- page-granular online softmax, V scale folded into the
// softmax weights and V bias into one scalar per head, exact-K tail, warp merge, split-KV partials -- is the same.
//
// Work split: grid (S, Hkv, n_splits), 4 warps per CTA.  Split z owns a contiguous page range (split_range: one
// page quota per split for the batch, splits past a sequence's end return at once); warp w takes pages
// start + w, start + w + 4, ...  Each warp streams its pages through its own ring of NS shared-memory slots with
// one 1-D bulk copy per page record (cp.async.bulk, completion on an mbarrier; no multicast), issued NS pages
// ahead by lane 0, with the block-table entries prefetched 32 pages at a time into registers.  All waits are
// bounded: on a timeout the kernel records an error flag, writes NaN outputs and returns.
//
// Per 16-token tile of a page, with m16n8k16 fp16 MMAs (fp32 accumulation):
//   QK:  S^T[16 tok x 8 heads] = K'[16 tok x D] . Qh^T[D x 8 heads]     (tokens on M, heads on N)
//        K' = c * ks + (kb - kb_ref) in fp16 (HFMA2), kb_ref = the K bias of the sequence's first page: the large
//        per-channel offsets cancel before rounding, and the constant q . kb_ref shifts every score of (s, h)
//        equally, which the softmax ignores (the exact-K tail subtracts it too).  Qh = fp16(q * scale * log2 e)
//        is therefore constant for the whole CTA (B fragments loaded once); scores are in log2 units (exp2).
//   PV:  O^T[16 dims x 8 heads] += V^T[16 dims x 16 tok] . P'^T[16 tok x 8 heads], P' = fp16(p * vs_t): the
//        S^T accumulators become P' B fragments with one movmatrix.trans per 8x8 block.
// Codes become exact fp16 with the magic-number trick (a code under the exponent of 1024, then one subtract);
// the D dimension is permuted so every lane's fragments come from whole 32-bit words of its token rows.
#include <cuda.h>
#include <stdio.h>
#include <string.h>

#include "kush_async.cuh"
#include "kush_common.cuh"

namespace kush {

constexpr int MMA_NW = 4;

__device__ int g_decode_error = 0;            // set when a bounded wait gave up (read by kush_sm100_device_error)

// ------------------------------------------------------------------ PTX helpers
// (a & b) ^ c in one LOP3
__device__ __forceinline__ uint32_t and_xor(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t a) {
    uint32_t r;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(a));
    return r;
}
__device__ __forceinline__ float fast_exp2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
// int8 pages (rows of 128 bytes: the 8 token rows an ldmatrix reads would share their banks 8 ways) keep their K and
// V code rows in shared memory XOR-swizzled in 16-byte chunks (TMA SWIZZLE_32B / 64B / 128B: chunk bits [4, 4 + b)
// ^= address bits [7, 7 + b), m = 2^b - 1), so those rows, and the rows of a k-fragment load, fall in distinct
// banks; m = 0 is the unswizzled layout.  Every region base is a multiple of the swizzle's 1024-byte period.  int4
// pages (64-byte rows, 4-way) measured faster as one contiguous 1-D copy per page without the swizzle.
__device__ __forceinline__ uint32_t swz(uint32_t o, uint32_t m) { return o ^ (((o >> 7) & m) << 4); }

// lane 0 (predicated): arm `bar` for `bytes`, bring a page's K code box and V code box (tensor copies of the 3-D
// map [row bytes, rows of a block, blocks], coordinates (0, row, blk) and (0, row + vrows, blk)) and its scale bytes
// (1-D copy) into shared memory.  No multicast.
__device__ __forceinline__ void refill_tma_lane0(uint32_t lane, uint32_t bar, uint32_t dst_codes, uint32_t vbox,
                                                 const CUtensorMap* map, int32_t row, int32_t vrows, int32_t blk,
                                                 uint32_t dst_scales, const void* src_scales, uint32_t scale_bytes,
                                                 uint32_t bytes) {
    asm volatile(
        "{\n .reg .pred p;\n setp.eq.u32 p, %0, 0;\n"
        " @p mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %2;\n"
        " @p cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%3], [%4, {%5, %6, %7}], [%1];\n"
        " @p cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%8], [%4, {%5, %9, %7}], [%1];\n"
        " @p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%10], [%11], %12, [%1];\n}\n" ::"r"(lane),
        "r"(bar), "r"(bytes), "r"(dst_codes), "l"(map), "r"(0), "r"(row), "r"(blk), "r"(dst_codes + vbox),
        "r"(row + vrows), "r"(dst_scales), "l"(src_scales), "r"(scale_bytes)
        : "memory");
}

// lane 0 (predicated): a page as one 1-D copy of its record (int4 slots)
__device__ __forceinline__ void refill_lane0(uint32_t lane, uint32_t bar, uint32_t dst, const void* src, uint32_t bytes) {
    asm volatile(
        "{\n .reg .pred p;\n setp.eq.u32 p, %0, 0;\n"
        " @p mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %3;\n"
        " @p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%2], [%4], %3, [%1];\n}\n" ::"r"(lane),
        "r"(bar), "r"(dst), "r"(bytes), "l"(src)
        : "memory");
}

// lane 0 (predicated): a page as two 1-D copies (code rows, then scales) into split slots, for pools a tensor map
// cannot describe
__device__ __forceinline__ void refill_bulk_lane0(uint32_t lane, uint32_t bar, uint32_t dst_codes, const uint8_t* src,
                                                  uint32_t code_bytes, uint32_t dst_scales, uint32_t scale_bytes) {
    asm volatile(
        "{\n .reg .pred p;\n setp.eq.u32 p, %0, 0;\n"
        " @p mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %2;\n"
        " @p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%3], [%4], %5, [%1];\n"
        " @p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%6], [%7], %8, [%1];\n}\n" ::"r"(lane),
        "r"(bar), "r"(code_bytes + scale_bytes), "r"(dst_codes), "l"(src), "r"(code_bytes), "r"(dst_scales),
        "l"(src + code_bytes), "r"(scale_bytes)
        : "memory");
}

// fp16 constants as f16x2 words
constexpr uint32_t H2_1032 = 0x64086408u;       // 1024 + 8: int4 low-nibble offset
constexpr uint32_t H2_1152 = 0x64806480u;       // 1024 + 128: int8 offset
constexpr uint32_t H2_INV16 = 0x2C002C00u;      // 1/16
constexpr uint32_t H2_M72 = 0xD480D480u;        // -72 = -(1024/16 + 8)

// ------------------------------------------------------------------ layouts
template <int D, int BITS>
struct Lay {
    static constexpr int DC = BITS == 8 ? D : D / 2;
    static constexpr int CB = DC / 4;           // K: bytes of a token row per lane (quarter rows, lane % 4)
    static constexpr int CW = CB / 4;           // K: 32-bit words of it
    static constexpr int KT = D / 16;           // k-tiles of QK
    static constexpr int NPAIR = 2 * KT;        // K: f16x2 registers per token row per lane
    static constexpr int VB = DC / 8;           // V: bytes of a token row per lane (eighth rows, lane / 4)
    static constexpr int MT = D / 16;           // m-tiles (16 output dims) of PV
    // first of the two dims held by K pair e of lane quarter tid (pairs: e = 2 kt -> a0/a1/b0, 2 kt + 1 -> a2/a3/b1)
    __device__ static int kdim(int tid, int e) {
        if constexpr (BITS == 4) {
            const int wi = e >> 2, sub = e & 3;
            return tid * CB + 4 * wi + (sub & 1) * 2 + (sub >> 1) * (D / 2);
        } else {
            return tid * CB + 4 * (e >> 1) + 2 * (e & 1);
        }
    }
    // output dim of PV fragment row g (hi = 0) or g + 8 (hi = 1) of m-tile mt (the v_frags layout)
    __device__ static int vdim(int g, int mt, int hi) {
        if constexpr (BITS == 4) return hi * (D / 2) + 16 * (mt >> 1) + 2 * g + (mt & 1);
        else return 16 * mt + 2 * g + hi;
    }
};

// this lane's scale (or bias) pairs of one page, in K pair order, with 16-byte loads from the record in shared
// memory.  int4: pair e = 4 wi + sub covers dims run[sub >> 1] + 2 (2 wi + (sub & 1)), two runs of CB dims (one in
// each half of D); int8: pair e covers dims tid * CB + 2 e, one run of CB dims.
template <int D, int BITS>
__device__ __forceinline__ void load_pairs(const uint8_t* arr, int tid, uint32_t (&out)[2 * (D / 16)]) {
    using L = Lay<D, BITS>;
    constexpr int RUNS = BITS == 4 ? 2 : 1;
    constexpr int RW = L::CB / 2;                              // words per run
    uint32_t run[RUNS][RW];
#pragma unroll
    for (int h = 0; h < RUNS; h++) {
        const uint4* src = reinterpret_cast<const uint4*>(arr + 2 * (tid * L::CB + h * (D / 2)));
#pragma unroll
        for (int i = 0; i < RW / 4; i++) {
            const uint4 v = src[i];
            run[h][4 * i] = v.x;
            run[h][4 * i + 1] = v.y;
            run[h][4 * i + 2] = v.z;
            run[h][4 * i + 3] = v.w;
        }
    }
#pragma unroll
    for (int e = 0; e < 2 * L::KT; e++) {
        if constexpr (BITS == 4) out[e] = run[(e & 3) >> 1][2 * (e >> 2) + (e & 1)];
        else out[e] = run[0][e];
    }
}

// K' = c * ks + dkb of token rows g (r = 0) and g + 8 (r = 1) of a 16-token tile, straight into m16n8k16 A-fragment
// order: a[kt] = {row g pair 2kt, row g+8 pair 2kt, row g pair 2kt+1, row g+8 pair 2kt+1} (pair order of Lay::kdim).
// The lane's bytes of row r, chunk i are at codes + koff[r][i] (swizzled offsets).
template <int D, int BITS>
__device__ __forceinline__ void k_frags(const uint8_t* codes, const uint32_t (&koff)[2][(Lay<D, BITS>::CW + 3) / 4],
                                        const uint32_t (&ks)[2 * (D / 16)], const uint32_t (&dkb)[2 * (D / 16)],
                                        uint32_t (&a)[D / 16][4]) {
    using L = Lay<D, BITS>;
    uint32_t w[2][L::CW];
#pragma unroll
    for (int r = 0; r < 2; r++) {
        if constexpr (L::CW % 4 != 0) {                        // D = 64 int4: 8 bytes per lane
            const uint2 v = *reinterpret_cast<const uint2*>(codes + koff[r][0]);
            w[r][0] = v.x;
            w[r][1] = v.y;
        } else {
#pragma unroll
            for (int i = 0; i < L::CW / 4; i++) {
                const uint4 v = *reinterpret_cast<const uint4*>(codes + koff[r][i]);
                w[r][4 * i] = v.x;
                w[r][4 * i + 1] = v.y;
                w[r][4 * i + 2] = v.z;
                w[r][4 * i + 3] = v.w;
            }
        }
    }
#pragma unroll
    for (int wi = 0; wi < L::CW; wi++) {
#pragma unroll
        for (int r = 0; r < 2; r++) {
            if constexpr (BITS == 4) {
                // pairs e = 4 wi + sub: sub 0 lo(b0,b1), 1 lo(b2,b3), 2 hi(b0,b1), 3 hi(b2,b3); kt = e >> 1
                const uint32_t x = prmt(w[r][wi], 0, 0x3120);      // bytes [b0, b2, b1, b3]
                const uint32_t y = x >> 8;                          // bytes [b2, b1, b3, 0]
                const int e = 4 * wi;
                const uint32_t c0 = h2_sub(and_xor(x, 0x000F000Fu, H2_1032), H2_1032);
                const uint32_t c1 = h2_sub(and_xor(y, 0x000F000Fu, H2_1032), H2_1032);
                const uint32_t c2 = h2_fma(and_xor(x, 0x00F000F0u, 0x64806480u), H2_INV16, H2_M72);
                const uint32_t c3 = h2_fma(and_xor(y, 0x00F000F0u, 0x64806480u), H2_INV16, H2_M72);
                a[2 * wi][r] = h2_fma(c0, ks[e], dkb[e]);
                a[2 * wi][2 + r] = h2_fma(c1, ks[e + 1], dkb[e + 1]);
                a[2 * wi + 1][r] = h2_fma(c2, ks[e + 2], dkb[e + 2]);
                a[2 * wi + 1][2 + r] = h2_fma(c3, ks[e + 3], dkb[e + 3]);
            } else {
                // pairs e = 2 wi + sub: (b0,b1), (b2,b3); kt = wi
                const uint32_t u = w[r][wi] ^ 0x80808080u;          // signed code -> c + 128
                const uint32_t c0 = h2_sub(prmt(u, 0x64646464u, 0x5140), H2_1152);
                const uint32_t c1 = h2_sub(prmt(u, 0x64646464u, 0x7342), H2_1152);
                a[wi][r] = h2_fma(c0, ks[2 * wi], dkb[2 * wi]);
                a[wi][2 + r] = h2_fma(c1, ks[2 * wi + 1], dkb[2 * wi + 1]);
            }
        }
    }
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// V^T A fragments of one 16-token tile from the record's V rows at shared address vq.  The rows are read as 8x8
// matrices of 16-bit units (8 tokens x 16 bytes) with ldmatrix.trans, which hands lane (g, tid) the 2 bytes 2g, 2g+1
// of a 16-byte chunk for tokens 2tid and 2tid+1 in one register: the token interleave the A fragment needs.
//   int4: chunk k, byte b gives m-tile 2k + b: row g = low nibbles (dim 16k + 2g + b), row g+8 = high nibbles
//   int8: chunk k gives m-tile k: row g = byte 2g (dim 16k + 2g), row g+8 = byte 2g+1
// a[mt] = {row g x tokens 2tid,2tid+1 | row g+8 x same | row g x tokens 2tid+8,+9 | row g+8 x same}, exact codes.
// voff[ld]: this lane's (swizzled) row address offset of load ld -- matrices (tokens 0-7, chunk 2ld), (0-7, 2ld+1),
// (8-15, 2ld), (8-15, 2ld+1), lane (mi, rr) addressing row rr of matrix mi.
template <int D, int BITS>
__device__ __forceinline__ void v_frags(uint32_t vq, const uint32_t (&voff)[Lay<D, BITS>::DC / 32], uint32_t (&a)[D / 16][4]) {
    using L = Lay<D, BITS>;
    constexpr int NCH = L::DC / 16;                       // 16-byte chunks per token row
#pragma unroll
    for (int ld = 0; ld < NCH / 2; ld++) {
        uint32_t r[4];
        ldsm_x4_trans(vq + voff[ld], r);
#pragma unroll
        for (int c = 0; c < 2; c++) {                     // chunk k = 2 ld + c
            const int k = 2 * ld + c;
            const uint32_t lo_t = r[c], hi_t = r[2 + c];  // tokens 2tid,2tid+1 | 2tid+8,2tid+9
            if constexpr (BITS == 4) {
#pragma unroll
                for (int b = 0; b < 2; b++) {
                    const uint32_t x0 = b ? lo_t >> 8 : lo_t, x1 = b ? hi_t >> 8 : hi_t;
                    const int mt = 2 * k + b;
                    a[mt][0] = h2_sub(and_xor(x0, 0x000F000Fu, H2_1032), H2_1032);
                    a[mt][1] = h2_fma(and_xor(x0, 0x00F000F0u, 0x64806480u), H2_INV16, H2_M72);
                    a[mt][2] = h2_sub(and_xor(x1, 0x000F000Fu, H2_1032), H2_1032);
                    a[mt][3] = h2_fma(and_xor(x1, 0x00F000F0u, 0x64806480u), H2_INV16, H2_M72);
                }
            } else {
                const uint32_t u0 = lo_t ^ 0x80808080u, u1 = hi_t ^ 0x80808080u;   // signed code -> c + 128
                a[k][0] = h2_sub(prmt(u0, 0x64646464u, 0x4240), H2_1152);       // byte 2g of tokens t0, t1
                a[k][1] = h2_sub(prmt(u0, 0x64646464u, 0x4341), H2_1152);       // byte 2g + 1
                a[k][2] = h2_sub(prmt(u1, 0x64646464u, 0x4240), H2_1152);
                a[k][3] = h2_sub(prmt(u1, 0x64646464u, 0x4341), H2_1152);
            }
        }
    }
}

template <int D, int BITS, int P, int NT>
struct MmaCfg {
    static constexpr int RB = Fmt<D, BITS, P>::RB;
    static constexpr int CODES = 2 * P * Fmt<D, BITS, P>::DC;     // K then V code rows of a page
    static constexpr int SCALES = RB - CODES;                      // ks, kb, vs, vb
    // int8: split slots (code rows, swizzled by tensor copies, apart from the scales); int4: one record per slot
    static constexpr bool SPLIT = BITS == 8;
    static constexpr int CSTRIDE = SPLIT ? CODES : RB;             // code slot stride
    // ring slots per warp: deep enough to keep ~2 pages in flight per warp at 4 CTAs per SM
    static constexpr int NS = RB <= 3072 ? 4 : 2;
    static constexpr int GMAX = 8 * NT;
    static constexpr int MERGE = 4 * ((MMA_NW + 1) * GMAX * D + 2 * (MMA_NW + 1) * GMAX);
    // after the merge area: the tail page's record from its V code rows on (V rows, then at their record offsets the
    // V scales and biases), staged for the tail partial
    static constexpr int TSTAGE = (MERGE + 15) / 16 * 16;
    static constexpr int TEND = TSTAGE + RB - Fmt<D, BITS, P>::OFF_VQ;
    static constexpr int RING = MMA_NW * NS * RB > TEND ? MMA_NW * NS * RB : (TEND + 127) / 128 * 128;
    static constexpr int BARS = (8 * MMA_NW * NS + 127) / 128 * 128;
    // shared memory: [bars | pad to 1024 | ring: int8 code slots [NW][NS][CODES] + scale slots [NW][NS][SCALES], int4
    // record slots [NW][NS][RB] (reused by the merge) | q * scale (fp32, [G][D]) | kb_ref (fp32, [D]) | kb_ref (fp16,
    // [D])]; the pad aligns
    // the code slots to the swizzle period
    static constexpr int SMEM = 1024 + BARS + RING + 4 * (GMAX * D + D) + 2 * D;
    static_assert(!SPLIT || (CODES % 1024 == 0 && SCALES % 16 == 0), "code slots must keep the swizzle period");
    // CTAs per SM the register budget targets (the larger tiles need more registers per thread)
    static constexpr int MINB = (D == 64 || (D == 128 && NT == 1 && !(BITS == 8 && P == 32))) ? 4
                                : NT == 1 && D == 128 ? 3 : 2;
};

// scores more than 2^TAU above the running max trigger a rescale; below that the stale max is kept (weights
// p = exp2(s - m) <= 2^TAU stay far from fp16 overflow in p * vs)
constexpr float TAU = 4.0f;

// The split-KV combine inside the decode launch (kush_sm100_decode_fused_combine).  Each CTA of (sequence, kv head)
// sh counts itself on counters[sh] after its partial is stored; the last of the n_splits CTAs sets the count back to
// 0 (so the counters are ready for the next launch) and merges every split into out.  The arithmetic is merge_splits'
// (combine_kernel / combine_rot_kernel: the max over the splits, f = e^(m_z - M), L and o accumulated with fmaf in
// split order, o / L), so the output is bit-identical to the decode followed by kush_sm100_combine(_rotated); the
// work is laid out for one pass of loads: the (m, l) pairs of the unit (contiguous) and the factors f in shared
// memory, then each thread's partial outputs with all loads of a head in flight.
// smem: cap floats of shared memory no longer in use; units whose 3 * n_splits * G + 2 * G (+ G * D with ROT) floats
// do not fit merge each output straight from global memory (merge_splits, the same arithmetic).
template <int D, bool ROT, class IN>
__device__ __noinline__ void combine_if_last(int32_t* counters, int64_t sh, int n_splits, int G,
                                             const float* part_ml, const float* part_o, IN* out, float* smem, int cap) {
    __shared__ int last;
    __threadfence();                                  // this CTA's partial is visible before it is counted
    __syncthreads();
    if (threadIdx.x == 0) {
        last = atomicAdd(&counters[sh], 1) == n_splits - 1;
        if (last) counters[sh] = 0;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    const int nz = n_splits * G;
    const float* ml = part_ml + sh * nz * 2;          // [split][head][m, l] of this unit
    const float* po = part_o + sh * nz * D;           // [split][head][D]
    float* sml = smem;                                // the unit's (m, l) pairs
    float* fz = smem + 2 * nz;                        // f of (split, head)
    float* sL = fz + nz;                              // L per head
    float* stage = sL + 2 * G;
    if (3 * nz + 2 * G + (ROT ? G * D : 0) > cap) {
        stage = smem;
        for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
            const int hd = idx / D, d = idx % D;
            const float r = merge_splits<true>(ml + 2 * hd, po + int64_t(hd) * D + d, n_splits, G, D);
            if constexpr (ROT) stage[idx] = r;
            else out[sh * G * D + idx] = from_f32<IN>(r);
        }
    } else {
    for (int i = threadIdx.x; i < 2 * nz; i += blockDim.x) sml[i] = __ldcg(ml + i);
    __syncthreads();
    for (int hd = threadIdx.x; hd < G; hd += blockDim.x) {
        float M = -INFINITY;
        for (int z = 0; z < n_splits; z++) M = fmaxf(M, sml[2 * (z * G + hd)]);
        float L = 0.0f;
        for (int z = 0; z < n_splits; z++) {
            const float mz = sml[2 * (z * G + hd)];
            const float f = mz > -INFINITY ? __expf(mz - M) : 0.0f;
            fz[z * G + hd] = f;
            if (mz > -INFINITY) L = fmaf(sml[2 * (z * G + hd) + 1], f, L);
        }
        sL[hd] = L;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int hd = idx / D, d = idx % D;
        float o = 0.0f;
#pragma unroll 4
        for (int z = 0; z < n_splits; z++) {
            const float v = __ldcg(po + (int64_t(z) * G + hd) * D + d);
            if (sml[2 * (z * G + hd)] > -INFINITY) o = fmaf(fz[z * G + hd], v, o);
        }
        const float L = sL[hd];
        const float r = L > 0.0f ? o / L : 0.0f;
        if constexpr (ROT) stage[idx] = r;
        else out[sh * G * D + idx] = from_f32<IN>(r);
    }
    }
    if constexpr (ROT) {
        __syncthreads();
        constexpr int R = D / WARP;
        const int lane = threadIdx.x % WARP;
        for (int hd = threadIdx.x / WARP; hd < G; hd += blockDim.x / WARP) {
            float x[R];
#pragma unroll
            for (int i = 0; i < R; i++) x[i] = stage[hd * D + lane + WARP * i];
            fwht_warp<D>(x, lane);
#pragma unroll
            for (int i = 0; i < R; i++) out[(sh * G + hd) * D + lane + WARP * i] = from_f32<IN>(x[i]);
        }
    }
}

// grid (S, Hkv, n_splits), block 128.  ROT: q rotated in the prologue and the output rotated back before its store;
// ORD: CTA x works on sequence order[x] (separate instantiations, so the plain kernels keep their code)
template <int D, int BITS, int P, int NT, class IN, bool ROT, bool ORD>
__global__ void __launch_bounds__(MMA_NW * WARP, (MmaCfg<D, BITS, P, NT>::MINB)) decode_mma_kernel(
    const IN* __restrict__ q, IN* __restrict__ out, const uint8_t* __restrict__ cache, int64_t block_stride,
    int64_t head_stride, const IN* __restrict__ tail_k, const int32_t* __restrict__ tail_idx,
    const int32_t* __restrict__ block_table, const int32_t* __restrict__ seq_lens, int64_t max_pages, int H, int G,
    float sm_log2, int n_splits, float* __restrict__ part_ml, float* __restrict__ part_o,
    const __grid_constant__ CUtensorMap tmap, int use_tma, uint32_t swz_m, int32_t rows_per_head, int32_t box_rows,
    const int32_t* __restrict__ order, int32_t* __restrict__ counters) {
    using F = Fmt<D, BITS, P>;
    using L = Lay<D, BITS>;
    using C = MmaCfg<D, BITS, P, NT>;
    constexpr int NW = MMA_NW, NS = C::NS, KT = L::KT, MT = L::MT, MTT = P / 16;
    pdl_wait();                                                         // previous kernel on the stream done
    if (n_splits == 1) pdl_trigger();         // no combine follows: the next launch may start behind the last wave
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);                 // [NW][NS]
    const uint32_t smem0 = smem_u32(smem);
    uint8_t* ring = smem + (((smem0 + C::BARS + 1023u) & ~1023u) - smem0);   // code + scale slots, reused by the merge
    float* qsm = reinterpret_cast<float*>(ring + C::RING);              // [G][D] q * scale * log2e
    float* kbr = qsm + G * D;                                           // [D] kb_ref
    __half* kb16 = reinterpret_cast<__half*>(kbr + D);                  // [D] kb_ref as fp16 (read in K pair order)
    const int s = ORD ? order[blockIdx.x] : blockIdx.x, h = blockIdx.y, z = blockIdx.z;     // launch order
    const int wid = threadIdx.x / WARP, lane = threadIdx.x % WARP, g = lane >> 2, tid = lane & 3;
    const int64_t n = seq_lens[s];
    const int tail_n = int(n % P);
    const int64_t full = n / P;
    const SplitRange sr = split_range(seq_lens, int(gridDim.x), s, z, n_splits, P);
    if (!sr.active) {                                                   // no pages here: an empty partial
        for (int hd = threadIdx.x; hd < G; hd += NW * WARP) {
            const int64_t pb = ((int64_t(s) * H + h) * n_splits + z) * G + hd;
            part_ml[pb * 2] = -INFINITY;
            part_ml[pb * 2 + 1] = 0.0f;
        }
        if (counters)
            combine_if_last<D, ROT>(counters, int64_t(s) * H + h, n_splits, G, part_ml, part_o, out,
                                    reinterpret_cast<float*>(smem + 1024), (C::SMEM - 1024) / 4);
        return;
    }
    const int64_t p0 = sr.p0, p1 = sr.p1;
    const int32_t* bt = block_table + int64_t(s) * max_pages;
    const int64_t qbase = (int64_t(s) * H + h) * G * D;
    const uint8_t* hcache = cache + int64_t(h) * head_stride;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NW * NS; i++) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    // my pages: p0 + wid + i * NW, i < npw; start their copies before anything else
    const int64_t mine0 = p0 + wid;
    const int npw = mine0 < p1 ? int((p1 - mine0 + NW - 1) / NW) : 0;
    uint8_t* wcodes = ring + wid * NS * C::CSTRIDE;                     // this warp's code (int4: record) slots
    uint8_t* wscl = ring + NW * NS * C::CODES + wid * NS * C::SCALES;   // and its scale slots (int8)
    uint64_t* wbar = bars + wid * NS;
    auto bt_at = [&](int i) -> int32_t { return i < npw ? bt[mine0 + int64_t(i) * NW] : 0; };
    int32_t btw = bt_at(lane), btn = bt_at(32 + lane);                 // block ids of my pages, 32 at a time
    const uint32_t codes_u = smem_u32(wcodes), scl_u = smem_u32(wscl), bar_u = smem_u32(wbar);
    const int32_t hrow = h * rows_per_head;                             // the record's first row in the tensor map
    auto issue = [&](int i, int32_t blk) {                              // lane 0: page i -> slot i % NS
        const uint32_t slot = uint32_t(i) % NS;
        const uint8_t* src = hcache + int64_t(blk) * block_stride;
        if constexpr (!C::SPLIT)
            refill_lane0(uint32_t(lane), bar_u + 8 * slot, codes_u + slot * C::RB, src, C::RB);
        else if (use_tma)
            refill_tma_lane0(uint32_t(lane), bar_u + 8 * slot, codes_u + slot * C::CODES, C::CODES / 2, &tmap, hrow,
                             box_rows, blk, scl_u + slot * C::SCALES, src + C::CODES, C::SCALES, C::RB);
        else
            refill_bulk_lane0(uint32_t(lane), bar_u + 8 * slot, codes_u + slot * C::CODES, src, C::CODES,
                              scl_u + slot * C::SCALES, C::SCALES);
    };
    // this lane's swizzled offsets in a 16-token tile: K rows g, g + 8 at its bytes; V ldmatrix row addresses
    // (a tile 16 rows further keeps the same swizzle: 16 rows move the row bits by a multiple of the period)
    const uint32_t sm = C::SPLIT ? swz_m : 0u;                         // int4: a constant 0 (offsets fold away)
    uint32_t koff[2][(L::CW + 3) / 4], voff[L::DC / 32];
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
        for (int i = 0; i < (L::CW + 3) / 4; i++) koff[r][i] = swz(uint32_t((g + 8 * r) * F::DC + tid * L::CB + 16 * i), sm);
#pragma unroll
    for (int ld = 0; ld < L::DC / 32; ld++)
        voff[ld] = swz(uint32_t((((lane >> 3) >> 1) * 8 + (lane & 7)) * F::DC + 16 * (2 * ld + ((lane >> 3) & 1))), sm);
    __syncthreads();                                                    // barriers initialised
#pragma unroll 1
    for (int i = 0; i < NS && i < npw; i++) issue(i, __shfl_sync(0xffffffffu, btw, i));

    if constexpr (ROT) {                              // q rotated in fp32 (canonical FWHT) as it loads, then scaled
        for (int hd = wid; hd < G; hd += NW) {
            float x[D / WARP];
#pragma unroll
            for (int i = 0; i < D / WARP; i++) x[i] = to_f32(q[qbase + hd * D + lane + WARP * i]);
            fwht_warp<D>(x, lane);
#pragma unroll
            for (int i = 0; i < D / WARP; i++) qsm[hd * D + lane + WARP * i] = x[i] * sm_log2;
        }
    } else {
        for (int i = threadIdx.x; i < G * D; i += NW * WARP) qsm[i] = to_f32(q[qbase + i]) * sm_log2;
    }
    // kb_ref: K bias of the sequence's first page (only when one is full; a tail-only sequence uses 0)
    const uint8_t* rec0 = full > 0 ? hcache + int64_t(bt[0]) * block_stride : nullptr;
    for (int i = threadIdx.x; i < D; i += NW * WARP) {
        const __half kb = rec0 ? reinterpret_cast<const __half*>(rec0 + F::OFF_KB)[i] : __float2half_rn(0.0f);
        kbr[i] = __half2float(kb);
        kb16[i] = kb;
    }
    __syncthreads();

    // B fragments: Qh^T for heads nt*8 + g at this lane's K pairs; the kb_ref pairs in registers for 16-token pages,
    // read per tile from kb16 for 32-token pages (whose two tiles per page need the 16 registers)
    constexpr bool KREF_REGS = P == 16;
    uint32_t bq[NT][2 * KT];
    uint32_t kref_r[KREF_REGS ? 2 * KT : 1];
#pragma unroll
    for (int e = 0; e < 2 * KT; e++) {
        const int d = L::kdim(tid, e);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int head = nt * 8 + g;
            bq[nt][e] = head < G ? pack_h2(qsm[head * D + d], qsm[head * D + d + 1]) : 0u;
        }
        if constexpr (KREF_REGS) kref_r[e] = pack_h2(kbr[d], kbr[d + 1]);
    }

    float o[MT][NT][4];                                                  // O^T accumulators
#pragma unroll
    for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int k = 0; k < 4; k++) o[mt][nt][k] = 0.0f;
    float m[NT][2], l[NT][2], vbacc[NT][2];                              // heads nt*8 + 2tid + {0,1} (lane partials)
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            m[nt][e] = -INFINITY;
            l[nt][e] = 0.0f;
            vbacc[nt][e] = 0.0f;
        }
    bool ok = true;
    int fail_at = npw;

#pragma unroll 1
    for (int i = 0; i < npw; i++) {
        const int slot = int(uint32_t(i) % NS);
        if (!mbar_wait_u32(bar_u + 8 * slot, (uint32_t(i) / NS) & 1u)) {
            ok = false;
            fail_at = i;
            break;
        }
        const uint8_t* codes = wcodes + slot * C::CSTRIDE;               // K rows, then V rows (int8: swizzled)
        const uint8_t* scl = C::SPLIT ? wscl + slot * C::SCALES : codes + C::CODES;   // ks, kb, vs, vb
        // one 16-token tile at a time (P = 32 pages have two): QK, online softmax, PV.  The softmax is tile-granular,
        // which keeps the register footprint of both page sizes the same.
#pragma unroll
        for (int mtt = 0; mtt < MTT; mtt++) {
            float sc[NT][4];
            {
                // the page's K scale and bias pairs for this lane's dims (K' = c * ks + (kb - kb_ref)); reloaded per
                // tile rather than held across the tiles of a 32-token page (register pressure)
                uint32_t ks[2 * KT], dkb[2 * KT];
                load_pairs<D, BITS>(scl, tid, ks);
                load_pairs<D, BITS>(scl + 2 * D, tid, dkb);
                if constexpr (KREF_REGS) {
#pragma unroll
                    for (int e = 0; e < 2 * KT; e++) dkb[e] = h2_sub(dkb[e], kref_r[e]);
                } else {
                    uint32_t kref[2 * KT];
                    load_pairs<D, BITS>(reinterpret_cast<const uint8_t*>(kb16), tid, kref);
#pragma unroll
                    for (int e = 0; e < 2 * KT; e++) dkb[e] = h2_sub(dkb[e], kref[e]);
                }
                uint32_t ka[KT][4];                                       // A fragments of this 16-token tile
                k_frags<D, BITS>(codes + mtt * 16 * F::DC, koff, ks, dkb, ka);
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    float s0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s1[4] = {0.0f, 0.0f, 0.0f, 0.0f};   // two chains
#pragma unroll
                    for (int kt = 0; kt < KT; kt += 2) {
                        mma16816(s0, ka[kt][0], ka[kt][1], ka[kt][2], ka[kt][3], bq[nt][2 * kt], bq[nt][2 * kt + 1]);
                        mma16816(s1, ka[kt + 1][0], ka[kt + 1][1], ka[kt + 1][2], ka[kt + 1][3], bq[nt][2 * kt + 2],
                                 bq[nt][2 * kt + 3]);
                    }
                    const float2 a01 = __fadd2_rn(make_float2(s0[0], s0[1]), make_float2(s1[0], s1[1]));
                    const float2 a23 = __fadd2_rn(make_float2(s0[2], s0[3]), make_float2(s1[2], s1[3]));
                    sc[nt][0] = a01.x;
                    sc[nt][1] = a01.y;
                    sc[nt][2] = a23.x;
                    sc[nt][3] = a23.y;
                }
            }
            // online softmax with a lazily moved max; lane holds tokens mtt*16 + g (+8), heads nt*8 + 2tid + {0,1}
            bool bump = false;
            float lmx[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                lmx[nt][0] = fmaxf(sc[nt][0], sc[nt][2]);
                lmx[nt][1] = fmaxf(sc[nt][1], sc[nt][3]);
                bump |= lmx[nt][0] > m[nt][0] + TAU || lmx[nt][1] > m[nt][1] + TAU;
            }
            if (__any_sync(0xffffffffu, bump)) {                         // rare: move the max to the exact one
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    float corr[2];
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        float mx = lmx[nt][e];
#pragma unroll
                        for (int off = 4; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                        const float mn = fmaxf(m[nt][e], mx);
                        corr[e] = fast_exp2(m[nt][e] - mn);
                        m[nt][e] = mn;
                        l[nt][e] *= corr[e];
                        vbacc[nt][e] *= corr[e];
                    }
#pragma unroll
                    for (int mt = 0; mt < MT; mt++) {
                        o[mt][nt][0] *= corr[0];
                        o[mt][nt][1] *= corr[1];
                        o[mt][nt][2] *= corr[0];
                        o[mt][nt][3] *= corr[1];
                    }
                }
            }
            float vsv[2], vbv[2];
#pragma unroll
            for (int r = 0; r < 2; r++) {
                vsv[r] = h_load(scl + 4 * D, mtt * 16 + g + 8 * r);
                vbv[r] = h_load(scl + 4 * D + 2 * P, mtt * 16 + g + 8 * r);
            }
            uint32_t pb[NT][2];                                           // P'^T B fragments of this tile
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                // head pair (2tid, 2tid+1) of token row r in packed fp32x2 arithmetic (sm_100 FADD2/FFMA2/FMUL2)
                const float2 negm = make_float2(-m[nt][0], -m[nt][1]);
                float2 lp = make_float2(l[nt][0], l[nt][1]), vp = make_float2(vbacc[nt][0], vbacc[nt][1]);
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    const float2 d = __fadd2_rn(make_float2(sc[nt][2 * r], sc[nt][2 * r + 1]), negm);
                    const float2 p = make_float2(fast_exp2(d.x), fast_exp2(d.y));
                    lp = __fadd2_rn(lp, p);
                    vp = __ffma2_rn(p, make_float2(vbv[r], vbv[r]), vp);
                    const float2 pv = __fmul2_rn(p, make_float2(vsv[r], vsv[r]));
                    pb[nt][r] = movmatrix_t(pack_h2(pv.x, pv.y));        // r = 0: tokens 0-7, 1: tokens 8-15
                }
                l[nt][0] = lp.x;
                l[nt][1] = lp.y;
                vbacc[nt][0] = vp.x;
                vbacc[nt][1] = vp.y;
            }
            uint32_t va[MT][4];
            v_frags<D, BITS>(smem_u32(codes) + C::CODES / 2 + mtt * 16 * F::DC, voff, va);
#pragma unroll
            for (int mt = 0; mt < MT; mt++)
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
                    mma16816(o[mt][nt], va[mt][0], va[mt][1], va[mt][2], va[mt][3], pb[nt][0], pb[nt][1]);
        }
        __syncwarp();
        // refill this slot with page i + NS
        const int j = i + NS;
        if (j < npw) {
            if ((j & 31) == 0) {
                btw = btn;
                btn = bt_at(j + 32 + lane);
            }
            issue(j, __shfl_sync(0xffffffffu, btw, j & 31));
        }
    }
    if (!ok) {
        // a copy never completed: record it, wait (bounded) for this warp's copies still in flight, produce NaN
        if (lane == 0) atomicExch(&g_decode_error, 1);
        for (int i = fail_at + 1; i < fail_at + NS && i < npw; i++)
            mbar_wait_u32(bar_u + 8 * (uint32_t(i) % NS), (uint32_t(i) / NS) & 1u);
    }
    ok = __syncthreads_and(ok);

    // merge (kushkash/kush/gpu.mojo:438-466): per warp m, l, O + vbacc -> shared; partial NW = the exact-K tail
    float* c_acc = reinterpret_cast<float*>(ring);                        // [NW + 1][G][D]
    float* c_m = c_acc + (NW + 1) * G * D;                                // [NW + 1][G]
    float* c_l = c_m + (NW + 1) * G;
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                l[nt][e] += __shfl_xor_sync(0xffffffffu, l[nt][e], off);
                vbacc[nt][e] += __shfl_xor_sync(0xffffffffu, vbacc[nt][e], off);
            }
        }
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int head = nt * 8 + 2 * tid + e;
            if (head < G) {
#pragma unroll
                for (int mt = 0; mt < MT; mt++) {
                    c_acc[(wid * G + head) * D + L::vdim(g, mt, 0)] = o[mt][nt][e] + vbacc[nt][e];
                    c_acc[(wid * G + head) * D + L::vdim(g, mt, 1)] = o[mt][nt][2 + e] + vbacc[nt][e];
                }
                if (g == 0) {
                    c_m[wid * G + head] = m[nt][e];
                    c_l[wid * G + head] = l[nt][e];
                }
            }
        }
    // the tail page: exact K from tail_k, V rows from its record, fp32 on the CUDA cores; warp w takes heads w, w+NW..
    {
        const bool has_tail = tail_n > 0 && sr.last;
        const IN* tk = has_tail ? tail_k + ((int64_t(tail_idx[s]) * H + h) * P + min(lane, P - 1)) * D : nullptr;
        const uint8_t* trec = has_tail ? hcache + int64_t(bt[full]) * block_stride : nullptr;
        constexpr int R = D / WARP;
        // the record's V rows [0, tail_n) and its V scales and biases into shared memory, all 16-byte loads in flight
        // at once (read per token from global memory, the tail cost one round trip per token)
        uint8_t* tv = ring + C::TSTAGE;
        if (has_tail) {
            const int nv = tail_n * F::DC / 16;
            for (int i = threadIdx.x; i < nv + P / 4; i += NW * WARP) {
                const int off = i < nv ? F::OFF_VQ + 16 * i : F::OFF_VS + 16 * (i - nv);
                *reinterpret_cast<uint4*>(tv + off - F::OFF_VQ) = *reinterpret_cast<const uint4*>(trec + off);
            }
        }
        __syncthreads();
        for (int hd = wid; hd < G; hd += NW) {
            const float* qh = qsm + hd * D;
            float qkref = 0.0f;                                          // q . kb_ref (the shift of every score)
            for (int d = lane; d < D; d += WARP) qkref = fmaf(qh[d], kbr[d], qkref);
            qkref = warp_sum(qkref);
            float x = -INFINITY;
            if (has_tail && lane < tail_n) {
                constexpr int VE = 16 / sizeof(IN);                      // elements per 16-byte load
                float acc = 0.0f;
                for (int d0 = 0; d0 < D; d0 += VE) {
                    const uint4 raw = *reinterpret_cast<const uint4*>(tk + d0);
                    const IN* e = reinterpret_cast<const IN*>(&raw);
#pragma unroll
                    for (int k = 0; k < VE; k++) acc = fmaf(qh[d0 + k], to_f32(e[k]), acc);
                }
                x = acc - qkref;
            }
            const float mx = warp_max(x);
            const float p = (has_tail && lane < tail_n) ? fast_exp2(x - mx) : 0.0f;
            const float lsum = warp_sum(p);
            if (lane == 0) {
                c_m[NW * G + hd] = has_tail ? mx : -INFINITY;
                c_l[NW * G + hd] = lsum;
            }
            float acc[R];
#pragma unroll
            for (int i = 0; i < R; i++) acc[i] = 0.0f;
            for (int t = 0; t < tail_n && has_tail; t++) {               // lane holds dims lane + 32 i
                const float pt = __shfl_sync(0xffffffffu, p, t);
                const float vs = h_load(tv + F::OFF_VS - F::OFF_VQ, t) * pt, vb = h_load(tv + F::OFF_VB - F::OFF_VQ, t) * pt;
#pragma unroll
                for (int i = 0; i < R; i++)
                    acc[i] = fmaf(float(code_at<D, BITS>(tv + t * F::DC, lane + WARP * i)), vs, acc[i] + vb);
            }
#pragma unroll
            for (int i = 0; i < R; i++) c_acc[(NW * G + hd) * D + lane + WARP * i] = acc[i];
        }
    }
    __syncthreads();
    if (ROT && n_splits == 1) {                       // one warp per head: merge, rotate back (canonical FWHT), store
        constexpr int R = D / WARP;
        for (int hd = wid; hd < G; hd += NW) {
            float M = -INFINITY;
            for (int w = 0; w <= NW; w++) M = fmaxf(M, c_m[w * G + hd]);
            float Ls = 0.0f, x[R];
#pragma unroll
            for (int i = 0; i < R; i++) x[i] = 0.0f;
            if (M > -INFINITY) {
                for (int w = 0; w <= NW; w++) {
                    const float mw = c_m[w * G + hd];
                    if (mw > -INFINITY) {
                        const float f = fast_exp2(mw - M);
                        Ls += c_l[w * G + hd] * f;
#pragma unroll
                        for (int i = 0; i < R; i++) x[i] += f * c_acc[(w * G + hd) * D + lane + WARP * i];
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < R; i++) x[i] = !ok ? NAN : Ls > 0.0f ? x[i] / Ls : 0.0f;
            fwht_warp<D>(x, lane);
#pragma unroll
            for (int i = 0; i < R; i++) out[qbase + hd * D + lane + WARP * i] = from_f32<IN>(x[i]);
        }
        return;
    }
    for (int idx = threadIdx.x; idx < G * D; idx += NW * WARP) {
        const int hd = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w = 0; w <= NW; w++) M = fmaxf(M, c_m[w * G + hd]);
        float Ls = 0.0f, acc = 0.0f;
        if (M > -INFINITY) {
            for (int w = 0; w <= NW; w++) {
                const float mw = c_m[w * G + hd];
                if (mw > -INFINITY) {
                    const float f = fast_exp2(mw - M);
                    Ls += c_l[w * G + hd] * f;
                    acc += f * c_acc[(w * G + hd) * D + d];
                }
            }
        }
        if (!ok) acc = NAN;
        if (n_splits == 1) {
            out[qbase + idx] = from_f32<IN>(Ls > 0.0f ? acc / Ls : (ok ? 0.0f : NAN));
        } else {
            const int64_t pb = ((int64_t(s) * H + h) * n_splits + z) * G + hd;
            part_o[pb * D + d] = acc;
            if (d == 0) {
                part_ml[pb * 2] = M * 0.69314718055994531f;           // log2 units -> natural, for the combine
                part_ml[pb * 2 + 1] = Ls;
            }
        }
    }
    if (n_splits > 1 && counters)
        combine_if_last<D, ROT>(counters, int64_t(s) * H + h, n_splits, G, part_ml, part_o, out,
                                reinterpret_cast<float*>(smem + 1024), (C::SMEM - 1024) / 4);
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// the driver's cuTensorMapEncodeTiled (through the runtime's entry-point query: no link against libcuda), or null
static EncodeTiled encode_tiled() {
    static EncodeTiled fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return EncodeTiled(nullptr);
        return reinterpret_cast<EncodeTiled>(p);
    }();
    return fn;
}

// The pool as a 3-D uint8 tensor [sr bytes, block_stride / sr rows, blocks] with sr the widest swizzle row (<= 128,
// <= a code row) dividing both byte strides; box = one page's K (or V) code rows.  False (plain copies) when no sr
// >= 32 fits or the driver refuses the map.
template <int D, int BITS, int P>
bool make_page_map(const void* cache, int64_t block_stride, int64_t head_stride, CUtensorMap& map, uint32_t& m,
                   int32_t& rows_per_head, int32_t& box_rows) {
    constexpr int DC = Fmt<D, BITS, P>::DC;
    int sr = DC < 128 ? DC : 128;
    while (sr >= 32 && (block_stride % sr || head_stride % sr)) sr >>= 1;
    const EncodeTiled enc = encode_tiled();
    if (sr < 32 || !enc || block_stride / sr > (int64_t(1) << 31) || head_stride / sr > (int64_t(1) << 24)) return false;
    const cuuint64_t gdim[3] = {cuuint64_t(sr), cuuint64_t(block_stride / sr), cuuint64_t(0x7FFFFFFF)};
    const cuuint64_t gstride[2] = {cuuint64_t(sr), cuuint64_t(block_stride)};
    const cuuint32_t box[3] = {cuuint32_t(sr), cuuint32_t(P * DC / sr), 1u};
    const cuuint32_t estride[3] = {1u, 1u, 1u};
    const CUtensorMapSwizzle sw = sr == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                  : sr == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(cache), gdim, gstride, box, estride,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    m = uint32_t(sr / 16 - 1);
    rows_per_head = int32_t(head_stride / sr);
    box_rows = P * DC / sr;
    return true;
}

template <int D, int BITS, int P, int NT, class IN, bool ROT, bool ORD>
int launch_mma_rot(int G, const void* q, void* out, const void* cache, int64_t block_stride, int64_t head_stride,
                   const void* tail_k, const int32_t* tail_idx, const int32_t* block_table, const int32_t* seq_lens,
                   int64_t max_pages, int32_t hkv, float scale, int32_t n_splits, float* part_ml, float* part_o,
                   int32_t n_seqs, const int32_t* order, int32_t* counters, cudaStream_t stream) {
    using C = MmaCfg<D, BITS, P, NT>;
    auto kern = decode_mma_kernel<D, BITS, P, NT, IN, ROT, ORD>;
    CUtensorMap map;
    memset(&map, 0, sizeof(map));
    uint32_t swz_m = 0;
    int32_t rows_per_head = 0, box_rows = 0;
    const bool tma = C::SPLIT &&
                     make_page_map<D, BITS, P>(cache, block_stride, head_stride, map, swz_m, rows_per_head, box_rows);
    if (!tma) swz_m = 0;
    static unsigned long long attr_set = 0;             // one bit per device: the attribute is per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_set >> (dev & 63) & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return set_error(KUSH_ERR_CUDA, "decode: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        attr_set |= 1ull << (dev & 63);
    }
    dim3 grid(n_seqs, hkv, n_splits);
    launch_pdl(kern, grid, dim3(MMA_NW * WARP), C::SMEM, stream, static_cast<const IN*>(q), static_cast<IN*>(out),
               static_cast<const uint8_t*>(cache), block_stride, head_stride, static_cast<const IN*>(tail_k), tail_idx,
               block_table, seq_lens, max_pages, hkv, G, scale * 1.4426950408889634f, n_splits, part_ml, part_o, map,
               tma ? 1 : 0, swz_m, rows_per_head, box_rows, order, counters);
    return check_launch("kush_sm100_decode (tensor cores)");
}

template <int D, int BITS, int P, int NT, class IN>
int launch_mma(int G, const void* q, void* out, const void* cache, int64_t block_stride, int64_t head_stride,
               const void* tail_k, const int32_t* tail_idx, const int32_t* block_table, const int32_t* seq_lens,
               int64_t max_pages, int32_t hkv, float scale, int32_t n_splits, float* part_ml, float* part_o,
               int32_t n_seqs, int rot, const int32_t* order, int32_t* counters, cudaStream_t stream) {
    if (rot)                                          // (the rotated decode runs in the natural order)
        return launch_mma_rot<D, BITS, P, NT, IN, true, false>(G, q, out, cache, block_stride, head_stride, tail_k,
                                                               tail_idx, block_table, seq_lens, max_pages, hkv, scale,
                                                               n_splits, part_ml, part_o, n_seqs, nullptr, counters, stream);
    if (order)
        return launch_mma_rot<D, BITS, P, NT, IN, false, true>(G, q, out, cache, block_stride, head_stride, tail_k,
                                                               tail_idx, block_table, seq_lens, max_pages, hkv, scale,
                                                               n_splits, part_ml, part_o, n_seqs, order, counters, stream);
    return launch_mma_rot<D, BITS, P, NT, IN, false, false>(G, q, out, cache, block_stride, head_stride, tail_k,
                                                            tail_idx, block_table, seq_lens, max_pages, hkv, scale,
                                                            n_splits, part_ml, part_o, n_seqs, nullptr, counters, stream);
}

int decode_mma_supported(int D, int bits, int P, int dtype, int G) {
    if (dtype != KUSH_F16 && dtype != KUSH_BF16) return 0;
    if ((D != 64 && D != 128 && D != 256) || (bits != 4 && bits != 8) || (P != 16 && P != 32)) return 0;
    return G >= 1 && G <= (D == 256 ? 8 : 16);
}

int launch_decode_mma(int D, int bits, int P, int dtype, int G, const void* q, void* out, const void* cache,
                      int64_t block_stride, int64_t head_stride, const void* tail_k, const int32_t* tail_idx,
                      const int32_t* block_table, const int32_t* seq_lens, int64_t max_pages, int32_t hkv, float scale,
                      int32_t n_splits, float* part_ml, float* part_o, int32_t n_seqs, int rot, const int32_t* order,
                      int32_t* counters, cudaStream_t stream) {
    auto go = [&](auto Dc, auto Bc, auto Pc, auto in) -> int {
        using IN = decltype(in);
        if constexpr (std::is_same_v<IN, float>) {
            return KUSH_ERR_UNSUPPORTED;
        } else if constexpr (Dc.value == 256) {
            return launch_mma<Dc.value, Bc.value, Pc.value, 1, IN>(G, q, out, cache, block_stride, head_stride, tail_k,
                                                                   tail_idx, block_table, seq_lens, max_pages, hkv,
                                                                   scale, n_splits, part_ml, part_o, n_seqs, rot, order, counters, stream);
        } else {
            if (G <= 8)
                return launch_mma<Dc.value, Bc.value, Pc.value, 1, IN>(G, q, out, cache, block_stride, head_stride,
                                                                       tail_k, tail_idx, block_table, seq_lens,
                                                                       max_pages, hkv, scale, n_splits, part_ml,
                                                                       part_o, n_seqs, rot, order, counters, stream);
            return launch_mma<Dc.value, Bc.value, Pc.value, 2, IN>(G, q, out, cache, block_stride, head_stride, tail_k,
                                                                   tail_idx, block_table, seq_lens, max_pages, hkv,
                                                                   scale, n_splits, part_ml, part_o, n_seqs, rot, order, counters, stream);
        }
    };
    return dispatch_fmt(D, bits, P, dtype, go);
}

}  // namespace kush

extern "C" int kush_sm100_device_error(int32_t clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, kush::g_decode_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v) {
        const int zero = 0;
        cudaMemcpyToSymbol(kush::g_decode_error, &zero, sizeof(int));
    }
    const int w = kush::write_error_flag(clear), gt = kush::gather_error_flag(clear);
    if (w < 0 || gt < 0) return -1;
    return (v ? 1 : 0) | (w ? 2 : 0) | (gt ? 4 : 0);
}
