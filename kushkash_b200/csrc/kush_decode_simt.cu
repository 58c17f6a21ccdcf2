// Fused dequant paged decode attention on the CUDA cores (fp32 arithmetic), and the split-KV combine.
//
// This kernel serves the configurations the tensor-core kernel (kush_decode_mma.cu) does not take: fp32 inputs
// (where callers expect fp32-level agreement) and very large GQA groups.  It computes exactly the algebra of the
// reference (kushkash/kush/gpu.mojo:20-23, CPU restatement kushkash/kush/cpu.mojo:320-451): per page, the K scale
// folds into q and the K bias into one scalar per head; V scales fold into the softmax weights and V biases into
// one scalar per head; page-granular online softmax; the last n % P tokens take K from the exact tail.
//
// grid (S, Hkv, n_splits), block NW warps.  Split z owns a contiguous page range (split_range: a quota of pages per
// split for the whole batch); warp w takes pages start + w, start + w + NW, ...; the warp that would take the next
// page also takes the tail (the last split with pages only).  Per page: lane t = token t for the QK dots (q' broadcast from shared memory), lane = output
// dims for the PV accumulation (accumulators in shared memory, G*D floats per warp).
#include "kush_common.cuh"

namespace kush {

constexpr int SIMT_NW = 4;

template <int D, int BITS, int P, class IN>
__global__ void __launch_bounds__(SIMT_NW * WARP) decode_simt_kernel(
    const IN* __restrict__ q, IN* __restrict__ out, const uint8_t* __restrict__ cache, int64_t block_stride,
    int64_t head_stride, const IN* __restrict__ tail_k, const int32_t* __restrict__ tail_idx,
    const int32_t* __restrict__ block_table, const int32_t* __restrict__ seq_lens, int64_t max_pages, int H, int G,
    float sm, int n_splits, float* __restrict__ part_ml, float* __restrict__ part_o, int rot,
    const int32_t* __restrict__ order) {
    using F = Fmt<D, BITS, P>;
    constexpr int NW = SIMT_NW;
    pdl_wait();                                            // previous kernel on the stream done
    constexpr int R = D / WARP;
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    float* qsm = smem;                                     // [G][D] q * sm
    float* qs_all = qsm + G * D;                           // [NW][G][D] q * sm * k_scale of the warp's page
    float* acc_all = qs_all + NW * G * D;                  // [NW][G][D] unnormalised output
    float* w_all = acc_all + NW * G * D;                   // [NW][G][P] scores -> weights
    float* st_all = w_all + NW * G * P;                    // [NW][3][G] m, l, vbacc

    const int s = order ? order[blockIdx.x] : blockIdx.x, h = blockIdx.y, z = blockIdx.z;    // launch order
    const int wid = threadIdx.x / WARP, lane = threadIdx.x % WARP;
    const int64_t n = seq_lens[s];
    const int tail_n = int(n % P);
    const int64_t full = n / P;
    const SplitRange sr = split_range(seq_lens, int(gridDim.x), s, z, n_splits, P);
    if (!sr.active) {                                      // no pages here: an empty partial
        for (int g = threadIdx.x; g < G; g += NW * WARP) {
            const int64_t pb = ((int64_t(s) * H + h) * n_splits + z) * G + g;
            part_ml[pb * 2] = -INFINITY;
            part_ml[pb * 2 + 1] = 0.0f;
        }
        return;
    }
    const int64_t p0 = sr.p0, p1 = sr.p1;
    const int32_t* bt = block_table + s * max_pages;
    const int64_t qbase = (int64_t(s) * H + h) * G * D;

    for (int i = threadIdx.x; i < G * D; i += NW * WARP) qsm[i] = rot ? to_f32(q[qbase + i]) : to_f32(q[qbase + i]) * sm;
    if (rot) {                                             // q rotated in fp32 (canonical FWHT), then scaled
        __syncthreads();
        for (int g = wid; g < G; g += NW) {
            float x[R];
#pragma unroll
            for (int i = 0; i < R; i++) x[i] = qsm[g * D + lane + WARP * i];
            fwht_warp<D>(x, lane);
#pragma unroll
            for (int i = 0; i < R; i++) qsm[g * D + lane + WARP * i] = x[i] * sm;
        }
    }
    float* qs = qs_all + wid * G * D;
    float* acc = acc_all + wid * G * D;
    float* wt = w_all + wid * G * P;
    float* m = st_all + wid * 3 * G;
    float* l = m + G;
    float* vb = l + G;
    for (int i = lane; i < G * D; i += WARP) acc[i] = 0.0f;
    for (int g = lane; g < G; g += WARP) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
        vb[g] = 0.0f;
    }
    __syncthreads();

    // online-softmax step of head g over cnt scores held by lanes t < cnt (score x); returns the weight of lane t
    auto softmax_step = [&](int g, float x, int cnt) -> float {
        const bool valid = lane < cnt;
        const float mo = m[g];
        const float mn = fmaxf(mo, warp_max(valid ? x : -INFINITY));
        const float corr = __expf(mo - mn);
        const float e = valid ? __expf(x - mn) : 0.0f;
        const float tot = warp_sum(e);
        __syncwarp();
        if (lane == 0) {
            m[g] = mn;
            l[g] = l[g] * corr + tot;
            vb[g] *= corr;
        }
        for (int d = lane; d < D; d += WARP) acc[g * D + d] *= corr;
        return e;
    };

    auto v_accumulate = [&](const uint8_t* rec, int cnt) {
        // V phase: lane = dims lane + 32i; weights already hold p * vs_t; V bias into vb[g]
#pragma unroll
        for (int i = 0; i < R; i++) {
            const int d = lane + WARP * i;
            for (int t = 0; t < cnt; t++) {
                const float c = float(code_at<D, BITS>(rec + F::OFF_VQ + t * F::DC, d));
                for (int g = 0; g < G; g++) acc[g * D + d] += wt[g * P + t] * c;
            }
        }
    };

    for (int64_t lp = p0 + wid; lp < p1; lp += NW) {
        const uint8_t* rec = cache + int64_t(bt[lp]) * block_stride + int64_t(h) * head_stride;
        // 1. fold the page's K scale into q, K bias into one scalar per head
        for (int g = 0; g < G; g++) {
            float kbias = 0.0f;
            for (int d = lane; d < D; d += WARP) {
                const float qv = qsm[g * D + d];
                qs[g * D + d] = qv * h_load(rec + F::OFF_KS, d);
                kbias += qv * h_load(rec + F::OFF_KB, d);
            }
            kbias = warp_sum(kbias);
            __syncwarp();
            // 2. scores: lane t = token t
            float x = 0.0f;
            if (lane < P) {
                const uint8_t* row = rec + lane * F::DC;
                for (int d = 0; d < D; d++) x += qs[g * D + d] * float(code_at<D, BITS>(row, d));
                x += kbias;
            }
            // 3. page-granular online softmax
            const float e = softmax_step(g, x, P);
            const float vst = lane < P ? h_load(rec + F::OFF_VS, lane) : 0.0f;
            const float vbt = lane < P ? h_load(rec + F::OFF_VB, lane) : 0.0f;
            const float vbsum = warp_sum(e * vbt);
            if (lane < P) wt[g * P + lane] = e * vst;
            if (lane == 0) vb[g] += vbsum;
            __syncwarp();
        }
        __syncwarp();
        v_accumulate(rec, P);
        __syncwarp();
    }
    // tail page: last split, the warp that would take the next page (kushkash/kush/gpu.mojo:1001-1028)
    const int64_t npg = max(int64_t(0), p1 - p0);
    if (tail_n > 0 && sr.last && wid == int(npg % NW)) {
        const IN* tk = tail_k + (int64_t(tail_idx[s]) * H + h) * P * D;
        const uint8_t* trec = cache + int64_t(bt[full]) * block_stride + int64_t(h) * head_stride;
        for (int g = 0; g < G; g++) {
            float x = 0.0f;
            if (lane < tail_n)
                for (int d = 0; d < D; d++) x += qsm[g * D + d] * to_f32(tk[lane * D + d]);
            const float e = softmax_step(g, x, tail_n);
            const float vst = lane < tail_n ? h_load(trec + F::OFF_VS, lane) : 0.0f;
            const float vbt = lane < tail_n ? h_load(trec + F::OFF_VB, lane) : 0.0f;
            const float vbsum = warp_sum(e * vbt);
            if (lane < P) wt[g * P + lane] = lane < tail_n ? e * vst : 0.0f;
            if (lane == 0) vb[g] += vbsum;
            __syncwarp();
        }
        v_accumulate(trec, tail_n);
        __syncwarp();
    }
    __syncthreads();

    // merge the warps (kushkash/kush/gpu.mojo:438-466 _merge_store): acc + vbacc per warp, rescaled to the max
    for (int idx = threadIdx.x; idx < G * D; idx += NW * WARP) {
        const int g = idx / D, d = idx % D;
        float M = -INFINITY;
        for (int w = 0; w < NW; w++) M = fmaxf(M, st_all[w * 3 * G + g]);
        float L = 0.0f, o = 0.0f;
        if (M > -INFINITY) {
            for (int w = 0; w < NW; w++) {
                const float mw = st_all[w * 3 * G + g];
                if (mw > -INFINITY) {
                    const float f = __expf(mw - M);
                    L += st_all[w * 3 * G + G + g] * f;
                    o += f * (acc_all[(w * G + g) * D + d] + st_all[w * 3 * G + 2 * G + g]);
                }
            }
        }
        if (n_splits == 1) {
            if (rot) qsm[idx] = L > 0.0f ? o / L : 0.0f;                // rotated back below
            else out[qbase + idx] = from_f32<IN>(L > 0.0f ? o / L : 0.0f);
        } else {
            const int64_t pb = ((int64_t(s) * H + h) * n_splits + z) * G + g;
            part_o[pb * D + d] = o;
            if (d == 0) {
                part_ml[pb * 2] = M;
                part_ml[pb * 2 + 1] = L;
            }
        }
    }
    if (rot && n_splits == 1) {                            // the output rotated back (canonical FWHT), a warp per head
        __syncthreads();
        for (int g = wid; g < G; g += NW) {
            float x[R];
#pragma unroll
            for (int i = 0; i < R; i++) x[i] = qsm[g * D + lane + WARP * i];
            fwht_warp<D>(x, lane);
#pragma unroll
            for (int i = 0; i < R; i++) out[qbase + g * D + lane + WARP * i] = from_f32<IN>(x[i]);
        }
    }
}

// grid (S * Hkv * G), block D: merge the split-K partials of one (sequence, kv head, q head); thread d owns output
// dim d (kushkash/kush/gpu.mojo:469-491 kush_combine, with one block per q head so long split lists run in parallel)
template <class IN>
__global__ void __launch_bounds__(256) combine_kernel(IN* __restrict__ out, const float* __restrict__ part_ml,
                                                      const float* __restrict__ part_o, int n_splits, int G, int D) {
    pdl_wait();                                            // previous kernel on the stream done
    const int64_t sh = blockIdx.x / G, g = blockIdx.x % G;
    const int d = threadIdx.x;
    const float* ml = part_ml + (sh * n_splits * G + g) * 2;     // split z at ml[2 z G]
    const float* po = part_o + (sh * n_splits * G + g) * D + d;  // split z at po[z G D]
    out[(sh * G + g) * D + d] = from_f32<IN>(merge_splits(ml, po, n_splits, G, D));
}

// combine_kernel with the merged output rotated back (canonical FWHT) before its store: the row of D values goes
// through shared memory to one warp
template <int D, class IN>
__global__ void __launch_bounds__(D) combine_rot_kernel(IN* __restrict__ out, const float* __restrict__ part_ml,
                                                        const float* __restrict__ part_o, int n_splits, int G) {
    __shared__ float row[D];
    pdl_wait();                                            // previous kernel on the stream done

    const int64_t sh = blockIdx.x / G, g = blockIdx.x % G;
    const int d = threadIdx.x;
    const float* ml = part_ml + (sh * n_splits * G + g) * 2;
    const float* po = part_o + (sh * n_splits * G + g) * D + d;
    row[d] = merge_splits(ml, po, n_splits, G, D);
    __syncthreads();
    if (d < WARP) {
        float x[D / WARP];
#pragma unroll
        for (int i = 0; i < D / WARP; i++) x[i] = row[d + WARP * i];
        fwht_warp<D>(x, d);
#pragma unroll
        for (int i = 0; i < D / WARP; i++) out[(sh * G + g) * D + d + WARP * i] = from_f32<IN>(x[i]);
    }
}

template <int D, int BITS, int P, class IN>
int launch_decode_simt(const void* q, void* out, const void* cache, int64_t block_stride, int64_t head_stride,
                       const void* tail_k, const int32_t* tail_idx, const int32_t* block_table, const int32_t* seq_lens,
                       int64_t max_pages, int32_t hkv, int32_t G, float scale, int32_t n_splits, float* part_ml,
                       float* part_o, int32_t n_seqs, int rot, const int32_t* order, cudaStream_t stream) {
    constexpr int NW = SIMT_NW;
    const size_t smem = sizeof(float) * (size_t(G) * D + 2 * size_t(NW) * G * D + size_t(NW) * G * P + 3 * size_t(NW) * G);
    if (smem > 200 * 1024) return set_error(KUSH_ERR_UNSUPPORTED, "decode: group %d too large for head_dim %d", G, D);
    auto kern = decode_simt_kernel<D, BITS, P, IN>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    dim3 grid(n_seqs, hkv, n_splits);
    launch_pdl(kern, grid, dim3(NW * WARP), smem, stream, static_cast<const IN*>(q), static_cast<IN*>(out),
               static_cast<const uint8_t*>(cache), block_stride, head_stride, static_cast<const IN*>(tail_k), tail_idx,
               block_table, seq_lens, max_pages, hkv, G, scale, n_splits, part_ml, part_o, rot, order);
    return check_launch("kush_sm100_decode (cuda cores)");
}

template <class IN>
int launch_combine(void* out, const float* part_ml, const float* part_o, int32_t n_splits, int32_t hkv, int32_t G,
                   int32_t D, int32_t n_seqs, cudaStream_t stream) {
    const int64_t blocks = int64_t(n_seqs) * hkv * G;
    if (blocks > 0x7fffffff) return set_error(KUSH_ERR_ARG, "kush_sm100_combine: grid too large");
    launch_pdl(combine_kernel<IN>, dim3(unsigned(blocks)), dim3(D), 0, stream, static_cast<IN*>(out), part_ml, part_o,
               n_splits, G, D);
    return check_launch("kush_sm100_combine");
}

int launch_decode_simt_any(int D, int bits, int P, int dtype, int G, const void* q, void* out, const void* cache,
                           int64_t block_stride, int64_t head_stride, const void* tail_k, const int32_t* tail_idx,
                           const int32_t* block_table, const int32_t* seq_lens, int64_t max_pages, int32_t hkv,
                           float scale, int32_t n_splits, float* part_ml, float* part_o, int32_t n_seqs, int rot,
                           const int32_t* order, cudaStream_t stream) {
    return dispatch_fmt(D, bits, P, dtype, [&](auto Dc, auto Bc, auto Pc, auto in) {
        return launch_decode_simt<Dc.value, Bc.value, Pc.value, decltype(in)>(
            q, out, cache, block_stride, head_stride, tail_k, tail_idx, block_table, seq_lens, max_pages, hkv, G,
            scale, n_splits, part_ml, part_o, n_seqs, rot, order, stream);
    });
}

}  // namespace kush

using namespace kush;

extern "C" int kush_sm100_combine_rotated(int32_t head_dim, int32_t dtype, int32_t group, void* out,
                                          const float* part_ml, const float* part_o, int32_t n_splits, int32_t hkv,
                                          int32_t n_seqs, void* stream) {
    if (n_seqs < 0 || hkv < 1 || group < 1 || n_splits < 1)
        return set_error(KUSH_ERR_ARG, "kush_sm100_combine_rotated: n_seqs %d hkv %d group %d n_splits %d", n_seqs, hkv,
                         group, n_splits);
    if (n_seqs == 0) return KUSH_OK;
    if (!out || !part_ml || !part_o) return set_error(KUSH_ERR_ARG, "kush_sm100_combine_rotated: null pointer");
    const int64_t blocks = int64_t(n_seqs) * hkv * group;
    if (blocks > 0x7fffffff) return set_error(KUSH_ERR_ARG, "kush_sm100_combine_rotated: grid too large");
    int rc = dispatch_dim(head_dim, [&](auto D) {
        return dispatch_dtype(dtype, [&](auto in) {
            using IN = decltype(in);
            launch_pdl(combine_rot_kernel<D.value, IN>, dim3(unsigned(blocks)), dim3(D.value), 0,
                       static_cast<cudaStream_t>(stream), static_cast<IN*>(out), part_ml, part_o, n_splits, group);
            return check_launch("kush_sm100_combine_rotated");
        });
    });
    if (rc == KUSH_ERR_UNSUPPORTED)
        return set_error(rc, "kush_sm100_combine_rotated: head_dim %d / dtype %d", head_dim, dtype);
    return rc;
}

extern "C" int kush_sm100_combine(int32_t head_dim, int32_t dtype, int32_t group, void* out, const float* part_ml,
                                  const float* part_o, int32_t n_splits, int32_t hkv, int32_t n_seqs, void* stream) {
    if (n_seqs < 0 || hkv < 1 || group < 1 || n_splits < 1)
        return set_error(KUSH_ERR_ARG, "kush_sm100_combine: n_seqs %d hkv %d group %d n_splits %d", n_seqs, hkv, group,
                         n_splits);
    if (n_seqs == 0) return KUSH_OK;
    if (!out || !part_ml || !part_o) return set_error(KUSH_ERR_ARG, "kush_sm100_combine: null pointer");
    if (head_dim != 64 && head_dim != 128 && head_dim != 256)
        return set_error(KUSH_ERR_UNSUPPORTED, "kush_sm100_combine: head_dim %d", head_dim);
    int rc = dispatch_dtype(dtype, [&](auto in) {
        return launch_combine<decltype(in)>(out, part_ml, part_o, n_splits, hkv, group, head_dim, n_seqs,
                                            static_cast<cudaStream_t>(stream));
    });
    if (rc == KUSH_ERR_UNSUPPORTED) return set_error(rc, "kush_sm100_combine: dtype %d", dtype);
    return rc;
}
