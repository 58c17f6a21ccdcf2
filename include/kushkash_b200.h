/*
 * kushkash_b200.h -- C ABI of libkush_sm100.so, the sm_100a (B200) kernels of kushkash's two hot paths:
 * quantize-on-write into int4/int8 page records, and fused dequant paged decode attention.
 *
 * Each entry point replaces one GPU kernel of the reference (kushkash/kush/gpu.mojo), launched by the reference's
 * ctypes loader (kushkash/_cuda.py:92-103, Kernel.__call__) from kushkash/_ops.py.  Arguments keep the reference
 * kernel's order and meaning; what the reference fixes at compile time (head_dim, bits, q-heads-per-kv-head,
 * dtype: kushkash/_build.py:112-149 GpuConfig) and its launch grid become leading / trailing plain arguments, plus
 * the page size (16 or 32 tokens; kushkash fixes 32, kushkash/kush/quant.mojo:16).  Every pointer is a device
 * address; strides are in elements unless named *_stride in bytes (block_stride, head_stride).  The kernels run
 * on `stream` (a cudaStream_t; NULL = legacy default stream), allocate nothing and never synchronise the host.
 *
 * Return value: KUSH_OK, or a negative status; kush_sm100_last_error() then describes the failure.
 */
#ifndef KUSHKASH_B200_H
#define KUSHKASH_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KUSH_OK 0
#define KUSH_ERR_UNSUPPORTED (-1) /* head_dim / bits / page / dtype / group combination not built */
#define KUSH_ERR_ARG (-2)         /* invalid argument: null pointer, misaligned address or stride, bad size */
#define KUSH_ERR_CUDA (-3)        /* the launch failed: a CUDA error */

/* element type of q, out, k/v rows and tail_k (the reference's IN: kushkash/_build.py:28) */
#define KUSH_F16 0
#define KUSH_BF16 1
#define KUSH_F32 2

/* Message of the last failed call made on this host thread ("" if none). */
const char *kush_sm100_last_error(void);

/* Library version string. */
const char *kush_sm100_version(void);

/* Bytes of one (page, kv head) record: 2*P*DC + 4*D + 4*P, DC = D (int8) or D/2 (int4)
 * (kushkash/kush/quant.mojo:60-62, kushkash/_ops.py:29-31 record_bytes). 0 if unsupported. */
int64_t kush_sm100_record_bytes(int32_t head_dim, int32_t bits, int32_t page);

/* Decode append: one new token per sequence.  Replaces kush_append (kushkash/kush/gpu.mojo:207-238) as launched
 * by Ops.append (kushkash/_ops.py:66-80).  Row s of k_new / v_new (row strides k_stride / v_stride, head h at
 * +h*head_dim) goes to position seq_lens[s] + pos_offset (HF: 0 with advance = 1; vLLM: -1, seq_lens already
 * counting the token); negative positions are skipped.  K goes to the exact tail tail_k[tail_idx[s]][h][slot],
 * V is quantized into row `slot` of the page's record; the page's last slot quantizes its K from the tail.
 * advance != 0 stores pos + 1 into seq_lens[s].  The token's page must be mapped in block_table
 * ([n_seqs] rows, row stride max_pages). */
int kush_sm100_append(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, const void *k_new,
                      const void *v_new, int64_t k_stride, int64_t v_stride, int32_t *seq_lens, int32_t pos_offset,
                      int32_t advance, const int32_t *tail_idx, void *cache, int64_t block_stride, int64_t head_stride,
                      void *tail_k, const int32_t *block_table, int64_t max_pages, int32_t hkv, int32_t n_seqs,
                      void *stream);

/* Ragged multi-token write.  Replaces kush_write (kushkash/kush/gpu.mojo:241-276) as launched by Ops.write
 * (kushkash/_ops.py:82-101).  Sequence s owns rows [query_start_loc[s], query_start_loc[s+1]) at positions
 * ending at seq_lens[s]; job j covers logical page job_page[j] of sequence job_seq[j].  mode 0: write the page's
 * new V rows and, for a page now complete, quantize its K (older rows from the tail, newer from the new rows);
 * mode 1: copy a still-partial page's new K rows into the tail.  The reference launches mode 0 for every job,
 * then mode 1.  mode 2 does both in ONE launch (the tail stash of a sequence runs in the CTA that reads the old
 * tail, after it has read it), with the same result as mode 0 then mode 1.  A job with job_seq[j] < 0 is padding
 * and is skipped (the lists of kush_sm100_write_jobs, launched with their capacity). */
int kush_sm100_write(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, const void *k_new,
                     const void *v_new, int64_t k_stride, int64_t v_stride, const int32_t *query_start_loc,
                     const int32_t *seq_lens, const int32_t *tail_idx, const int32_t *job_seq,
                     const int32_t *job_page, int32_t mode, void *cache, int64_t block_stride, int64_t head_stride,
                     void *tail_k, const int32_t *block_table, int64_t max_pages, int32_t hkv, int32_t n_jobs,
                     void *stream);

/* Fused dequant paged decode attention.  Replaces kush_decode_tc / kush_decode (kushkash/kush/gpu.mojo:566-807,
 * 840-1040) as launched by Ops.decode (kushkash/_ops.py:191-211): out[s] ([hkv*group, head_dim], q head =
 * kv_head*group + g) = attention of q[s] over the seq_lens[s] cached tokens of sequence s, softmax scale `scale`.
 * Full pages come from the records, the last n % page tokens take K from the exact tail and V from their record.
 * n_splits > 1 (split-KV / flash-decoding): split z of (s, h) owns a contiguous page range and writes its
 * partial (M, L) to part_ml [n_seqs][hkv][n_splits][group][2] and unnormalised O to part_o
 * [n_seqs][hkv][n_splits][group][head_dim] (fp32); kush_sm100_combine then writes out.  q, out contiguous. */
int kush_sm100_decode(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, int32_t group, const void *q,
                      void *out, const void *cache, int64_t block_stride, int64_t head_stride, const void *tail_k,
                      const int32_t *tail_idx, const int32_t *block_table, const int32_t *seq_lens, int64_t max_pages,
                      int32_t hkv, float scale, int32_t n_splits, float *part_ml, float *part_o, int32_t n_seqs,
                      void *stream);

/* Size of the fixed split-KV scratch used by kush_sm100_decode_noalloc: 2M floats (8 MiB) per GPU. */
#define KUSH_NOALLOC_SCRATCH_FLOATS (1 << 21)

/* kush_sm100_decode followed, when n_splits > 1, by kush_sm100_combine, for callers that cannot allocate or pass a
 * scratch buffer (a serving engine's decode step that must not allocate, or a C FFI caller without a CUDA
 * allocator): the split partials live in a fixed 8 MiB device array inside the library, which every GPU that loads
 * the library holds until exit.  No counterpart in the reference (its decode takes a caller-allocated `work`).
 * Limit: n_seqs * hkv * n_splits * group * (head_dim + 2) <= KUSH_NOALLOC_SCRATCH_FLOATS, else KUSH_ERR_ARG.
 * The first call on each device (and on a context made again after a reset) looks up the array's device address
 * (make it before any stream capture); all calls share the array, so calls that overlap on the GPU race and must be
 * serialised by the caller.  Allocates nothing. */
int kush_sm100_decode_noalloc(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, int32_t group,
                              const void *q, void *out, const void *cache, int64_t block_stride, int64_t head_stride,
                              const void *tail_k, const int32_t *tail_idx, const int32_t *block_table,
                              const int32_t *seq_lens, int64_t max_pages, int32_t hkv, float scale, int32_t n_splits,
                              int32_t n_seqs, void *stream);

/* Split-KV merge.  Replaces kush_combine (kushkash/kush/gpu.mojo:469-491) as launched by Ops.decode
 * (kushkash/_ops.py:212-213): out = sum_z exp(M_z - M) O_z / sum_z exp(M_z - M) L_z per (s, h, g). */
int kush_sm100_combine(int32_t head_dim, int32_t dtype, int32_t group, void *out, const float *part_ml,
                       const float *part_o, int32_t n_splits, int32_t hkv, int32_t n_seqs, void *stream);

/* ---- Rotation fused into the decode step with rotation on (kushkash's default at 4 bits),
 * the reference rotates q, k, v and the output with cuBLAS GEMMs around its kernels (kushkash/_ops.py:489-518,
 * cache.py:146-183).  These entry points take the unrotated rows and apply the canonical Walsh-Hadamard rotation
 * (as kush_sm100_fwht) inside the kernels.  No counterpart kernels in the reference. */

/* kush_sm100_append of rows k_new / v_new rotated first: pages and tail bit-identical to kush_sm100_fwht (rounded
 * to dtype) followed by kush_sm100_append. */
int kush_sm100_append_rotated(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, const void *k_new,
                              const void *v_new, int64_t k_stride, int64_t v_stride, int32_t *seq_lens,
                              int32_t pos_offset, int32_t advance, const int32_t *tail_idx, void *cache,
                              int64_t block_stride, int64_t head_stride, void *tail_k, const int32_t *block_table,
                              int64_t max_pages, int32_t hkv, int32_t n_seqs, void *stream);

/* kush_sm100_decode over a rotated cache with an unrotated q: q is rotated in fp32 inside the kernel and the output
 * rotated back before its store (n_splits == 1; with n_splits > 1 follow with kush_sm100_combine_rotated). */
int kush_sm100_decode_rotated(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, int32_t group,
                              const void *q, void *out, const void *cache, int64_t block_stride, int64_t head_stride,
                              const void *tail_k, const int32_t *tail_idx, const int32_t *block_table,
                              const int32_t *seq_lens, int64_t max_pages, int32_t hkv, float scale, int32_t n_splits,
                              float *part_ml, float *part_o, int32_t n_seqs, void *stream);

/* kush_sm100_combine with the merged output rotated back before its store. */
int kush_sm100_combine_rotated(int32_t head_dim, int32_t dtype, int32_t group, void *out, const float *part_ml,
                               const float *part_o, int32_t n_splits, int32_t hkv, int32_t n_seqs, void *stream);

/* ---- Launch order of the decode.  CTA x of a decode normally works on sequence x; with ragged lengths and many waves
 * of CTAs, a long sequence that starts in the last wave sets the end of the launch.  No counterpart in the
 * reference. */

/* order[0..n_seqs) = the sequences ranked by full pages (seq_lens / page), most first; ties in any order, pages
 * above 4095 share the top rank.  One CTA; compute it once per step (the layers share seq_lens). */
int kush_sm100_order_longest_first(const int32_t *seq_lens, int32_t n_seqs, int32_t page, int32_t *order,
                                   void *stream);

#define KUSH_DECODE_ROTATE 1 /* kush_sm100_decode_ex flag: as kush_sm100_decode_rotated */

/* kush_sm100_decode with options: flags (KUSH_DECODE_ROTATE) and, if order is not NULL, CTA x working on sequence
 * order[x] (a permutation of 0..n_seqs-1, e.g. from kush_sm100_order_longest_first).  The outputs do not depend on
 * the order; the rotated tensor-core decode runs in the natural order. */
int kush_sm100_decode_ex(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, int32_t group, const void *q,
                         void *out, const void *cache, int64_t block_stride, int64_t head_stride, const void *tail_k,
                         const int32_t *tail_idx, const int32_t *block_table, const int32_t *seq_lens,
                         int64_t max_pages, int32_t hkv, float scale, int32_t n_splits, float *part_ml, float *part_o,
                         int32_t n_seqs, int32_t flags, const int32_t *order, void *stream);

/* kush_sm100_decode_ex followed by its split-KV combine, in ONE launch: the reference's two launches of a split
 * decode (kush_decode_tc then kush_combine, kushkash/_ops.py:204-211) become one.  For n_splits > 1 every CTA of
 * (sequence s, kv head h) adds 1 to counters[s * hkv + h] once its partial is in part_ml / part_o, and the last of
 * them sets the count back to 0 and merges the n_splits partials into out with the arithmetic of
 * kush_sm100_combine (or kush_sm100_combine_rotated with KUSH_DECODE_ROTATE): out equals that decode + combine bit
 * for bit.  counters: n_seqs * hkv int32, all 0 before the first call (each call leaves them 0 again).  Two launches
 * that run at the same time must not share counters.  n_splits = 1 ignores counters.  Configurations the
 * tensor-core kernel does not build (fp32, large groups) run the CUDA-core decode and kush_sm100_combine as two
 * launches. */
int kush_sm100_decode_fused_combine(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, int32_t group,
                                    const void *q, void *out, const void *cache, int64_t block_stride,
                                    int64_t head_stride, const void *tail_k, const int32_t *tail_idx,
                                    const int32_t *block_table, const int32_t *seq_lens, int64_t max_pages,
                                    int32_t hkv, float scale, int32_t n_splits, float *part_ml, float *part_o,
                                    int32_t *counters, int32_t n_seqs, int32_t flags, const int32_t *order,
                                    void *stream);

/* Which decode kernel a configuration takes: 1 = tensor-core kernel (mma), 0 = CUDA-core kernel,
 * KUSH_ERR_UNSUPPORTED if neither is built.  Mirrors GpuConfig.tensor_cores (kushkash/_build.py:120-122). */
int kush_sm100_decode_tensor_cores(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, int32_t group);

/* Bounded-wait watchdog of the kernels that wait: bit 0 set if a decode launch gave up waiting for a page copy (its
 * outputs were written as NaN), bit 1 if a bulk write gave up waiting for its input rows (the records of that
 * warp's remaining items were not written), bit 2 if a peer-gather wait gave up on a peer (kush_sm100_gather_wait:
 * the gathered outputs are incomplete); 0 if none.  clear != 0 resets the flags.
 * Synchronous (reads device variables); -1 on a CUDA error.  No counterpart in the reference, whose kernels have
 * no bounded waits. */
int kush_sm100_device_error(int32_t clear);

/* Exhaustive self-check of the bulk write's scale arithmetic on the current device: mismatches[0] / [1] = fp32
 * values d in [2^-100, 2^100] for which the write's d / 15 / d / 255 (Markstein's correction step, scalar and
 * fp32x2 forms) differs from the IEEE quotient, mismatches[2] = fp16 scales whose reciprocal (hardware
 * approximation plus one Newton step) differs from the IEEE reciprocal.  All three are 0 on a correct build.
 * Synchronous; allocates 24 bytes of device memory.  No counterpart in the reference (a diagnostic of this
 * implementation's arithmetic). */
int kush_sm100_selfcheck(uint64_t *mismatches);

/* Canonical Walsh-Hadamard rotation of `rows` rows of head_dim values: y[r] = fwht(x[r]) (row strides in
 * elements; y may alias x).  Replaces kush_fwht (kushkash/kush/gpu.mojo:95-112) as launched by Ops.fwht
 * (kushkash/_ops.py:104-127): fp32 butterflies over strides 1, 2, ..., D/2 in that order, then one multiply by
 * fp32 1/sqrt(D) (kushkash/kush/quant.mojo:90-122), bit-identical to the CPU. */
int kush_sm100_fwht(int32_t head_dim, int32_t dtype, const void *x, void *y, int64_t x_stride, int64_t y_stride,
                    int64_t rows, void *stream);

/* Packed-prefill unpack.  Replaces kush_unpack (kushkash/kush/gpu.mojo:303-375) as launched by Ops.unpack
 * (kushkash/_ops.py:129-179): full history pages (block page_blk[i] -> rows page_dst[i] + t), partial pages
 * (block tail_blk[i], tail_info[3i..3i+2] = (first row, tokens, tail slot): K from tail_k, V from the record)
 * and new rows (row j of k_new / v_new -> row new_dst[j]) into kp / vp ([rows][hkv][head_dim]).  History is
 * dequantized as fma(code, scale, bias) in fp32, optionally rotated back (rot != 0), rounded once to dtype.
 * Entries with page_blk[i] < 0, tail_blk[i] < 0 or new_dst[j] < 0 are padding and are skipped (the plans of
 * kush_sm100_unpack_plan, launched with their capacities). */
int kush_sm100_unpack(int32_t head_dim, int32_t bits, int32_t page, int32_t dtype, const void *cache,
                      int64_t block_stride, int64_t head_stride, int32_t hkv, const int32_t *page_blk,
                      const int32_t *page_dst, int32_t n_pages, const int32_t *tail_blk, const int32_t *tail_info,
                      int32_t n_tail, const void *tail_k, const void *k_new, const void *v_new, int64_t k_stride,
                      int64_t v_stride, const int32_t *new_dst, int32_t n_new, void *kp, void *vp, int32_t rot,
                      void *stream);

/* The write jobs of a step, built on the device.  Replaces the per-step host lists of kushkash's serving backends
 * (kushkash/vllm/backend.py:434-447 _prefill_host, kushkash/sglang/backend.py:255, both over kushkash/_ops.py:343-344
 * pages_touched, uploaded through the pinned ring of vllm/backend.py:283-312): sequence s, with rows
 * [query_start_loc[s], query_start_loc[s+1]) ending at position seq_lens[s], gets one job per logical page its rows
 * touch, ctx / page .. (seq_lens[s] - 1) / page with ctx = seq_lens[s] - its rows, in sequence then page order (the
 * reference's order).  job_seq / job_page hold max_jobs entries: the jobs, then padding (job_seq = -1) that
 * kush_sm100_write skips, so the write can be launched with n_jobs = max_jobs without the count coming back to the
 * host.  *n_jobs (device) = the number of jobs (more than max_jobs means the lists were cut).  max_jobs >= rows /
 * page + 2 * n_seqs always suffices.  One CTA; no host synchronisation, capture-safe. */
int kush_sm100_write_jobs(const int32_t *query_start_loc, const int32_t *seq_lens, int32_t n_seqs, int32_t page,
                          int32_t *job_seq, int32_t *job_page, int32_t max_jobs, int32_t *n_jobs, void *stream);

/* The packed-prefill plan of kush_sm100_unpack for a step, built on the device.  Replaces the host-side plans of
 * kushkash's serving backends (kushkash/sglang/backend.py:90-110, kushkash/vllm/backend.py:388-413) for a layout that
 * packs every sequence's history and new rows together: sequence s at rows [kv_start[s], kv_start[s+1]) (kv_start
 * [n_seqs + 1], the cu_seqlens of a varlen attention), history (ctx = seq_lens[s] - its new rows) first.  Full
 * history pages -> page_blk / page_dst, the partial history page -> tail_blk / tail_info (first row, tokens,
 * tail_idx[s]), new row j of the step -> new_dst[j].  Each list is filled to its capacity with padding that
 * kush_sm100_unpack skips.  counts[4] (device) = full pages, partial pages, new rows, packed rows.  One CTA; no
 * host synchronisation, capture-safe. */
int kush_sm100_unpack_plan(const int32_t *query_start_loc, const int32_t *seq_lens, const int32_t *tail_idx,
                           const int32_t *block_table, int64_t max_pages, int32_t n_seqs, int32_t page,
                           int32_t *kv_start, int32_t *page_blk, int32_t *page_dst, int32_t max_page_entries,
                           int32_t *tail_blk, int32_t *tail_info, int32_t max_tail_entries, int32_t *new_dst,
                           int32_t max_new, int32_t *counts, void *stream);

/* ---- Output gather of KV-head sharding over peer memory (one process per GPU, CUDA IPC over NVLink).
 * Replaces the library all_gather that follows the sharded decode (kushkash_b200/shard.py gather_heads; the
 * reference has no multi-GPU path of its own, its tensor parallelism is vLLM's).  No counterpart in the reference. */

#define KUSH_IPC_HANDLE_BYTES 64

/* cudaMalloc of `bytes`, zero-filled: memory other processes can map with kush_sm100_ipc_open.  Synchronous. */
int kush_sm100_ipc_alloc(int64_t bytes, void **ptr);
int kush_sm100_ipc_free(void *ptr);
/* The KUSH_IPC_HANDLE_BYTES-byte handle of an allocation made by kush_sm100_ipc_alloc (cudaIpcGetMemHandle). */
int kush_sm100_ipc_handle(const void *ptr, uint8_t *handle);
/* Map a peer's allocation from its handle (cudaIpcOpenMemHandle, peer access enabled lazily); close unmaps it. */
int kush_sm100_ipc_open(const uint8_t *handle, void **ptr);
int kush_sm100_ipc_close(void *ptr);

/* Split-KV combine of this rank's kv heads (as kush_sm100_combine) whose results are stored into every rank's
 * gathered output: outs is a device array of `world` pointers, outs[r] = rank r's [n_seqs][hkv*world*group]
 * [head_dim] buffer (this rank's own buffer at outs[rank]); this rank's heads land at q heads
 * [rank*hkv*group, (rank+1)*hkv*group).  After the last store, ctr[1] (this rank's gather count) is incremented and
 * written with release semantics to flags[r][rank] of every rank r (flags: device array of `world` pointers to each
 * rank's [world] uint32 counts).  ctr ([2] uint32, zero-initialised, this rank's memory) also counts the launch's
 * finished blocks.  Every rank must run the same sequence of gathers. */
int kush_sm100_combine_gather(int32_t head_dim, int32_t dtype, int32_t group, void *const *outs, int32_t rank,
                              int32_t world, const float *part_ml, const float *part_o, int32_t n_splits, int32_t hkv,
                              int32_t n_seqs, uint32_t *const *flags, uint32_t *ctr, void *stream);

/* One warp that waits until every rank's count in this rank's flags[world] has reached ctr[1] (this rank's own
 * count, set by its kush_sm100_combine_gather earlier on `stream`): after it, the gathered output of that gather is
 * complete for the kernels that follow on `stream`.  The wait gives up after 2 s and sets bit 2 of
 * kush_sm100_device_error. */
int kush_sm100_gather_wait(const uint32_t *flags, int32_t world, const uint32_t *ctr, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* KUSHKASH_B200_H */
