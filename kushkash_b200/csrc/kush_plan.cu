// Per-step metadata of the ragged write and of the prefill with history, built on the device.
//
// kushkash's serving backends build these lists on the host every step (numpy) and upload them through a pinned
// ring: the write jobs, one per (sequence, logical page touched) -- kushkash/vllm/backend.py:434-447 and
// kushkash/sglang/backend.py:255 over kushkash/_ops.py:343-344 pages_touched -- and the packed-prefill plan of the
// unpack -- kushkash/sglang/backend.py:90-110, vllm/backend.py:388-413.  Here one small kernel derives them from
// the device-resident query_start_loc / seq_lens / block table of the step, so a step needs no host work, no
// host->device copy and no synchronisation, and the builders can sit inside a captured step graph.  Output arrays
// have a capacity fixed by the caller (an upper bound it knows on the host); the entries past the real count are
// padding (job_seq, page_blk, tail_blk, new_dst = -1) that kush_sm100_write and kush_sm100_unpack skip, so those can
// be launched with the capacity.  The real counts are also written to device memory.
#include "kush_common.cuh"

namespace kush {

constexpr int PLAN_THREADS = 1024;

// exclusive scan of one int per thread over the CTA; returns this thread's offset, *total gets the CTA's sum
__device__ __forceinline__ int64_t block_exclusive_scan(int64_t x, int64_t* warp_sums, int64_t* total) {
    const int lane = threadIdx.x % WARP, w = threadIdx.x / WARP, nw = blockDim.x / WARP;
    int64_t incl = x;
#pragma unroll
    for (int o = 1; o < WARP; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == WARP - 1) warp_sums[w] = incl;
    __syncthreads();
    if (w == 0) {
        int64_t v = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < WARP; o <<= 1) {
            const int64_t y = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += y;
        }
        if (lane < nw) warp_sums[lane] = v;                // inclusive prefix of the warp sums
    }
    __syncthreads();
    const int64_t before = w ? warp_sums[w - 1] : 0;
    *total = warp_sums[nw - 1];
    __syncthreads();                                       // warp_sums free for the next round
    return before + incl - x;
}

// One CTA, 1024 sequences at a time: a scan gives each sequence's first job, then every warp fills the jobs of
// its sequences with its lanes.  Sequence s has rows [qsl[s], qsl[s+1]) ending at position seq_lens[s] (ctx =
// seq_lens[s] - its rows): its jobs are its logical pages ctx / P .. (seq_lens[s] - 1) / P when it has rows, in
// sequence order then page order -- the order and content of the reference's list over pages_touched
// (kushkash/_ops.py:343-344).  A sequence with more rows than positions (ctx < 0) gets no jobs.
__global__ void __launch_bounds__(PLAN_THREADS) write_jobs_kernel(const int32_t* __restrict__ qsl,
                                                                 const int32_t* __restrict__ seq_lens, int n_seqs,
                                                                 int P, int32_t* __restrict__ job_seq,
                                                                 int32_t* __restrict__ job_page, int max_jobs,
                                                                 int32_t* __restrict__ n_jobs) {
    __shared__ int64_t warp_sums[PLAN_THREADS / WARP];
    __shared__ int64_t c_off[PLAN_THREADS];
    __shared__ int32_t c_cnt[PLAN_THREADS], c_first[PLAN_THREADS];
    pdl_wait();
    const int lane = threadIdx.x % WARP, w = threadIdx.x / WARP;
    int64_t carry = 0;
    for (int base = 0; base < n_seqs; base += blockDim.x) {
        const int s = base + threadIdx.x;
        int64_t cnt = 0, first = 0;
        if (s < n_seqs) {
            const int64_t total = seq_lens[s], ctx = total - (int64_t(qsl[s + 1]) - qsl[s]);
            if (total > ctx && ctx >= 0) {
                first = ctx / P;
                cnt = (total - 1) / P - first + 1;
            }
        }
        int64_t sum;
        c_off[threadIdx.x] = carry + block_exclusive_scan(cnt, warp_sums, &sum);
        c_cnt[threadIdx.x] = int32_t(cnt);
        c_first[threadIdx.x] = int32_t(first);
        __syncthreads();
        for (int k = w; k < PLAN_THREADS && base + k < n_seqs; k += PLAN_THREADS / WARP) {
            const int64_t off = c_off[k];
            for (int i = lane; i < c_cnt[k] && off + i < max_jobs; i += WARP) {
                job_seq[off + i] = base + k;
                job_page[off + i] = c_first[k] + i;
            }
        }
        __syncthreads();
        carry += sum;
    }
    for (int64_t i = carry + threadIdx.x; i < max_jobs; i += blockDim.x) {
        job_seq[i] = -1;
        job_page[i] = 0;
    }
    if (threadIdx.x == 0) *n_jobs = int32_t(min(carry, int64_t(0x7fffffff)));
}

// One CTA, 1024 sequences at a time (scan, then the warps fill their sequences' entries with their lanes).  The
// prefill-with-history layout of kush_sm100_unpack: sequence s packed at rows [kv_start[s], kv_start[s+1]),
// kv_start[s] = sum of seq_lens before s -- its history (ctx = seq_lens[s] - its new rows) first, then its new
// rows.  Full history pages p < ctx / P: page_blk = block_table[s][p], page_dst = kv_start[s] + p P; a partial
// history page (ctx % P tokens): tail_blk = block_table[s][ctx / P], tail_info = (kv_start[s] + (ctx / P) P,
// ctx % P, tail_idx[s]); new row j of the step: new_dst[j] = kv_start[s] + ctx + (j - qsl[s]).
// counts = (full pages, partial pages, new rows, packed rows).
__global__ void __launch_bounds__(PLAN_THREADS) unpack_plan_kernel(
    const int32_t* __restrict__ qsl, const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ tail_idx,
    const int32_t* __restrict__ block_table, int64_t max_pages, int n_seqs, int P, int32_t* __restrict__ kv_start,
    int32_t* __restrict__ page_blk, int32_t* __restrict__ page_dst, int max_page_entries,
    int32_t* __restrict__ tail_blk, int32_t* __restrict__ tail_info, int max_tail_entries,
    int32_t* __restrict__ new_dst, int max_new, int32_t* __restrict__ counts) {
    __shared__ int64_t warp_sums[PLAN_THREADS / WARP];
    __shared__ int64_t c_op[PLAN_THREADS], c_row[PLAN_THREADS];
    __shared__ int32_t c_ctx[PLAN_THREADS], c_q0[PLAN_THREADS], c_new[PLAN_THREADS];
    pdl_wait();
    const int lane = threadIdx.x % WARP, w = threadIdx.x / WARP;
    int64_t c_pages = 0, c_tail = 0, c_rows = 0;
    for (int base = 0; base < n_seqs; base += blockDim.x) {
        const int s = base + threadIdx.x;
        int64_t total = 0, ctx = 0, q0 = 0;
        if (s < n_seqs) {
            total = seq_lens[s];
            q0 = qsl[s];
            ctx = max(int64_t(0), total - (int64_t(qsl[s + 1]) - q0));
        }
        const int64_t full = ctx / P, part = ctx % P ? 1 : 0;
        int64_t sp, st, sr;
        const int64_t op = c_pages + block_exclusive_scan(full, warp_sums, &sp);
        const int64_t ot = c_tail + block_exclusive_scan(part, warp_sums, &st);
        const int64_t orow = c_rows + block_exclusive_scan(total, warp_sums, &sr);
        c_op[threadIdx.x] = op;
        c_row[threadIdx.x] = orow;
        c_ctx[threadIdx.x] = int32_t(ctx);
        c_q0[threadIdx.x] = int32_t(q0);
        c_new[threadIdx.x] = int32_t(total - ctx);
        if (s < n_seqs) {
            kv_start[s] = int32_t(orow);
            if (part && ot < max_tail_entries) {
                tail_blk[ot] = block_table[int64_t(s) * max_pages + full];
                tail_info[3 * ot] = int32_t(orow + full * P);
                tail_info[3 * ot + 1] = int32_t(ctx % P);
                tail_info[3 * ot + 2] = tail_idx[s];
            }
        }
        __syncthreads();
        for (int k = w; k < PLAN_THREADS && base + k < n_seqs; k += PLAN_THREADS / WARP) {
            const int32_t* bt = block_table + int64_t(base + k) * max_pages;
            const int64_t o = c_op[k], r = c_row[k];
            const int nfull = c_ctx[k] / P;
            for (int p = lane; p < nfull && o + p < max_page_entries; p += WARP) {
                page_blk[o + p] = bt[p];
                page_dst[o + p] = int32_t(r + int64_t(p) * P);
            }
            for (int t = lane; t < c_new[k] && int64_t(c_q0[k]) + t < max_new; t += WARP)
                new_dst[c_q0[k] + t] = int32_t(r + c_ctx[k] + t);
        }
        __syncthreads();
        c_pages += sp;
        c_tail += st;
        c_rows += sr;
    }
    for (int64_t i = c_pages + threadIdx.x; i < max_page_entries; i += blockDim.x) {
        page_blk[i] = -1;
        page_dst[i] = 0;
    }
    for (int64_t i = c_tail + threadIdx.x; i < max_tail_entries; i += blockDim.x) {
        tail_blk[i] = -1;
        tail_info[3 * i] = tail_info[3 * i + 1] = tail_info[3 * i + 2] = 0;
    }
    const int64_t last = n_seqs > 0 ? qsl[n_seqs] : 0;    // new rows past the step's: padding
    for (int64_t j = last + threadIdx.x; j < max_new; j += blockDim.x) new_dst[j] = -1;
    if (threadIdx.x == 0) {
        kv_start[n_seqs] = int32_t(c_rows);
        counts[0] = int32_t(c_pages);
        counts[1] = int32_t(c_tail);
        counts[2] = n_seqs > 0 ? qsl[n_seqs] - qsl[0] : 0;
        counts[3] = int32_t(c_rows);
    }
}

}  // namespace kush

using namespace kush;

extern "C" int kush_sm100_write_jobs(const int32_t* query_start_loc, const int32_t* seq_lens, int32_t n_seqs,
                                     int32_t page, int32_t* job_seq, int32_t* job_page, int32_t max_jobs,
                                     int32_t* n_jobs, void* stream) {
    if (n_seqs < 0 || max_jobs < 0 || (page != 16 && page != 32))
        return set_error(KUSH_ERR_ARG, "kush_sm100_write_jobs: n_seqs %d, max_jobs %d, page %d", n_seqs, max_jobs, page);
    if (!query_start_loc || !seq_lens || !n_jobs || (max_jobs > 0 && (!job_seq || !job_page)))
        return set_error(KUSH_ERR_ARG, "kush_sm100_write_jobs: null pointer");
    launch_pdl(write_jobs_kernel, dim3(1), dim3(PLAN_THREADS), 0, static_cast<cudaStream_t>(stream), query_start_loc,
               seq_lens, n_seqs, int(page), job_seq, job_page, int(max_jobs), n_jobs);
    return check_launch("kush_sm100_write_jobs");
}

extern "C" int kush_sm100_unpack_plan(const int32_t* query_start_loc, const int32_t* seq_lens,
                                      const int32_t* tail_idx, const int32_t* block_table, int64_t max_pages,
                                      int32_t n_seqs, int32_t page, int32_t* kv_start, int32_t* page_blk,
                                      int32_t* page_dst, int32_t max_page_entries, int32_t* tail_blk,
                                      int32_t* tail_info, int32_t max_tail_entries, int32_t* new_dst, int32_t max_new,
                                      int32_t* counts, void* stream) {
    if (n_seqs < 0 || max_page_entries < 0 || max_tail_entries < 0 || max_new < 0 || max_pages < 1 ||
        (page != 16 && page != 32))
        return set_error(KUSH_ERR_ARG, "kush_sm100_unpack_plan: n_seqs %d, capacities %d %d %d, max_pages %lld, page %d",
                         n_seqs, max_page_entries, max_tail_entries, max_new, (long long)max_pages, page);
    if (!query_start_loc || !seq_lens || !tail_idx || !block_table || !kv_start || !counts ||
        (max_page_entries && (!page_blk || !page_dst)) || (max_tail_entries && (!tail_blk || !tail_info)) ||
        (max_new && !new_dst))
        return set_error(KUSH_ERR_ARG, "kush_sm100_unpack_plan: null pointer");
    launch_pdl(unpack_plan_kernel, dim3(1), dim3(PLAN_THREADS), 0, static_cast<cudaStream_t>(stream), query_start_loc,
               seq_lens, tail_idx, block_table, max_pages, n_seqs, int(page), kv_start, page_blk, page_dst,
               int(max_page_entries), tail_blk, tail_info, int(max_tail_entries), new_dst, int(max_new), counts);
    return check_launch("kush_sm100_unpack_plan");
}
