"""kushkash_b200.Ops: the library's own PyTorch-facing operator object, one per (device, head_dim, bits, group,
dtype, page), calling the C ABI of libkush_sm100.so (include/kushkash_b200.h) directly.

Two ways reach the same kernels:
  * the reference's own operator layer (kushkash/_ops.py Ops, cache.py KushCache, the HF / vLLM / SGLang
    integrations), unchanged, through the drop-in loader kushkash_b200._cuda (kushkash_b200.dropin.install());
  * this class, which the benchmarks, the sharding layer and the parity tests use.  Its calls take the same
    tensors with the same meaning as kushkash.Ops (kushkash/_ops.py:42-213) -- so code written against one reads
    the same against the other -- plus what the reference cannot express: the page size (16 or 32 tokens), the
    rotation fused into the kernels, a decode launch order and the split-KV partials without their combine.

Tensor conventions (the record layout of kushkash/kush/quant.mojo:53-87):
  cache        [blocks, H, ...] uint8 (any view whose (block, head) records are contiguous; byte strides are passed)
  tail_k       [slots, H, P, D] in the kernel dtype: exact K of each sequence's unfinished page (slot tail_idx[s])
  k, v rows    [rows, H, D], row strides free, head stride D
  q, out       [S, H * G, D] contiguous, q head = kv_head * G + g
  index tensors int32 on the device

Every call is asynchronous on torch's current stream of the device; nothing allocates except the optional outputs
of fwht() and longest_first().  There is no CPU path and no PyTorch fallback: a non-CUDA device, a missing library
or an unsupported configuration raises.
"""
from __future__ import annotations

import os

import torch

from . import _cuda
from ._build import PAGE, GpuConfig

_DTYPE_NAMES = {torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float32"}
MAX_SPLITS = 256
MIN_SPLIT_PAGES = 16
LONG_SPLIT_PAGES = 100


def record_bytes(head_dim: int, bits: int, page: int = PAGE) -> int:
    """Bytes of one (page, kv head) record: P code rows each for K and V (D bytes at 8 bits, D/2 at 4) and fp16
    K scale / bias per channel and V scale / bias per token (the format of kushkash/kush/quant.mojo:53-87)."""
    dc = head_dim if bits == 8 else head_dim // 2
    return 2 * page * dc + 4 * head_dim + 4 * page


def split_factor(num_seqs: int, num_kv_heads: int, max_full_pages: int, sms: int, ctas_per_sm: int = 4) -> int:
    """Split-KV factor: enough splits that the decode grid fills the ~ctas_per_sm resident CTAs of every SM once (any
    integer, not only powers of two), at most MAX_SPLITS and at least MIN_SPLIT_PAGES pages per split; 1 when the
    (sequence, kv head) units alone fill half the GPU.  (The reference grows powers of two up to 32 while the grid
    has fewer than 6 blocks per SM, kushkash/_ops.py:182-189; on B200 fewer, fuller splits measured faster: per-split
    setup, merge and the combine grow with the split count -- 8 sequences x 4 kv heads x 64 pages decode fastest at 4
    splits, not 16.)"""
    units, cap = num_seqs * num_kv_heads, ctas_per_sm * sms
    if units == 0 or units * 2 >= cap or max_full_pages < 8:
        return 1
    ns = max(1, min(MAX_SPLITS, cap // units, max_full_pages // MIN_SPLIT_PAGES))
    # Past two CTAs per SM, splits of fewer than LONG_SPLIT_PAGES pages lose more to per-split setup and merge than
    # the extra CTAs give back (config 4 geometry with 2 kv heads: 74 splits of 55 pages 65.7 us, 37 of 111 56.1 us;
    # with 4 kv heads 37 splits of 111 pages stay the fastest): keep two CTAs per SM and splits of ~LONG_SPLIT_PAGES.
    if units * ns > 2 * sms and max_full_pages // ns < LONG_SPLIT_PAGES:
        ns = max(-(-2 * sms // units), min(ns, -(-max_full_pages // LONG_SPLIT_PAGES)))
    return ns


def _pool(cache: torch.Tensor) -> tuple[int, int, int]:
    """(address, block stride, head stride) of a record pool, strides in bytes."""
    e = cache.element_size()
    return cache.data_ptr(), cache.stride(0) * e, cache.stride(1) * e


def _table(block_table: torch.Tensor) -> tuple[int, int]:
    """(address, row stride in entries) of a block table."""
    return block_table.data_ptr(), block_table.stride(0)


def _need(ok: bool, what: str) -> None:
    if not ok:
        raise ValueError(what)


class Ops:
    """The kernels of one (device, head_dim, bits, group, dtype, page) configuration."""

    def __init__(self, device: torch.device, head_dim: int, bits: int, group: int, dtype: torch.dtype,
                 page: int = PAGE):
        device = torch.device(device)
        _need(device.type == "cuda", "kushkash_b200 runs on CUDA (B200, sm_100a) devices only; it has no CPU path")
        _need(head_dim in (64, 128, 256), "GPU head_dim must be 64, 128 or 256")
        _need(dtype in _DTYPE_NAMES, f"dtype must be one of {tuple(_DTYPE_NAMES)}")
        self.dev = device.index if device.index is not None else torch.cuda.current_device()
        self.device = torch.device("cuda", self.dev)
        self.D, self.bits, self.G, self.dtype, self.P = head_dim, bits, group, dtype, page
        self.cfg = GpuConfig(head_dim, bits, group, _DTYPE_NAMES[dtype], _cuda.arch(self.dev), page)
        self.sms = _cuda.sm_count(self.dev)
        self.lib = _cuda.lib()
        self._fmt = (head_dim, bits, page, self.cfg.dtype_code)        # leading arguments of most entry points
        self.fused_write = os.environ.get("KUSHKASH_FUSED_WRITE", "1") != "0"

    def _run(self, entry: str, *args) -> None:
        """Call one C entry point with torch's current stream of this device appended; raise on a failed status."""
        fn = getattr(self.lib, entry)
        if torch.cuda.current_device() == self.dev:
            rc = fn(*args, _cuda.raw_stream(self.dev))
        else:
            with torch.cuda.device(self.dev):
                rc = fn(*args, _cuda.raw_stream(self.dev))
        _cuda.check(rc, entry)

    # ---------------------------------------------------------------- quantize-on-write
    def append(self, k: torch.Tensor, v: torch.Tensor, seq_lens: torch.Tensor, tail_idx: torch.Tensor,
               cache: torch.Tensor, block_table: torch.Tensor, tail_k: torch.Tensor, pos_offset: int, advance: bool,
               *, rotate: bool = False) -> None:
        """One new token per sequence: row s of k / v lands at position seq_lens[s] + pos_offset (negative positions
        are skipped); advance stores pos + 1 into seq_lens.  rotate: rotate the rows first (canonical Walsh-Hadamard,
        bit for bit what fwht() then append() store)."""
        entry = "kush_sm100_append_rotated" if rotate else "kush_sm100_append"
        self._run(entry, *self._fmt, k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0), seq_lens.data_ptr(),
                  int(pos_offset), int(bool(advance)), tail_idx.data_ptr(), *_pool(cache), tail_k.data_ptr(),
                  *_table(block_table), k.shape[1], k.shape[0])

    def write(self, k: torch.Tensor, v: torch.Tensor, query_start_loc: torch.Tensor, seq_lens: torch.Tensor,
              tail_idx: torch.Tensor, job_seq: torch.Tensor, job_page: torch.Tensor, cache: torch.Tensor,
              block_table: torch.Tensor, tail_k: torch.Tensor) -> None:
        """Ragged multi-token write: sequence s owns rows [qsl[s], qsl[s+1]) at the positions that end at
        seq_lens[s] (which already counts them); job j is logical page job_page[j] of sequence job_seq[j].  One
        launch (mode 2); KUSHKASH_FUSED_WRITE=0 (or fused_write = False) runs the two-launch form (modes 0, 1)."""
        n_jobs = job_seq.numel()
        if n_jobs == 0:
            return
        for mode in ((2,) if self.fused_write else (0, 1)):
            self._run("kush_sm100_write", *self._fmt, k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0),
                      query_start_loc.data_ptr(), seq_lens.data_ptr(), tail_idx.data_ptr(), job_seq.data_ptr(),
                      job_page.data_ptr(), mode, *_pool(cache), tail_k.data_ptr(), *_table(block_table), k.shape[1],
                      n_jobs)

    def write_jobs(self, query_start_loc: torch.Tensor, seq_lens: torch.Tensor, max_jobs: int,
                   job_seq: torch.Tensor | None = None, job_page: torch.Tensor | None = None,
                   n_jobs: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """The jobs of write() for a step, built on the device (kush_sm100_write_jobs): one per (sequence, logical
        page its rows touch), in sequence then page order, then padding to max_jobs that write() skips.  Returns
        (job_seq, job_page, n_jobs) -- n_jobs a one-element device tensor.  max_jobs >= rows // P + 2 * S always
        suffices; nothing is read back to the host, so the call can be captured in a CUDA graph."""
        S = seq_lens.numel()
        _need(all(t.dtype == torch.int32 and t.is_contiguous() for t in (query_start_loc, seq_lens))
              and query_start_loc.numel() >= S + 1, "write_jobs: query_start_loc [S + 1] and seq_lens [S] must be "
              "contiguous int32")
        dev = seq_lens.device
        job_seq = torch.empty(max_jobs, dtype=torch.int32, device=dev) if job_seq is None else job_seq
        job_page = torch.empty(max_jobs, dtype=torch.int32, device=dev) if job_page is None else job_page
        n_jobs = torch.empty(1, dtype=torch.int32, device=dev) if n_jobs is None else n_jobs
        _need(job_seq.numel() >= max_jobs and job_page.numel() >= max_jobs and n_jobs.numel() >= 1,
              "write_jobs: output tensors smaller than max_jobs")
        self._run("kush_sm100_write_jobs", query_start_loc.data_ptr(), seq_lens.data_ptr(), S, self.P,
                  job_seq.data_ptr(), job_page.data_ptr(), max_jobs, n_jobs.data_ptr())
        return job_seq[:max_jobs], job_page[:max_jobs], n_jobs

    def unpack_plan(self, query_start_loc: torch.Tensor, seq_lens: torch.Tensor, tail_idx: torch.Tensor,
                    block_table: torch.Tensor, max_pages: int, max_tails: int, max_new: int) -> dict:
        """The plan of unpack() for a step that packs every sequence's history and new rows together (sequence s
        at rows kv_start[s] .. kv_start[s + 1]), built on the device (kush_sm100_unpack_plan); each list padded to
        its capacity with entries unpack() skips.  Returns kv_start [S + 1] (the varlen attention's cu_seqlens_k),
        page_blk, page_dst, tail_blk, tail_info, new_dst and counts [4] (full pages, partial pages, new rows, packed
        rows), all on the device."""
        S, dev = seq_lens.numel(), seq_lens.device
        _need(all(t.dtype == torch.int32 and t.is_contiguous() for t in (query_start_loc, seq_lens, tail_idx))
              and block_table.dtype == torch.int32 and block_table.stride(1) == 1,
              "unpack_plan: index tensors must be int32 (query_start_loc, seq_lens, tail_idx contiguous)")
        i32 = dict(dtype=torch.int32, device=dev)
        plan = dict(kv_start=torch.empty(S + 1, **i32), page_blk=torch.empty(max_pages, **i32),
                    page_dst=torch.empty(max_pages, **i32), tail_blk=torch.empty(max_tails, **i32),
                    tail_info=torch.empty(3 * max_tails, **i32), new_dst=torch.empty(max_new, **i32),
                    counts=torch.empty(4, **i32))
        self._run("kush_sm100_unpack_plan", query_start_loc.data_ptr(), seq_lens.data_ptr(), tail_idx.data_ptr(),
                  *_table(block_table), S, self.P, plan["kv_start"].data_ptr(), plan["page_blk"].data_ptr(),
                  plan["page_dst"].data_ptr(), max_pages, plan["tail_blk"].data_ptr(), plan["tail_info"].data_ptr(),
                  max_tails, plan["new_dst"].data_ptr(), max_new, plan["counts"].data_ptr())
        return plan

    # ---------------------------------------------------------------- rotation and unpack
    def fwht(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """The canonical Walsh-Hadamard rotation of every D-row of x (contiguous, this dtype) into out (a new
        tensor, or x itself, or any contiguous tensor of x's shape and dtype); returns out."""
        y = torch.empty_like(x) if out is None else out
        _need(x.dtype == self.dtype and y.dtype == self.dtype, f"fwht: tensors must be {self.dtype}")
        _need(x.is_contiguous() and y.is_contiguous() and x.shape == y.shape and x.shape[-1] == self.D,
              f"fwht: x and out must be contiguous, of one shape, with last dim {self.D}")
        rows = x.numel() // self.D
        if rows:
            self._run("kush_sm100_fwht", self.D, self.cfg.dtype_code, x.data_ptr(), y.data_ptr(), self.D, self.D,
                      rows)
        return y

    def unpack(self, cache: torch.Tensor, page_blk: torch.Tensor, page_dst: torch.Tensor, tail_blk: torch.Tensor,
               tail_info: torch.Tensor, tail_k: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
               new_dst: torch.Tensor, kp: torch.Tensor, vp: torch.Tensor, rot: bool) -> None:
        """Keys and values of a prefill with history into kp / vp ([rows, H, D], contiguous, this dtype): full pages
        (block page_blk[i] -> rows page_dst[i] + t), partial pages (block tail_blk[i], tail_info[i] = first row,
        tokens, tail slot; K from tail_k), new rows (row j of k_new / v_new -> row new_dst[j]); rot rotates history
        back.  Index values are not checked on the host (that would synchronise); the tensors' kinds are."""
        H = kp.shape[1]
        idx = (page_blk, page_dst, tail_blk, tail_info, new_dst)
        _need(all(t.dtype == torch.int32 and t.is_contiguous() for t in idx), "unpack: index tensors must be "
              "contiguous int32")
        _need(all(t.dtype == self.dtype for t in (tail_k, k_new, v_new, kp, vp)),
              f"unpack: tail_k, k_new, v_new, kp and vp must be {self.dtype}")
        _need(kp.shape == vp.shape and kp.dim() == 3 and kp.shape[2] == self.D and kp.is_contiguous()
              and vp.is_contiguous(), f"unpack: kp and vp must be contiguous [rows, H, {self.D}]")
        _need(all(t.dim() == 3 and tuple(t.shape[1:]) == (H, self.D) and t.stride(1) == self.D and t.stride(2) == 1
                  for t in (k_new, v_new)), "unpack: k_new / v_new rows must be [n, H, D] with head stride D")
        n_pages, n_tail, n_new = page_blk.numel(), tail_blk.numel(), new_dst.numel()
        _need(page_dst.numel() == n_pages and tail_info.numel() == 3 * n_tail
              and min(k_new.shape[0], v_new.shape[0]) >= n_new,
              "unpack: one page_dst per page, three tail_info ints per partial page, one k_new / v_new row per new_dst")
        if n_pages + n_tail + n_new == 0:
            return
        self._run("kush_sm100_unpack", *self._fmt, *_pool(cache), H, page_blk.data_ptr(), page_dst.data_ptr(),
                  n_pages, tail_blk.data_ptr(), tail_info.data_ptr(), n_tail, tail_k.data_ptr(), k_new.data_ptr(),
                  v_new.data_ptr(), k_new.stride(0), v_new.stride(0), new_dst.data_ptr(), n_new, kp.data_ptr(),
                  vp.data_ptr(), int(bool(rot)))

    # ---------------------------------------------------------------- decode
    def splits(self, num_seqs: int, num_kv_heads: int, max_full_pages: int) -> int:
        """Split-KV factor for this device (split_factor)."""
        return split_factor(num_seqs, num_kv_heads, max_full_pages, self.sms)

    def work_size(self, num_seqs: int, num_kv_heads: int, n_splits: int, fused: bool = False) -> int:
        """fp32 elements of the split-KV work buffer: S * Hkv * n_splits * G * (D + 2), the (M, L) pairs first, then
        the unnormalised outputs (the sizing rule of kushkash/_ops.py:195).  fused: S * Hkv more 32-bit slots at the
        end, the counters of decode(fused=True) (they must be 0 before the first fused decode: allocate the buffer
        with torch.zeros; every fused decode leaves them 0)."""
        return num_seqs * num_kv_heads * (n_splits * self.G * (self.D + 2) + (1 if fused else 0))

    def _parts(self, S: int, H: int, n_splits: int, work: torch.Tensor | None,
               fused: bool = False) -> tuple[int, int]:
        n_ml = S * H * n_splits * self.G * 2
        _need(work is not None and work.dtype == torch.float32 and work.is_contiguous()
              and work.numel() >= self.work_size(S, H, n_splits, fused),
              f"decode: n_splits={n_splits} needs a contiguous fp32 work buffer of >= "
              f"{self.work_size(S, H, n_splits, fused)} elements")
        return work.data_ptr(), work.data_ptr() + 4 * n_ml

    def decode(self, q: torch.Tensor, out: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor,
               seq_lens: torch.Tensor, tail_idx: torch.Tensor, tail_k: torch.Tensor, scale: float, n_splits: int = 1,
               work: torch.Tensor | None = None, *, rotate: bool = False, order: torch.Tensor | None = None,
               fused: bool = False) -> None:
        """out[s] = softmax-scaled attention of q[s] over the seq_lens[s] cached tokens of sequence s.  n_splits > 1
        splits each sequence's pages over CTAs (split-KV) and merges them with a second launch; it needs `work`
        (work_size() fp32 elements).  fused: the merge runs inside the decode launch instead (the last CTA of each
        (sequence, kv head) merges; the same output bit for bit); `work` then needs work_size(..., fused=True)
        elements whose last S * Hkv start at 0.  rotate: the cache holds rotated K / V; q is rotated inside the
        kernel and the output rotated back before its store.  order: a contiguous int32 permutation of the
        sequences, CTA x then decoding sequence order[x] (longest_first()); the outputs do not depend on it."""
        S, H = q.shape[0], tail_k.shape[1]
        ml = o = 0
        if n_splits > 1:
            ml, o = self._parts(S, H, n_splits, work, fused)
        if fused and n_splits > 1:
            if order is not None:
                _need(order.dtype == torch.int32 and order.numel() == S and order.is_contiguous(),
                      "decode: order must be a contiguous int32 permutation of the sequences")
            counters = ml + 4 * S * H * n_splits * self.G * (self.D + 2)
            self._run("kush_sm100_decode_fused_combine", *self._fmt, self.G, q.data_ptr(), out.data_ptr(),
                      *_pool(cache), tail_k.data_ptr(), tail_idx.data_ptr(), block_table.data_ptr(),
                      seq_lens.data_ptr(), block_table.stride(0), H, float(scale), n_splits, ml, o, counters, S,
                      1 if rotate else 0, order.data_ptr() if order is not None else None)
            return
        self._decode(q, out.data_ptr(), cache, block_table, seq_lens, tail_idx, tail_k, scale, n_splits, ml, o,
                     rotate, order)
        if n_splits > 1:
            entry = "kush_sm100_combine_rotated" if rotate else "kush_sm100_combine"
            self._run(entry, self.D, self.cfg.dtype_code, self.G, out.data_ptr(), ml, o, n_splits, H, S)

    def decode_partials(self, q: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor,
                        seq_lens: torch.Tensor, tail_idx: torch.Tensor, tail_k: torch.Tensor, scale: float,
                        n_splits: int, work: torch.Tensor) -> tuple[int, int]:
        """The split-KV decode (n_splits >= 2) without its combine: the per-split (M, L) and unnormalised outputs
        in `work`, for a combine that writes elsewhere (the peer gather of KV-head sharding, shard.PeerGather).
        Returns their device addresses (part_ml, part_o)."""
        _need(n_splits >= 2, "decode_partials needs n_splits >= 2")
        S, H = q.shape[0], tail_k.shape[1]
        ml, o = self._parts(S, H, n_splits, work)
        self._decode(q, o, cache, block_table, seq_lens, tail_idx, tail_k, scale, n_splits, ml, o)
        return ml, o

    def _decode(self, q, out_ptr: int, cache, block_table, seq_lens, tail_idx, tail_k, scale: float, n_splits: int,
                part_ml: int, part_o: int, rotate: bool = False, order: torch.Tensor | None = None) -> None:
        S, H = q.shape[0], tail_k.shape[1]
        head = (*self._fmt, self.G, q.data_ptr(), out_ptr, *_pool(cache), tail_k.data_ptr(), tail_idx.data_ptr(),
                block_table.data_ptr(), seq_lens.data_ptr(), block_table.stride(0), H, float(scale), n_splits,
                part_ml or None, part_o or None, S)
        if order is None:
            self._run("kush_sm100_decode_rotated" if rotate else "kush_sm100_decode", *head)
            return
        _need(order.dtype == torch.int32 and order.numel() == S and order.is_contiguous(),
              "decode: order must be a contiguous int32 permutation of the sequences")
        self._run("kush_sm100_decode_ex", *head, 1 if rotate else 0, order.data_ptr())

    def longest_first(self, seq_lens: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """A launch order for decode(order=): the sequences by full pages, most first (one small kernel; compute it
        once per step, as the layers share seq_lens)."""
        S = seq_lens.numel()
        _need(seq_lens.dtype == torch.int32 and seq_lens.is_contiguous(), "longest_first: seq_lens must be "
              "contiguous int32")
        order = torch.empty(S, dtype=torch.int32, device=seq_lens.device) if out is None else out
        _need(order.dtype == torch.int32 and order.numel() == S and order.is_contiguous(),
              "longest_first: out must be a contiguous int32 tensor of n_seqs entries")
        self._run("kush_sm100_order_longest_first", seq_lens.data_ptr(), S, self.P, order.data_ptr())
        return order
