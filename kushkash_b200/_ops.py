"""Operator surface over the page-record layout: the B200 replacement of the reference's dispatch layer
(kushkash/_ops.py:42-213, class Ops), with the same method names, arguments and error behaviour.

Tensor conventions (as kushkash/_ops.py:6-15):
  cache       any tensor whose dim 0 is the block and dim 1 the kv head, each (block, head) record contiguous:
              uint8 [pages, H, RB] or [blocks, H, P, RB // P]; byte strides are passed, so it may be a slice
  tail_k      [slots, H, P, D] in the kernel dtype: K of the page being filled, exact; sequence s uses slot
              tail_idx[s]; its V rows are already final in the page's record
  k, v rows   [rows, H, D] (row strides free, may differ between k and v; head stride D)
  q, out      [S, Hq, D] contiguous (q head = kv_head * G + g)
  rotation    the kernels do not rotate; callers pass rotated q, k, v (fwht / rotate) and rotate the output back

Every kernel runs on the CUDA device on torch's current stream.  There is no CPU path and no PyTorch fallback:
constructing Ops for a non-CUDA device raises, and a missing kernel library raises on first use.
"""
from __future__ import annotations

import math
import os

import torch

from ._build import PAGE, GpuConfig

_TORCH_DTYPES = {torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float32"}
MAX_SPLITS = 256
MIN_SPLIT_PAGES = 16
LONG_SPLIT_PAGES = 100


def record_bytes(head_dim: int, bits: int, page: int = PAGE) -> int:
    """Bytes of one (page, kv head) record (kushkash/_ops.py:29-31, kushkash/kush/quant.mojo:60-62)."""
    dc = head_dim if bits == 8 else head_dim // 2
    return 2 * page * dc + 4 * head_dim + 4 * page


def _byte_strides(cache: torch.Tensor) -> tuple[int, int]:
    """Block and head strides in bytes (kushkash/_ops.py:34-39)."""
    e = cache.element_size()
    return cache.stride(0) * e, cache.stride(1) * e


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


class Ops:
    """Kernels for one (device, head_dim, bits, q-heads-per-kv-head, dtype[, page]) (kushkash/_ops.py:42-63)."""

    def __init__(self, device: torch.device, head_dim: int, bits: int, group: int, dtype: torch.dtype,
                 page: int = PAGE):
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("kushkash_b200 runs on CUDA (B200, sm_100a) devices only; it has no CPU path")
        if head_dim not in (64, 128, 256):
            raise ValueError("GPU head_dim must be 64, 128 or 256")
        if dtype not in _TORCH_DTYPES:
            raise ValueError(f"dtype must be one of {tuple(_TORCH_DTYPES)}")
        from . import _cuda
        self.device, self.D, self.bits, self.G, self.dtype, self.P = device, head_dim, bits, group, dtype, page
        self.gpu = True
        dev = device.index if device.index is not None else torch.cuda.current_device()
        self.dev = dev
        self.cfg = GpuConfig(head_dim, bits, group, _TORCH_DTYPES[dtype], _cuda.arch(dev), page)
        self.k = _cuda.kernels(dev, self.cfg)
        self.sms = _cuda.sm_count(dev)
        self.fused_write = os.environ.get("KUSHKASH_FUSED_WRITE", "1") != "0"

    # ---------------------------------------------------------------- writes
    def append(self, k: torch.Tensor, v: torch.Tensor, seq_lens: torch.Tensor, tail_idx: torch.Tensor,
               cache: torch.Tensor, block_table: torch.Tensor, tail_k: torch.Tensor,
               pos_offset: int, advance: bool, *, rotate: bool = False) -> None:
        """One token per sequence: row s of k/v goes to position seq_lens[s] + pos_offset (kushkash/_ops.py:66-80).
        rotate=True (an extension): the rows are rotated (canonical Walsh-Hadamard) inside the kernel first, bit for
        bit what fwht() then append() store."""
        S, H = k.shape[0], k.shape[1]
        bs, hs = _byte_strides(cache)
        self.k["append_rotated" if rotate else "append"]((S, 1, 1), self.D, k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0), seq_lens.data_ptr(),
                         pos_offset, int(advance), tail_idx.data_ptr(), cache.data_ptr(), bs, hs,
                         tail_k.data_ptr(), block_table.data_ptr(), block_table.stride(0), H)

    def write(self, k: torch.Tensor, v: torch.Tensor, query_start_loc: torch.Tensor, seq_lens: torch.Tensor,
              tail_idx: torch.Tensor, job_seq: torch.Tensor, job_page: torch.Tensor, cache: torch.Tensor,
              block_table: torch.Tensor, tail_k: torch.Tensor) -> None:
        """Ragged multi-token write (kushkash/_ops.py:82-101).  Sequence s owns rows [qsl[s], qsl[s+1]) at positions
        ending at seq_lens[s] (already counting them); one job per (sequence, logical page) touched.  One launch
        (mode 2) unless KUSHKASH_FUSED_WRITE=0, which runs the reference's two launches (mode 0, then mode 1)."""
        n_jobs, H = job_seq.numel(), k.shape[1]
        if n_jobs == 0:
            return
        bs, hs = _byte_strides(cache)
        for mode in ((2,) if self.fused_write else (0, 1)):
            self.k["write"]((n_jobs, H, 1), self.D, k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0),
                            query_start_loc.data_ptr(), seq_lens.data_ptr(), tail_idx.data_ptr(),
                            job_seq.data_ptr(), job_page.data_ptr(), mode, cache.data_ptr(), bs, hs,
                            tail_k.data_ptr(), block_table.data_ptr(), block_table.stride(0), H)

    # ---------------------------------------------------------------- rotation
    def fwht(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Canonical Walsh-Hadamard rotation of every D-row of contiguous x (kushkash/_ops.py:104-127); out may be x."""
        D = self.D
        if x.shape[-1] != D or not x.is_contiguous():
            raise ValueError(f"fwht: x must be contiguous with last dim {D}")
        out = torch.empty_like(x) if out is None else out
        if out.shape != x.shape or out.dtype != x.dtype or not out.is_contiguous():
            raise ValueError("fwht: out must be contiguous, with x's shape and dtype")
        rows = x.numel() // D
        if rows == 0:
            return out
        if x.dtype != self.dtype:
            raise ValueError(f"fwht: x is {x.dtype}, these kernels take {self.dtype}")
        self.k["fwht"](((rows + 3) // 4, 1, 1), 128, x.data_ptr(), out.data_ptr(), D, D, rows)
        return out

    # ---------------------------------------------------------------- unpack (prefill with history)
    def unpack(self, cache: torch.Tensor, page_blk: torch.Tensor, page_dst: torch.Tensor, tail_blk: torch.Tensor,
               tail_info: torch.Tensor, tail_k: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
               new_dst: torch.Tensor, kp: torch.Tensor, vp: torch.Tensor, rot: bool) -> None:
        """One packed-prefill group's keys / values into kp, vp ([rows, Hkv, D], contiguous), one launch
        (kushkash/_ops.py:129-179); same checks and errors."""
        H, D = kp.shape[1], self.D
        n_pages, n_tail, n_new = page_blk.numel(), tail_blk.numel(), new_dst.numel()
        for t in (page_blk, page_dst, tail_blk, tail_info, new_dst):
            if t.dtype != torch.int32 or not t.is_contiguous():
                raise ValueError("unpack: index tensors must be contiguous int32")
        if not (kp.is_contiguous() and vp.is_contiguous() and kp.shape == vp.shape and kp.shape[2] == D):
            raise ValueError("unpack: kp / vp must be contiguous [rows, Hkv, D]")
        for t in (k_new, v_new):
            if t.shape[1:] != (H, D) or t.stride(2) != 1 or t.stride(1) != D:
                raise ValueError("unpack: k_new / v_new must be [n, Hkv, D] with unit dim stride and head stride D")
        if tail_info.numel() != 3 * n_tail or k_new.shape[0] < n_new or v_new.shape[0] < n_new:
            raise ValueError("unpack: tail_info must hold 3 ints per partial page; k_new / v_new one row per new_dst")
        if page_dst.numel() != n_pages:
            raise ValueError("unpack: page_dst must hold one row per page_blk entry")
        for t in (tail_k, k_new, v_new, kp, vp):
            if t.dtype != self.dtype:
                raise ValueError(f"unpack: tail_k, k_new, v_new, kp, vp must be {self.dtype}, got {t.dtype}")
        if n_pages + n_tail + n_new == 0:
            return
        bs, hs = _byte_strides(cache)
        grid = (n_pages + n_tail + (n_new + 31) // 32, H, 1)
        self.k["unpack"](grid, 128, cache.data_ptr(), bs, hs, H, page_blk.data_ptr(), page_dst.data_ptr(), n_pages,
                         tail_blk.data_ptr(), tail_info.data_ptr(), n_tail, tail_k.data_ptr(), k_new.data_ptr(),
                         v_new.data_ptr(), k_new.stride(0), v_new.stride(0), new_dst.data_ptr(), n_new, kp.data_ptr(),
                         vp.data_ptr(), int(rot))

    # ---------------------------------------------------------------- decode
    def splits(self, num_seqs: int, num_kv_heads: int, max_full_pages: int) -> int:
        """Split-KV factor for this device (split_factor)."""
        return split_factor(num_seqs, num_kv_heads, max_full_pages, self.sms)

    def work_size(self, num_seqs: int, num_kv_heads: int, n_splits: int) -> int:
        """fp32 elements of the split-KV work buffer: S * Hkv * n_splits * G * (D + 2) (kushkash/_ops.py:195)."""
        return num_seqs * num_kv_heads * n_splits * self.G * (self.D + 2)

    def decode(self, q: torch.Tensor, out: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor,
               seq_lens: torch.Tensor, tail_idx: torch.Tensor, tail_k: torch.Tensor,
               scale: float, n_splits: int = 1, work: torch.Tensor | None = None, *, rotate: bool = False,
               order: torch.Tensor | None = None) -> None:
        """out[s] = attention of q[s] ([Hq, D]) over the seq_lens[s] cached tokens of sequence s
        (kushkash/_ops.py:191-213).  n_splits > 1 needs `work` (fp32, >= S*Hkv*n_splits*G*(D+2) elements).
        rotate=True (an extension, for a cache written with rotation): q is rotated inside the kernel and the output
        rotated back before its store, in place of fwht(q) before and fwht(out) after.  order (an extension): an int32
        permutation of the S sequences, CTA x decoding sequence order[x] (longest_first()); same outputs."""
        S, H = q.shape[0], tail_k.shape[1]
        part_ml = part_o = 0
        if n_splits > 1:
            part_ml, part_o = self._parts(S, H, n_splits, work)
        self._decode(q, out.data_ptr(), cache, block_table, seq_lens, tail_idx, tail_k, scale, n_splits, part_ml,
                     part_o, rotate, order)
        if n_splits > 1:
            self.k["combine_rotated" if rotate else "combine"]((S, H, 1), 256, out.data_ptr(), part_ml, part_o,
                                                               n_splits, H)

    def decode_partials(self, q: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor,
                        seq_lens: torch.Tensor, tail_idx: torch.Tensor, tail_k: torch.Tensor, scale: float,
                        n_splits: int, work: torch.Tensor) -> tuple[int, int]:
        """The split-KV decode without its combine (n_splits >= 2): the per-split partials (m, l and unnormalised
        outputs) in `work`, for a combine that writes elsewhere -- the peer gather of KV-head sharding
        (kushkash_b200.shard.PeerGather).  Returns the device addresses (part_ml, part_o) inside `work`.  No
        counterpart in the reference."""
        if n_splits < 2:
            raise ValueError("decode_partials needs n_splits >= 2")
        S, H = q.shape[0], tail_k.shape[1]
        part_ml, part_o = self._parts(S, H, n_splits, work)
        self._decode(q, part_o, cache, block_table, seq_lens, tail_idx, tail_k, scale, n_splits, part_ml, part_o)
        return part_ml, part_o

    def _parts(self, S: int, H: int, n_splits: int, work: torch.Tensor | None) -> tuple[int, int]:
        nml = S * H * n_splits * self.G * 2
        if work is None or work.dtype != torch.float32 or work.numel() < nml + S * H * n_splits * self.G * self.D:
            raise ValueError(f"decode: n_splits={n_splits} needs an fp32 work buffer of "
                             f">= {self.work_size(S, H, n_splits)} elements")
        return work.data_ptr(), work.data_ptr() + nml * 4

    def _decode(self, q, out_ptr: int, cache, block_table, seq_lens, tail_idx, tail_k, scale: float, n_splits: int,
                part_ml: int, part_o: int, rotate: bool = False, order: torch.Tensor | None = None) -> None:
        S, H = q.shape[0], tail_k.shape[1]
        bs, hs = _byte_strides(cache)
        args = (q.data_ptr(), out_ptr, cache.data_ptr(), bs, hs, tail_k.data_ptr(), tail_idx.data_ptr(),
                block_table.data_ptr(), seq_lens.data_ptr(), block_table.stride(0), H, float(scale), n_splits, part_ml,
                part_o)
        if order is None:
            self.k["decode_rotated" if rotate else "decode"]((S, H, n_splits), 32 * self.cfg.warps, *args)
            return
        if order.dtype != torch.int32 or order.numel() != S or not order.is_contiguous():
            raise ValueError("decode: order must be a contiguous int32 permutation of the sequences")
        self.k["decode_ex"]((S, H, n_splits), 32 * self.cfg.warps, *args, 1 if rotate else 0, order.data_ptr())

    def longest_first(self, seq_lens: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """A launch order for decode(order=): the sequences by full pages, most first (one small kernel; compute it
        once per step, as the layers share seq_lens).  No counterpart in the reference."""
        S = seq_lens.numel()
        if seq_lens.dtype != torch.int32 or not seq_lens.is_contiguous():
            raise ValueError("longest_first: seq_lens must be contiguous int32")
        out = torch.empty(S, dtype=torch.int32, device=seq_lens.device) if out is None else out
        if out.dtype != torch.int32 or out.numel() != S or not out.is_contiguous():
            raise ValueError("longest_first: out must be a contiguous int32 tensor of n_seqs entries")
        self.k["order_longest_first"]((1, 1, 1), 1024, seq_lens.data_ptr(), S, out.data_ptr())
        return out


# ---------------------------------------------------------------- format helpers (pure PyTorch, for tests / callers)
def as_records(cache: torch.Tensor) -> torch.Tensor:
    """View any cache tensor ([blocks, H, ...], contiguous records) as uint8 [blocks, H, RB] (kushkash/_ops.py:288-292)."""
    c = cache.view(torch.uint8) if cache.dtype != torch.uint8 else cache
    return c.flatten(2) if c.dim() > 3 else c


def dequant_records(rec: torch.Tensor, head_dim: int, bits: int, dtype: torch.dtype, page: int = PAGE
                    ) -> tuple[torch.Tensor, torch.Tensor]:
    """Records [..., RB] (uint8) -> K, V [..., P, D] in dtype: codes * fp16 scale + fp16 bias
    (kushkash/_ops.py:217-251)."""
    D, P = head_dim, page
    dc = D if bits == 8 else D // 2
    kq = rec[..., :P * dc].view(torch.int8).unflatten(-1, (P, dc))
    vq = rec[..., P * dc:2 * P * dc].view(torch.int8).unflatten(-1, (P, dc))
    meta = rec[..., 2 * P * dc:].contiguous().view(torch.float16)
    ks, kb = meta[..., :D].unsqueeze(-2), meta[..., D:2 * D].unsqueeze(-2)
    vs, vb = meta[..., 2 * D:2 * D + P, None], meta[..., 2 * D + P:, None]

    def codes(c):
        if bits == 4:
            c = torch.cat([(c << 4) >> 4, c >> 4], -1)
        return c.to(dtype)
    return codes(kq) * ks.to(dtype) + kb.to(dtype), codes(vq) * vs.to(dtype) + vb.to(dtype)


def cached_kv(records: torch.Tensor, block_ids: torch.Tensor, n: int, tail_k: torch.Tensor, head_dim: int,
              bits: int, dtype: torch.dtype, page: int = PAGE) -> tuple[torch.Tensor, torch.Tensor]:
    """The n cached tokens of B sequences as K, V [B, Hk, n, D] (pages dequantized; the partial last page: exact K
    from tail_k [B, Hk, P, D], V from its record) (kushkash/_ops.py:295-306)."""
    B, Hk, D, P = block_ids.shape[0], tail_k.shape[1], head_dim, page
    pages = -(-n // P)
    k, v = dequant_records(records[block_ids[:, :pages].long()], D, bits, dtype, P)       # [B, p, Hk, P, D]
    k = k.permute(0, 2, 1, 3, 4).reshape(B, Hk, pages * P, D)
    v = v.permute(0, 2, 1, 3, 4).reshape(B, Hk, pages * P, D)[:, :, :n]
    r = n % P
    k = torch.cat([k[:, :, :n - r], tail_k[:, :, :r].to(dtype)], 2)
    return k, v


def pages_touched(ctx: int, total: int, page: int = PAGE) -> range:
    """Logical pages written when positions [ctx, total) are added (kushkash/_ops.py:342-344)."""
    return range(ctx // page, (total - 1) // page + 1) if total > ctx else range(0)


def rotation_enabled(bits: int, rotate: bool | None = None) -> bool:
    """KUSHKASH_ROTATE (auto | 1 | 0; auto = on for 4-bit) unless `rotate` is given (kushkash/_ops.py:350-359)."""
    if rotate is None:
        env = os.environ.get("KUSHKASH_ROTATE", "auto")
        if env not in ("auto", "0", "1"):
            raise ValueError(f"KUSHKASH_ROTATE must be auto, 0 or 1, got {env}")
        return bits == 4 if env == "auto" else env == "1"
    return bool(rotate)


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
