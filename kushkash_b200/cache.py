"""KushCache: the plain-tensor paged, quantized KV cache (int4 / int8) with fused decode attention, for
equal-length batches -- the B200 version of the reference's caller API (kushkash/cache.py:43-246), on CUDA only.

Memory per layer (kushkash/cache.py:6-12):
    pool     uint8 [pages, Hkv, RB]     one record per (page, kv head): codes + scales
    tail_k   [B, Hkv, P, D]             K of the page being filled, exact (model dtype); its V rows are already
                                        final in the page's record
Shared by all layers: block_table int32 [B, max_pages] (logical -> physical page).
With rotation on (rotate=, KUSHKASH_ROTATE; default on at 4 bits), pages and tail hold K H and V H (canonical
Walsh-Hadamard H); every public method takes and returns unrotated tensors.  The decode step rotates inside its
kernels (the rotated append, the decode that rotates q and its output); multi-token writes rotate with the fwht
kernel first.
`page` is the tokens per page record: 32 is kushkash's format, 16 the same layout with 16 rows.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ._build import PAGE
from ._ops import Ops, cached_kv, default_scale, record_bytes, rotation_enabled

_GPU_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


@dataclass
class MemoryStats:
    tokens: int            # tokens cached per sequence
    quantized_bytes: int   # page records in use, all layers
    tail_bytes: int        # exact K tails, all layers
    reserved_bytes: int    # pool capacity incl. unused pages
    fp16_bytes: int        # what an fp16 cache of the same content would take

    @property
    def ratio(self) -> float:
        used = self.quantized_bytes + self.tail_bytes
        return self.fp16_bytes / used if used else float("nan")


class KushCache:
    """
    Args (kushkash/cache.py:44-55):
        num_layers, num_kv_heads, num_q_heads, head_dim: model attention shape.
        batch_size: sequences per batch (they advance together).
        bits: 4 or 8.
        device: "cuda[:i]".
        dtype: dtype of q / k / v given to the cache and of the attention output.
        max_length: optional per-sequence capacity hint; pools grow on demand otherwise.
        scale: softmax scale (default 1/sqrt(head_dim)).
        rotate: Hadamard-rotate K, V and q inside the cache.  None: KUSHKASH_ROTATE (auto: on for 4-bit).
        page: tokens per page record (32, or 16).
    """

    def __init__(self, num_layers: int, num_kv_heads: int, num_q_heads: int, head_dim: int, *,
                 batch_size: int = 1, bits: int = 4, device: str | torch.device = "cuda",
                 dtype: torch.dtype = torch.float16, max_length: int | None = None, scale: float | None = None,
                 rotate: bool | None = None, page: int = PAGE):
        if bits not in (4, 8):
            raise ValueError("bits must be 4 or 8")
        if num_q_heads % num_kv_heads:
            raise ValueError("num_q_heads must be a multiple of num_kv_heads")
        if dtype not in _GPU_DTYPES:
            raise ValueError(f"dtype must be one of {_GPU_DTYPES}")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("kushkash_b200.KushCache runs on CUDA devices only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.L, self.H, self.D, self.B, self.P = num_layers, num_kv_heads, head_dim, batch_size, page
        self.G = num_q_heads // num_kv_heads
        self.bits = bits
        self.RB = record_bytes(head_dim, bits, page)
        self.dtype = self.kdtype = dtype
        self.scale = float(scale) if scale is not None else default_scale(head_dim)
        self.gpu = True
        self.ops = Ops(self.device, head_dim, bits, self.G, dtype, page)
        self.rot = rotation_enabled(bits, rotate)
        self._work = torch.empty(0, dtype=torch.float32, device=self.device)
        pages0 = max(1, -(-(max_length or 4 * page) // page))
        self._pages = 0
        self.pool = torch.empty(0, dtype=torch.uint8, device=self.device)
        self._alloc_pages(batch_size * pages0)
        self.block_table = torch.zeros(batch_size, pages0, dtype=torch.int32, device=self.device)
        self.tail_k = torch.zeros(num_layers, batch_size, num_kv_heads, page, head_dim, dtype=dtype, device=self.device)
        self.tail_idx = torch.arange(batch_size, dtype=torch.int32, device=self.device)
        self.seq_lens = torch.zeros(num_layers, batch_size, dtype=torch.int32, device=self.device)
        self._len = [0] * num_layers
        self._mapped = 0
        self._next = 0
        self._frozen_ns = 0
        self._capacity = 0

    # ---------------------------------------------------------------- page management
    def _alloc_pages(self, n: int) -> None:
        new = torch.zeros(self.L, n, self.H, self.RB, dtype=torch.uint8, device=self.device)
        if self._pages:
            new[:, :self._pages] = self.pool
        self.pool, self._pages = new, n

    def _map(self, need: int) -> None:
        """Map logical pages [0, need) of every sequence to physical pages from a bump allocator
        (kushkash/cache.py:106-126)."""
        if need <= self._mapped:
            return
        if self._frozen_ns:
            raise RuntimeError(f"cache capacity {self._capacity} exceeded (set a larger max_length)")
        add = need - self._mapped
        if self._next + add * self.B > self._pages:
            self._alloc_pages(max(2 * self._pages, self._next + add * self.B))
        if need > self.block_table.shape[1]:
            bt = torch.zeros(self.B, max(need, 2 * self.block_table.shape[1]), dtype=torch.int32, device=self.device)
            bt[:, :self.block_table.shape[1]] = self.block_table
            self.block_table = bt
        ids = torch.arange(self._next, self._next + add * self.B, dtype=torch.int32, device=self.device)
        self.block_table[:, self._mapped:need] = ids.view(self.B, add)
        self._next += add * self.B
        self._mapped = need

    def _rotate(self, x: torch.Tensor) -> torch.Tensor:
        """Canonical Walsh-Hadamard rotation of the last dim (its own inverse), in the kernel dtype."""
        x = x.to(self.kdtype).contiguous()
        return self.ops.fwht(x) if self.rot else x

    # ---------------------------------------------------------------- public API
    def length(self, layer: int = 0) -> int:
        return self._len[layer]

    def write(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append T new tokens for every sequence; k, v: [B, Hkv, T, D] (kushkash/cache.py:132-162).
        T == 1 takes the append kernel (which also advances seq_lens); longer chunks the ragged write kernel with
        one job per (sequence, logical page) touched."""
        B, H, T, D = k.shape
        if (B, H, D) != (self.B, self.H, self.D) or v.shape != k.shape:
            raise ValueError(f"expected k, v of shape [{self.B}, {self.H}, T, {self.D}], got {tuple(k.shape)}")
        if T == 0:
            return
        n, P = self._len[layer], self.P
        self._map(-(-(n + T) // P))
        args = dict(cache=self.pool[layer], block_table=self.block_table, tail_k=self.tail_k[layer])
        if T == 1:                                  # rotation (if on) inside the append kernel
            k = k.to(self.kdtype).reshape(B, H, D).contiguous()
            v = v.to(self.kdtype).reshape(B, H, D).contiguous()
            self.ops.append(k, v, self.seq_lens[layer], self.tail_idx, pos_offset=0, advance=True, rotate=self.rot,
                            **args)
        else:
            k = self._rotate(k).transpose(1, 2).contiguous().reshape(B * T, H, D)
            v = self._rotate(v).transpose(1, 2).contiguous().reshape(B * T, H, D)
            self.seq_lens[layer].fill_(n + T)
            pages = torch.arange(n // P, (n + T - 1) // P + 1, dtype=torch.int32, device=self.device)
            job_seq = torch.arange(B, dtype=torch.int32, device=self.device).repeat_interleave(pages.numel())
            qsl = torch.arange(B + 1, dtype=torch.int32, device=self.device) * T
            self.ops.write(k, v, qsl, self.seq_lens[layer], self.tail_idx, job_seq, pages.repeat(B), **args)
        self._len[layer] = n + T

    def attend(self, layer: int, q: torch.Tensor) -> torch.Tensor:
        """Decode attention of one query token per sequence over the whole cache; q: [B, Hq, D] -> [B, Hq, D]
        (kushkash/cache.py:164-183)."""
        if self._len[layer] == 0:
            raise RuntimeError("attend() on an empty cache")
        q = q.to(self.kdtype).contiguous()                 # rotated (if on) inside the decode kernel
        out = torch.empty_like(q)
        ns = self._frozen_ns or self.ops.splits(self.B, self.H, self._len[layer] // self.P)
        if ns > 1:
            need = self.ops.work_size(self.B, self.H, ns)
            if self._work.numel() < need:
                self._work = torch.empty(need, dtype=torch.float32, device=self.device)
        self.ops.decode(q, out, self.pool[layer], self.block_table, self.seq_lens[layer], self.tail_idx,
                        self.tail_k[layer], self.scale, ns, self._work, rotate=self.rot)
        return out.to(self.dtype)

    def dequantize(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """The cached K, V of `layer` as [B, Hkv, n, D] in self.dtype, rotated back if the cache rotates
        (testing only; kushkash/cache.py:203-208)."""
        k, v = cached_kv(self.pool[layer], self.block_table, self._len[layer], self.tail_k[layer], self.D,
                         self.bits, self.dtype, self.P)
        if self.rot:
            k, v = self._rotate(k), self._rotate(v)
        return k, v

    # ---------------------------------------------------------------- CUDA-graph support
    def freeze(self, max_tokens: int) -> None:
        """Pre-map pages for `max_tokens` per sequence and fix the split-KV factor, so decode steps do no host-side
        allocation and can be captured in a CUDA graph (kushkash/cache.py:211-221)."""
        self._map(-(-max_tokens // self.P))
        self._frozen_ns = self.ops.splits(self.B, self.H, max_tokens // self.P)
        need = self.ops.work_size(self.B, self.H, self._frozen_ns)
        if self._work.numel() < need:
            self._work = torch.empty(need, dtype=torch.float32, device=self.device)
        self._capacity = max_tokens

    def advance(self, steps: int = 1) -> None:
        """Host bookkeeping after replaying `steps` captured decode steps (kushkash/cache.py:223-228)."""
        if max(self._len) + steps > self._capacity:
            raise RuntimeError(f"cache capacity {self._capacity} exceeded")
        self._len = [n + steps for n in self._len]

    def reset(self) -> None:
        self._len = [0] * self.L
        self.seq_lens.zero_()
        self._mapped = 0
        self._next = 0
        self._frozen_ns = 0

    def memory(self) -> MemoryStats:
        n = max(self._len)
        P = self.P
        return MemoryStats(
            tokens=n,
            quantized_bytes=self.L * self.B * -(-n // P) * self.H * self.RB,
            tail_bytes=self.tail_k.numel() * self.tail_k.element_size(),
            reserved_bytes=self.pool.numel() + self.tail_k.numel() * self.tail_k.element_size(),
            fp16_bytes=self.L * self.B * self.H * n * self.D * 2 * 2,
        )
