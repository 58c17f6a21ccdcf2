"""TEST INFRASTRUCTURE, NOT PRODUCT CODE: ctypes bindings for the CPU oracle (libkush_oracle.so, a C restatement
of kushkash/kush/cpu.mojo).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, as the
checker; the product package kushkash_b200 never imports it.

`OracleOps` mirrors the CPU branch of the reference's operator surface (kushkash/_ops.py:42-213: append, write,
decode, fwht, unpack) on fp32 CPU tensors, plus the page size P (16 or 32) that the reference fixes at 32.
"""
from __future__ import annotations

import ctypes
import subprocess
from functools import lru_cache
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB = HERE / "libkush_oracle.so"

_I, _F = ctypes.c_int64, ctypes.c_float
# argument lists of kushkash/_cpu.py:10-24 (the `_p` variants take the page size first)
_SIGS = {
    "kush_cpu_append": [_I] * 18,
    "kush_cpu_write": [_I] * 20,
    "kush_cpu_decode": [_I] * 14 + [_F, _I],
    "kush_cpu_fwht": [_I] * 3,
    "kush_cpu_unpack": [_I] * 22,
    "kush_cpu_append_p": [_I] * 19,
    "kush_cpu_write_p": [_I] * 21,
    "kush_cpu_decode_p": [_I] * 15 + [_F, _I],
    "kush_cpu_unpack_p": [_I] * 23,
}


def build() -> Path:
    """Compile the oracle with its Makefile (gcc, no fast-math) if the library is missing or stale."""
    src = HERE / "kush_oracle.c"
    if not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


@lru_cache(None)
def lib() -> ctypes.CDLL:
    build()
    dll = ctypes.CDLL(str(LIB))
    for name, args in _SIGS.items():
        fn = getattr(dll, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int32
    dll.kush_oracle_set_threads.argtypes = [_I]
    dll.kush_oracle_set_threads.restype = ctypes.c_int
    dll.kush_oracle_f2h.argtypes = [ctypes.c_float]
    dll.kush_oracle_f2h.restype = ctypes.c_uint16
    dll.kush_oracle_h2f.argtypes = [ctypes.c_uint16]
    dll.kush_oracle_h2f.restype = ctypes.c_float
    return dll


def call(name: str, *args) -> None:
    """Same error behaviour as kushkash/_cpu.py:38-40: a -1 return is a ValueError."""
    if getattr(lib(), name)(*args) != 0:
        raise ValueError(f"{name}: unsupported head_dim/bits (CPU supports head_dim 64/128/256, bits 4/8)")


def set_threads(n: int) -> int:
    """Threads of the decode task pool (0 = OpenMP default); returns the count in use."""
    return int(lib().kush_oracle_set_threads(n))


def record_bytes(head_dim: int, bits: int, page: int = 32) -> int:
    """Bytes of one (page, kv head) record (kushkash/kush/quant.mojo:60-62 with P tokens)."""
    dc = head_dim if bits == 8 else head_dim // 2
    return 2 * page * dc + 4 * head_dim + 4 * page


def _byte_strides(cache: torch.Tensor) -> tuple[int, int]:
    e = cache.element_size()
    return cache.stride(0) * e, cache.stride(1) * e


class OracleOps:
    """The reference's CPU operator path (kushkash/_ops.py:42-213), page size P.  Every float tensor must be fp32
    and on the CPU; index tensors int32."""

    def __init__(self, head_dim: int, bits: int, group: int, page: int = 32):
        if head_dim not in (64, 128, 256):
            raise ValueError("CPU head_dim must be 64, 128 or 256")
        self.D, self.bits, self.G, self.P = head_dim, bits, group, page

    def append(self, k, v, seq_lens, tail_idx, cache, block_table, tail_k, pos_offset: int, advance: bool) -> None:
        S, H = k.shape[0], k.shape[1]
        bs, hs = _byte_strides(cache)
        call("kush_cpu_append_p", self.P, self.D, self.bits, k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0),
             seq_lens.data_ptr(), pos_offset, int(advance), cache.data_ptr(), bs, hs, tail_k.data_ptr(),
             tail_idx.data_ptr(), block_table.data_ptr(), block_table.stride(0), H, S)

    def write(self, k, v, query_start_loc, seq_lens, tail_idx, job_seq, job_page, cache, block_table, tail_k) -> None:
        n_jobs, H = job_seq.numel(), k.shape[1]
        if n_jobs == 0:
            return
        bs, hs = _byte_strides(cache)
        for mode in (0, 1):
            call("kush_cpu_write_p", self.P, self.D, self.bits, k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0),
                 query_start_loc.data_ptr(), seq_lens.data_ptr(), job_seq.data_ptr(), job_page.data_ptr(), n_jobs,
                 mode, cache.data_ptr(), bs, hs, tail_k.data_ptr(), tail_idx.data_ptr(), block_table.data_ptr(),
                 block_table.stride(0), H)

    def decode(self, q, out, cache, block_table, seq_lens, tail_idx, tail_k, scale: float) -> None:
        S, H = q.shape[0], tail_k.shape[1]
        bs, hs = _byte_strides(cache)
        call("kush_cpu_decode_p", self.P, self.D, self.bits, q.data_ptr(), out.data_ptr(), cache.data_ptr(), bs, hs,
             tail_k.data_ptr(), tail_idx.data_ptr(), block_table.data_ptr(), seq_lens.data_ptr(),
             block_table.stride(0), H, self.G, scale, S)

    def fwht(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if x.shape[-1] != self.D or not x.is_contiguous() or x.dtype != torch.float32:
            raise ValueError(f"fwht: x must be contiguous fp32 with last dim {self.D}")
        out = x.clone() if out is None else (out if out.data_ptr() == x.data_ptr() else out.copy_(x))
        rows = x.numel() // self.D
        if rows:
            call("kush_cpu_fwht", self.D, out.data_ptr(), rows)
        return out

    def unpack(self, cache, page_blk, page_dst, tail_blk, tail_info, tail_k, k_new, v_new, new_dst, kp, vp,
               rot: bool) -> None:
        H = kp.shape[1]
        bs, hs = _byte_strides(cache)
        call("kush_cpu_unpack_p", self.P, self.D, self.bits, cache.data_ptr(), bs, hs, H, page_blk.data_ptr(),
             page_dst.data_ptr(), page_blk.numel(), tail_blk.data_ptr(), tail_info.data_ptr(), tail_blk.numel(),
             tail_k.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), v_new.stride(0),
             new_dst.data_ptr(), new_dst.numel(), kp.data_ptr(), vp.data_ptr(), int(rot))

