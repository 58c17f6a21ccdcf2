"""ctypes shim over libkush_sm100.so: the B200 replacement of the reference's Mojo/PTX loader
(kushkash/_cuda.py:14-117).

Same contract: `kernels(device, cfg)` returns {name: callable(grid, block, *args)} for append, write, decode,
combine, fwht and unpack, called with the reference's argument lists (kushkash/_ops.py:73-75, 93-96, 120, 177,
209-213: raw data_ptr() ints, int32 scalars, one float softmax scale) and launched on torch's current stream of
the device.  The callables translate the launch grid into the C ABI's sizes (include/kushkash_b200.h); the block
size the reference passes is ignored, every kernel picks its own.

There is no fallback: if the library is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes
from functools import lru_cache
from pathlib import Path

import torch

from ._build import GpuConfig

LIB_PATH = Path(__file__).resolve().parent / "libkush_sm100.so"

KUSH_OK, KUSH_ERR_UNSUPPORTED, KUSH_ERR_ARG, KUSH_ERR_CUDA = 0, -1, -2, -3

_i32, _i64, _f32, _p = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p
# argument types of every entry point declared in include/kushkash_b200.h
SIGNATURES = {
    "kush_sm100_append": [_i32, _i32, _i32, _i32, _p, _p, _i64, _i64, _p, _i32, _i32, _p, _p, _i64, _i64, _p, _p,
                          _i64, _i32, _i32, _p],
    "kush_sm100_write": [_i32, _i32, _i32, _i32, _p, _p, _i64, _i64, _p, _p, _p, _p, _p, _i32, _p, _i64, _i64, _p, _p,
                         _i64, _i32, _i32, _p],
    "kush_sm100_decode": [_i32, _i32, _i32, _i32, _i32, _p, _p, _p, _i64, _i64, _p, _p, _p, _p, _i64, _i32, _f32, _i32,
                          _p, _p, _i32, _p],
    "kush_sm100_combine": [_i32, _i32, _i32, _p, _p, _p, _i32, _i32, _i32, _p],
    "kush_sm100_append_rotated": [_i32, _i32, _i32, _i32, _p, _p, _i64, _i64, _p, _i32, _i32, _p, _p, _i64, _i64, _p,
                                  _p, _i64, _i32, _i32, _p],
    "kush_sm100_decode_rotated": [_i32, _i32, _i32, _i32, _i32, _p, _p, _p, _i64, _i64, _p, _p, _p, _p, _i64, _i32,
                                  _f32, _i32, _p, _p, _i32, _p],
    "kush_sm100_combine_rotated": [_i32, _i32, _i32, _p, _p, _p, _i32, _i32, _i32, _p],
    "kush_sm100_decode_ex": [_i32, _i32, _i32, _i32, _i32, _p, _p, _p, _i64, _i64, _p, _p, _p, _p, _i64, _i32, _f32,
                             _i32, _p, _p, _i32, _i32, _p, _p],
    "kush_sm100_order_longest_first": [_p, _i32, _i32, _p, _p],
    "kush_sm100_write_jobs": [_p, _p, _i32, _i32, _p, _p, _i32, _p, _p],
    "kush_sm100_unpack_plan": [_p, _p, _p, _p, _i64, _i32, _i32, _p, _p, _p, _i32, _p, _p, _i32, _p, _i32, _p, _p],
    "kush_sm100_decode_fused_combine": [_i32, _i32, _i32, _i32, _i32, _p, _p, _p, _i64, _i64, _p, _p, _p, _p, _i64,
                                        _i32, _f32, _i32, _p, _p, _p, _i32, _i32, _p, _p],
    "kush_sm100_decode_noalloc": [_i32, _i32, _i32, _i32, _i32, _p, _p, _p, _i64, _i64, _p, _p, _p, _p, _i64, _i32,
                                  _f32, _i32, _i32, _p],
    "kush_sm100_decode_tensor_cores": [_i32, _i32, _i32, _i32, _i32],
    "kush_sm100_fwht": [_i32, _i32, _p, _p, _i64, _i64, _i64, _p],
    "kush_sm100_unpack": [_i32, _i32, _i32, _i32, _p, _i64, _i64, _i32, _p, _p, _i32, _p, _p, _i32, _p, _p, _p, _i64,
                          _i64, _p, _i32, _p, _p, _i32, _p],
    "kush_sm100_record_bytes": [_i32, _i32, _i32],
    "kush_sm100_device_error": [_i32],
    "kush_sm100_selfcheck": [_p],
    "kush_sm100_ipc_alloc": [_i64, _p],
    "kush_sm100_ipc_free": [_p],
    "kush_sm100_ipc_handle": [_p, _p],
    "kush_sm100_ipc_open": [_p, _p],
    "kush_sm100_ipc_close": [_p],
    "kush_sm100_combine_gather": [_i32, _i32, _i32, _p, _i32, _i32, _p, _p, _i32, _i32, _i32, _p, _p, _p],
    "kush_sm100_gather_wait": [_p, _i32, _p, _p],
    "kush_sm100_last_error": [],
    "kush_sm100_version": [],
}


@lru_cache(None)
def lib() -> ctypes.CDLL:
    """Load the kernel library (built in-tree by kushkash_b200/build.py); raises if it is missing."""
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m kushkash_b200.build` "
                           "(kushkash_b200 has no CPU or PyTorch fallback)")
    dll = ctypes.CDLL(str(LIB_PATH))
    for name, args in SIGNATURES.items():
        fn = getattr(dll, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int32
    dll.kush_sm100_record_bytes.restype = ctypes.c_int64
    dll.kush_sm100_last_error.restype = ctypes.c_char_p
    dll.kush_sm100_version.restype = ctypes.c_char_p
    return dll


def last_error() -> str:
    return (lib().kush_sm100_last_error() or b"").decode()


def check(rc: int, what: str) -> None:
    """Raise on a failed call: ValueError for an unsupported configuration or a bad argument (the reference raises
    ValueError / BuildError there), RuntimeError for a CUDA error (as kushkash/_cuda.py:39-43 does)."""
    if rc == KUSH_OK:
        return
    msg = last_error() or f"status {rc}"
    if rc in (KUSH_ERR_UNSUPPORTED, KUSH_ERR_ARG):
        raise ValueError(f"launch {what}: {msg}")
    raise RuntimeError(f"launch {what}: {msg}")


def device_error(clear: bool = True) -> int:
    """Bounded-wait flags since the last clear: bit 0 a decode launch gave up (its outputs are NaN), bit 1 a bulk
    write gave up (some of its records were not written), bit 2 a peer-gather wait gave up on a peer; 0 if none."""
    rc = lib().kush_sm100_device_error(int(clear))
    if rc < 0:
        raise RuntimeError("kush_sm100_device_error: CUDA error")
    return rc


def selfcheck() -> tuple[int, int, int]:
    """Mismatch counts of the bulk write's scale arithmetic against IEEE division (levels 15, 255) and reciprocal,
    checked exhaustively on the current device; (0, 0, 0) on a correct build."""
    out = (ctypes.c_uint64 * 3)()
    check(lib().kush_sm100_selfcheck(out), "kush_sm100_selfcheck")
    return out[0], out[1], out[2]


def ipc_alloc(nbytes: int) -> int:
    """Device address of `nbytes` of zero-filled cudaMalloc memory that other processes can map."""
    p = ctypes.c_void_p()
    check(lib().kush_sm100_ipc_alloc(int(nbytes), ctypes.byref(p)), "kush_sm100_ipc_alloc")
    return int(p.value)


def ipc_free(ptr: int) -> None:
    check(lib().kush_sm100_ipc_free(ptr), "kush_sm100_ipc_free")


def ipc_handle(ptr: int) -> bytes:
    """The CUDA IPC handle (64 bytes) of an ipc_alloc allocation."""
    buf = (ctypes.c_uint8 * 64)()
    check(lib().kush_sm100_ipc_handle(ptr, buf), "kush_sm100_ipc_handle")
    return bytes(buf)


def ipc_open(handle: bytes) -> int:
    """This process's address of a peer's allocation, from its handle."""
    if len(handle) != 64:
        raise ValueError("an IPC handle has 64 bytes")
    p = ctypes.c_void_p()
    check(lib().kush_sm100_ipc_open((ctypes.c_uint8 * 64).from_buffer_copy(handle), ctypes.byref(p)),
          "kush_sm100_ipc_open")
    return int(p.value)


def ipc_close(ptr: int) -> None:
    check(lib().kush_sm100_ipc_close(ptr), "kush_sm100_ipc_close")


def raw_stream(device: int) -> int:
    """torch's current stream of `device` (the reference launches there too, kushkash/_cuda.py:55-57)."""
    return torch._C._cuda_getCurrentRawStream(device)


def decode_tensor_cores(cfg: GpuConfig) -> bool:
    rc = lib().kush_sm100_decode_tensor_cores(cfg.head_dim, cfg.bits, cfg.page, cfg.dtype_code, cfg.group)
    if rc < 0:
        raise ValueError(f"decode: unsupported configuration {cfg}")
    return rc == 1


class Kernel:
    """One operation bound to (device, config): __call__(grid, block, *args) with the reference's argument list."""

    def __init__(self, device: int, cfg: GpuConfig, name: str):
        self.device, self.cfg, self.name = device, cfg, name
        self.fn = getattr(lib(), "kush_sm100_" + name)
        self._call = getattr(self, "_" + name.removesuffix("_rotated"))    # a rotated variant takes the same arguments

    def __call__(self, grid: tuple[int, int, int], block: int, *args) -> None:
        with torch.cuda.device(self.device):
            rc = self._call(grid, *args)
        check(rc, f"kush_sm100_{self.name}")

    # gpu.mojo:207-211 argument order
    def _append(self, grid, k, v, ks, vs, seq_lens, pos_offset, advance, tail_idx, cache, bs, hs, tail_k, bt, max_pages,
                hkv):
        c = self.cfg
        return self.fn(c.head_dim, c.bits, c.page, c.dtype_code, k, v, ks, vs, seq_lens, pos_offset, advance, tail_idx,
                       cache, bs, hs, tail_k, bt, max_pages, hkv, grid[0], raw_stream(self.device))

    # gpu.mojo:241-245 argument order
    def _write(self, grid, k, v, ks, vs, qsl, seq_lens, tail_idx, job_seq, job_page, mode, cache, bs, hs, tail_k, bt,
               max_pages, hkv):
        c = self.cfg
        return self.fn(c.head_dim, c.bits, c.page, c.dtype_code, k, v, ks, vs, qsl, seq_lens, tail_idx, job_seq,
                       job_page, mode, cache, bs, hs, tail_k, bt, max_pages, hkv, grid[0], raw_stream(self.device))

    # gpu.mojo:566-571 argument order
    def _decode(self, grid, q, out, cache, bs, hs, tail_k, tail_idx, bt, seq_lens, max_pages, hkv, scale, n_splits,
                part_ml, part_o):
        c = self.cfg
        return self.fn(c.head_dim, c.bits, c.page, c.dtype_code, c.group, q, out, cache, bs, hs, tail_k, tail_idx, bt,
                       seq_lens, max_pages, hkv, scale, n_splits, part_ml or None, part_o or None, grid[0],
                       raw_stream(self.device))

    # the decode's arguments, then flags and the launch order
    def _decode_ex(self, grid, q, out, cache, bs, hs, tail_k, tail_idx, bt, seq_lens, max_pages, hkv, scale, n_splits,
                   part_ml, part_o, flags, order):
        c = self.cfg
        return self.fn(c.head_dim, c.bits, c.page, c.dtype_code, c.group, q, out, cache, bs, hs, tail_k, tail_idx, bt,
                       seq_lens, max_pages, hkv, scale, n_splits, part_ml or None, part_o or None, grid[0], flags,
                       order or None, raw_stream(self.device))

    def _order_longest_first(self, grid, seq_lens, n_seqs, order):
        return self.fn(seq_lens, n_seqs, self.cfg.page, order, raw_stream(self.device))

    # gpu.mojo:469-470 argument order
    def _combine(self, grid, out, part_ml, part_o, n_splits, hkv):
        c = self.cfg
        return self.fn(c.head_dim, c.dtype_code, c.group, out, part_ml, part_o, n_splits, hkv, grid[0],
                       raw_stream(self.device))

    # gpu.mojo:95-98 argument order
    def _fwht(self, grid, x, y, x_stride, y_stride, rows):
        c = self.cfg
        return self.fn(c.head_dim, c.dtype_code, x, y, x_stride, y_stride, rows, raw_stream(self.device))

    # gpu.mojo:303-310 argument order
    def _unpack(self, grid, cache, bs, hs, hkv, page_blk, page_dst, n_pages, tail_blk, tail_info, n_tail, tail_k, k_new,
                v_new, k_stride, v_stride, new_dst, n_new, kp, vp, rot):
        c = self.cfg
        return self.fn(c.head_dim, c.bits, c.page, c.dtype_code, cache, bs, hs, hkv, page_blk, page_dst, n_pages,
                       tail_blk, tail_info, n_tail, tail_k, k_new, v_new, k_stride, v_stride, new_dst, n_new, kp, vp, rot,
                       raw_stream(self.device))


NAMES = ("append", "write", "decode", "combine", "fwht", "unpack", "append_rotated", "decode_rotated", "combine_rotated",
         "decode_ex", "order_longest_first")


@lru_cache(None)
def kernels(device: int, cfg) -> dict[str, Kernel]:
    """{name: Kernel} for one device and configuration (kushkash/_cuda.py:106-108).  `cfg` is this package's
    GpuConfig or any object with the reference GpuConfig's fields (head_dim, bits, group, dtype, arch; page 32
    when it has none)."""
    if not isinstance(cfg, GpuConfig):
        cfg = GpuConfig(cfg.head_dim, cfg.bits, cfg.group, cfg.dtype, cfg.arch, getattr(cfg, "page", 32))
    return {name: Kernel(device, cfg, name) for name in NAMES}


def arch(device: int) -> str:
    major, minor = torch.cuda.get_device_capability(device)
    return f"sm_{major}{minor}"


def sm_count(device: int) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count
