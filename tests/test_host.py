"""Host-side logic on the CPU (no GPU): the C-ABI library loads and exports every entry point include/*.h declares,
configuration checks, the split-KV heuristic, format helpers, and the product's refusal of a CPU device."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def declared_entry_points() -> list[str]:
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        names += re.findall(r"^\w[\w\s\*]*?\b(kush_sm100_\w+)\s*\(", h.read_text(), re.M)
    return names


def test_library_exports_every_declared_symbol():
    from kushkash_b200._cuda import LIB_PATH, SIGNATURES, lib
    names = declared_entry_points()
    assert len(names) >= 10, names
    dll = ctypes.CDLL(str(LIB_PATH))
    for n in names:
        assert hasattr(dll, n), f"{n} declared in include/ but not exported"
        assert n in SIGNATURES, f"{n} has no ctypes signature in kushkash_b200/_cuda.py"
    assert lib().kush_sm100_version().startswith(b"kushkash_b200")


def test_record_bytes_agree():
    from kushkash_b200._cuda import lib
    from kushkash_b200 import record_bytes
    from oracle.kush_oracle import record_bytes as oracle_rb
    for D in (64, 128, 256):
        for bits in (4, 8):
            for P in (16, 32):
                assert lib().kush_sm100_record_bytes(D, bits, P) == record_bytes(D, bits, P) == oracle_rb(D, bits, P)
                assert record_bytes(D, bits, P) % 16 == 0
    assert record_bytes(128, 4) == 4736 and record_bytes(128, 8) == 8832 and record_bytes(128, 4, 16) == 2624
    assert lib().kush_sm100_record_bytes(96, 4, 32) == 0


def test_unsupported_configuration_reports_error_without_gpu():
    from kushkash_b200._cuda import KUSH_ERR_UNSUPPORTED, lib, last_error
    rc = lib().kush_sm100_fwht(96, 1, ctypes.c_void_p(16), ctypes.c_void_p(16), 96, 96, 1, None)
    assert rc == KUSH_ERR_UNSUPPORTED and "head_dim 96" in last_error()
    assert lib().kush_sm100_decode_tensor_cores(96, 4, 32, 1, 4) == KUSH_ERR_UNSUPPORTED


def test_gpu_config_validation():
    from kushkash_b200 import BuildError, GpuConfig
    GpuConfig(128, 4, 4, "bfloat16", "sm_100", 16)
    for bad in ((96, 4, 4, "bfloat16", "sm_100"), (128, 3, 4, "bfloat16", "sm_100"),
                (128, 4, 4, "float64", "sm_100"), (128, 4, 0, "bfloat16", "sm_100"),
                (128, 4, 4, "bfloat16", "sm_90")):
        with pytest.raises(BuildError):
            GpuConfig(*bad)
    with pytest.raises(BuildError):
        GpuConfig(128, 4, 4, "bfloat16", "sm_100", 64)


def test_ops_refuses_cpu_device():
    from kushkash_b200 import Ops
    with pytest.raises(ValueError, match="CUDA"):
        Ops(torch.device("cpu"), 128, 4, 4, torch.float32)


def test_split_factor():
    from kushkash_b200._ops import split_factor
    assert split_factor(256, 8, 256, 148) == 1                    # 2048 units fill the GPU
    assert split_factor(4, 8, 4096, 148) == 18                    # config 4, one GPU: 32 units x 18 = 576 CTAs
    assert split_factor(4, 4, 4096, 148) == 37                    # config 4 over 2 GPUs: 16 units x 37 = 592 CTAs
    assert split_factor(4, 2, 4096, 148) == 41                    # over 4 GPUs: ~100-page splits, >= 2 CTAs per SM
    assert split_factor(4, 1, 4096, 148) == 74                    # over 8 GPUs: 2 CTAs per SM
    assert split_factor(1, 1, 7, 148) == 1                        # too few pages to split
    assert split_factor(1, 1, 16, 148) == 1                       # >= 16 pages per split
    assert split_factor(1, 1, 64, 148) == 4
    assert split_factor(8, 4, 64, 148) == 4                       # 4 splits of 16 pages
    assert split_factor(1, 1, 10 ** 6, 148) == 256                # capped
    for S, H, n in ((1, 1, 10 ** 6), (3, 5, 999), (64, 8, 8192)):
        ns = split_factor(S, H, n, 148)
        assert 1 <= ns <= 256 and (ns == 1 or n // ns >= 16)
