"""Kernel configuration surface of the reference's JIT build (kushkash/_build.py:112-149 GpuConfig), kept so that
callers which read `ops.cfg.tensor_cores`, `ops.cfg.warps` or `cfg.kernels()` keep working.

The reference compiles one Mojo instantiation per (head_dim, bits, group, dtype, arch) at first use; here every
instantiation is compiled ahead of time into libkush_sm100.so (kushkash_b200/build.py), so the config only selects
arguments of the C ABI.  `page` (16 or 32 tokens) is new: the reference fixes 32 (kushkash/kush/quant.mojo:16).
"""
from __future__ import annotations

from dataclasses import dataclass

PAGE = 32
DTYPES = {"float16": 0, "bfloat16": 1, "float32": 2}         # KUSH_F16 / KUSH_BF16 / KUSH_F32 of kushkash_b200.h


class BuildError(RuntimeError):
    pass


def _sm(arch: str) -> int:
    """'sm_100' -> 100, 'sm_90a' -> 90."""
    return int(arch.split("_")[1].rstrip("af"))


@dataclass(frozen=True)
class GpuConfig:
    head_dim: int
    bits: int
    group: int            # q heads per kv head
    dtype: str            # q / out / new-token dtype: float16 | bfloat16 | float32
    arch: str             # sm_XY of the device
    page: int = PAGE      # tokens per page record

    def __post_init__(self):
        if self.head_dim not in (64, 128, 256):
            raise BuildError(f"head_dim must be 64, 128 or 256, got {self.head_dim}")
        if self.bits not in (4, 8):
            raise BuildError(f"bits must be 4 or 8, got {self.bits}")
        if self.page not in (16, 32):
            raise BuildError(f"page must be 16 or 32, got {self.page}")
        if self.dtype not in DTYPES:
            raise BuildError(f"dtype must be one of {tuple(DTYPES)}, got {self.dtype}")
        if self.group < 1:
            raise BuildError(f"group must be >= 1, got {self.group}")
        if _sm(self.arch) != 100:
            raise BuildError(f"kushkash_b200 kernels are built for sm_100a (B200) only; this device is {self.arch}")

    @property
    def dtype_code(self) -> int:
        return DTYPES[self.dtype]

    @property
    def tensor_cores(self) -> bool:
        """Whether decode takes the tensor-core kernel (else the fp32 CUDA-core kernel)."""
        from . import _cuda
        return _cuda.decode_tensor_cores(self)

    @property
    def warps(self) -> int:
        """Warps per decode block."""
        return 4

    def kernels(self) -> dict[str, str]:
        """Entry point per operation (the C ABI of include/kushkash_b200.h)."""
        return {"append": "kush_sm100_append", "write": "kush_sm100_write",
                "decode": f"kush_sm100_decode[{'tensor cores' if self.tensor_cores else 'cuda cores'}]",
                "combine": "kush_sm100_combine", "fwht": "kush_sm100_fwht", "unpack": "kush_sm100_unpack"}


def config_class(page: int) -> type:
    """GpuConfig whose `page` defaults to `page`: what the drop-in installs as kushkash._build.GpuConfig, so that the
    reference's Ops, which builds GpuConfig(head_dim, bits, group, dtype, arch), gets kernels for that page size."""
    if page == PAGE:
        return GpuConfig
    if page not in (16, 32):
        raise BuildError(f"page must be 16 or 32, got {page}")

    default = page

    @dataclass(frozen=True)
    class PagedGpuConfig(GpuConfig):
        page: int = default

    PagedGpuConfig.__name__ = PagedGpuConfig.__qualname__ = f"GpuConfig{page}"
    return PagedGpuConfig
