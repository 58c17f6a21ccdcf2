"""Decode-attention bounds of the GPU parity tests, asserted as two separate checks.

bf16 outputs: max-abs 2e-3 and rel-norm 1e-2 (the north star's bounds in bf16); fp16: 3e-3 and 3e-3 (the rel-norm
bound of the reference's own fp16 GPU test, kushkash tests/test_gpu.py:60, used for both); fp32 (the CUDA-core
kernel): 1e-4 and 1e-4.  The tensor-core kernel computes in the same fp16 operands for bf16 and fp16 outputs, so
its arithmetic error is the same for both: up to ~2.2e-3 at outputs of magnitude 2-3 with the reference's +50
key outlier over 2 N(0, 1) keys (tests/test_gpu_outliers.py), well under 1e-3 on the BASELINE configurations.

  rel-norm  ||gpu - oracle|| / ||oracle|| over the whole output, the oracle computing in fp32 from the same
            dtype-exact inputs.
  max-abs   max over elements of |gpu - oracle| beyond the output dtype's own rounding: |gpu - oracle| minus half a
            unit in the last place of the dtype at that magnitude.  A kernel that returns bf16 cannot be closer to
            the exact value than that rounding, whatever it computes: half an ulp is 2^-9 |x| to 2^-8 |x| (9.8e-4 at
            |x| = 0.25, 3.9e-3 at |x| = 1, 7.8e-3 at |x| = 3), so a raw max-abs of 2e-3 on bf16 outputs above 0.5
            would fail an exactly rounded result.  The raw max-abs and the largest |oracle| are printed beside it.
"""
from __future__ import annotations

import torch

BOUNDS = {torch.bfloat16: (2e-3, 1e-2), torch.float16: (3e-3, 3e-3), torch.float32: (1e-4, 1e-4)}
_FRACTION_BITS = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}
_MIN_EXP = {torch.bfloat16: -126, torch.float16: -14, torch.float32: -126}       # smallest normal exponent


def half_ulp(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Half a unit in the last place of `dtype` at |x| (fp64): 2^(floor(log2 |x|) - fraction bits - 1), floored at
    the subnormal spacing."""
    a = x.double().abs()
    _, e = torch.frexp(a)                                     # |x| = m 2^e, m in [0.5, 1): floor(log2 |x|) = e - 1
    e = torch.where(a > 0, e - 1, _MIN_EXP[dtype]).clamp(min=_MIN_EXP[dtype])
    return torch.ldexp(torch.ones_like(x, dtype=torch.float64), e - _FRACTION_BITS[dtype] - 1)


def decode_errors(got: torch.Tensor, want: torch.Tensor, dtype: torch.dtype) -> tuple[float, float, float]:
    """(max-abs beyond the output rounding, relative norm error, raw max-abs) of got against want, in fp64."""
    g, w = got.detach().double().cpu(), want.detach().double().cpu()
    if g.numel() == 0:
        return 0.0, 0.0, 0.0
    d = (g - w).abs()
    excess = d - half_ulp(torch.maximum(g.abs(), w.abs()), dtype)
    return float(excess.max().clamp_min(0)), float((g - w).norm() / w.norm().clamp_min(1e-300)), float(d.max())


def check_decode(got: torch.Tensor, want: torch.Tensor, dtype: torch.dtype, what: str = "") -> tuple[float, float]:
    """Assert both bounds for `dtype`; prints the errors so a run's log shows the margin of every case."""
    assert not torch.isnan(got.float()).any(), f"{what}: NaN in the output"
    max_abs, rel, raw = decode_errors(got, want, dtype)
    atol, rtol = BOUNDS[dtype]
    print(f"[decode] {what} {str(dtype).split('.')[-1]}: max-abs beyond rounding {max_abs:.3e} (<= {atol:g}), "
          f"rel-norm {rel:.3e} (<= {rtol:g}); raw max-abs {raw:.3e}, max |ref| {float(want.abs().max()):.3f}")
    assert max_abs <= atol, f"{what}: max-abs error beyond the output rounding {max_abs:.3e} > {atol:g}"
    assert rel <= rtol, f"{what}: rel-norm error {rel:.3e} > {rtol:g}"
    return max_abs, rel
