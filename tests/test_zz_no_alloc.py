"""The allocation-free decode entry point (kush_sm100_decode_noalloc), called through the C ABI with ctypes.

It serves callers that cannot pass a scratch buffer -- an engine's decode step that must not allocate, or a C FFI
caller without a CUDA allocator -- by keeping the split-KV partials in a fixed device array inside the library.
Here its output must equal the regular entry point's (kush_sm100_decode with a caller-allocated work buffer, via
Ops.decode) bit for bit -- both run the same decode and combine kernels on the same partial layout, only at another
address -- on two calls in a row (the second one finds the first call's partials still in the shared array), and
an oversized request must be refused.  This file is named to be collected last."""
import ctypes

import pytest
import torch

from cases import decode_inputs
from kushsim import fill, make_state

pytestmark = pytest.mark.gpu


def _noalloc(ops, q, out, st, n_splits):
    from kushkash_b200._cuda import lib, raw_stream
    bs, hs = st.pool.stride(0) * st.pool.element_size(), st.pool.stride(1) * st.pool.element_size()
    c = ops.cfg
    return lib().kush_sm100_decode_noalloc(
        c.head_dim, c.bits, c.page, c.dtype_code, c.group, q.data_ptr(), out.data_ptr(), st.pool.data_ptr(), bs, hs,
        st.tail_k.data_ptr(), st.tail_idx.data_ptr(), st.block_table.data_ptr(), st.seq_lens.data_ptr(),
        st.block_table.stride(0), st.tail_k.shape[1], ctypes.c_float(q.shape[-1] ** -0.5).value, n_splits,
        q.shape[0], raw_stream(q.device.index or 0))


@pytest.mark.parametrize("n_splits", [1, 8, 64])
def test_noalloc_decode_matches_work_buffer_decode(n_splits):
    from kushkash_b200 import Ops
    from kushkash_b200._cuda import last_error
    D, bits, G, P, B, H, n = 128, 4, 4, 16, 3, 2, 40 * 16 + 9
    dt = torch.bfloat16
    c = decode_inputs(D, bits, G, P, B, H, n)
    ops = Ops(torch.device("cuda"), D, bits, G, dt, P)
    st = make_state(B, H, D, bits, P, c["block_table"], c["n_blocks"], "cuda", dt)
    fill(ops, st, c["K"], c["V"], n, dt, "cuda")
    g = torch.Generator(device="cuda").manual_seed(n_splits)
    work = torch.empty(ops.work_size(B, H, n_splits), device="cuda")
    for call in range(2):
        q = torch.randn(B, H * G, D, device="cuda", generator=g).to(dt)
        want = torch.empty_like(q)
        ops.decode(q, want, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5, n_splits, work)
        got = torch.full_like(q, float("nan"))
        rc = _noalloc(ops, q, got, st, n_splits)
        assert rc == 0, last_error()
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), \
            (call, (got.float() - want.float()).abs().max().item())


def test_noalloc_rejects_requests_beyond_the_fixed_scratch():
    from kushkash_b200 import Ops
    from kushkash_b200._cuda import KUSH_ERR_ARG, last_error
    D, G, B, H = 128, 8, 64, 8
    ops = Ops(torch.device("cuda"), D, 4, G, torch.bfloat16, 32)
    st = make_state(B, H, D, 4, 32, torch.zeros(B, 2, dtype=torch.int32), 2, "cuda", torch.bfloat16)
    q = torch.zeros(B, H * G, D, dtype=torch.bfloat16, device="cuda")
    rc = _noalloc(ops, q, torch.empty_like(q), st, 256)                 # 64*8*256*8*130 floats > 2M
    assert rc == KUSH_ERR_ARG and "scratch" in last_error()
