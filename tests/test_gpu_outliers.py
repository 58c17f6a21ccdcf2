"""Decode parity at the reference's own outlier magnitudes.

The reference's tests put one key channel far from the rest: +40 on channel 3 over N(0, 1) keys in its CPU decode
test (kushkash tests/test_cpu.py:79-96) and +50 on channel 1 over 2 N(0, 1) keys in its GPU page test
(tests/test_gpu.py:14-33).  Here both shapes run through the sm_100a decode (tensor-core kernel for fp16 / bf16)
against the CPU oracle on the same inputs: int4 and int8, pages 16 and 32, GQA groups 4, 7 and 8, bf16 and fp16,
each with a bulk write of 45 tokens and then single-token appends across several page boundaries, the decode checked
after the bulk write and after every 23rd append (decode bounds: tests/tolerance.py, max-abs and rel-norm separately).
"""
import pytest
import torch

from kushsim import make_state, write_tokens
from oracle.kush_oracle import OracleOps
from tolerance import check_decode

pytestmark = pytest.mark.gpu

# (outlier channel, offset, key scale): kushkash tests/test_cpu.py:85 and tests/test_gpu.py:19-20
OUTLIERS = {"cpu40": (3, 40.0, 1.0), "gpu50": (1, 50.0, 2.0)}


def outlier_case(kind, bits, P, G, dtype, seed):
    ch, off, kscale = OUTLIERS[kind]
    B, H, D, bulk, appends = 2, 2, 128, 45, 70
    T = bulk + appends
    g = torch.Generator().manual_seed(seed)
    K = torch.randn(B, H, T, D, generator=g) * kscale
    K[..., ch] += off
    V = torch.randn(B, H, T, D, generator=g)
    K, V = K.to(dtype).float(), V.to(dtype).float()
    pages = -(-T // P)
    bt = torch.randperm(B * pages, generator=g).to(torch.int32).view(B, pages)
    ro, go = OracleOps(D, bits, G, P), _gpu_ops(D, bits, G, dtype, P)
    ref = make_state(B, H, D, bits, P, bt, B * pages)
    st = make_state(B, H, D, bits, P, bt, B * pages, "cuda", dtype)
    worst = [0.0, 0.0]
    n = 0
    for t1 in [bulk] + list(range(bulk + 1, T + 1)):
        write_tokens(ro, ref, K[:, :, n:t1], V[:, :, n:t1], n, torch.float32, "cpu")
        write_tokens(go, st, K[:, :, n:t1], V[:, :, n:t1], n, dtype, "cuda")
        n = t1
        if n != bulk and (n - bulk) % 23 and n != T:
            continue
        assert torch.equal(st.pool.cpu(), ref.pool), f"{kind} n={n}: pages differ from the oracle"
        q = torch.randn(B, H * G, D, generator=g).to(dtype).float()
        want = torch.empty(B, H * G, D)
        ro.decode(q, want, ref.pool, ref.block_table, ref.seq_lens, ref.tail_idx, ref.tail_k, D ** -0.5)
        for n_splits in (1, 3):
            out = torch.full((B, H * G, D), float("nan"), dtype=dtype, device="cuda")
            work = torch.empty(go.work_size(B, H, n_splits), device="cuda")
            go.decode(q.to("cuda", dtype), out, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k,
                      D ** -0.5, n_splits, work)
            e = check_decode(out, want, dtype, f"{kind} int{bits} P{P} G{G} n={n} splits={n_splits}")
            worst = [max(worst[0], e[0]), max(worst[1], e[1])]
    print(f"[outliers] {kind} int{bits} P{P} G{G} {dtype}: worst max abs {worst[0]:.3e}, rel-norm {worst[1]:.3e}")


def _gpu_ops(D, bits, G, dtype, P):
    from kushkash_b200 import Ops
    return Ops(torch.device("cuda"), D, bits, G, dtype, P)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("G", [4, 7, 8])
@pytest.mark.parametrize("P", [16, 32])
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("kind", list(OUTLIERS))
def test_decode_at_reference_outliers(kind, bits, P, G, dtype):
    outlier_case(kind, bits, P, G, dtype, seed=1000 * list(OUTLIERS).index(kind) + 100 * bits + 10 * G + P)
