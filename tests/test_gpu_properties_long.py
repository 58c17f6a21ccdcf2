"""Size-independent properties of the split-KV decode at BASELINE config 4's full size (4 x 131072 tokens, Qwen3-8B
heads 32 / 8, int4, page 32, key offsets N(0, 4)), over all 32 (sequence, kv head) units rather than a sample: the
outputs do not depend on where the pages lie (a relocated pool gives the same bits), the split count changes only the
merge's rounding, the fused combine equals the two-launch combine bit for bit, and each half of a two-way kv-head
partition -- its 4 heads' records, tail rows and q heads decoded on their own, as one GPU of the partition does --
equals those heads of the whole decode bit for bit.  The oracle checks a sample of these units in
tests/test_gpu_configs.py."""
import pytest
import torch

from test_gpu_configs import build
from tolerance import check_decode

pytestmark = pytest.mark.gpu

S, H, G, D, P = 4, 8, 4, 128, 32


@pytest.fixture(scope="module")
def config4():
    st, ops, K, V, bt = build([131072] * S, H=H, G=G, D=D, bits=4, P=P, seed=44, outliers=0, big=0.0, spread=4.0,
                              appends=3)
    del K, V
    q = torch.randn(S, H * G, D, generator=torch.Generator().manual_seed(45)).to("cuda", torch.bfloat16)
    return st, ops, q


def decode(ops, st, q, n_splits, pool=None, block_table=None, tail_k=None, fused=False):
    pool = st.pool if pool is None else pool
    block_table = st.block_table if block_table is None else block_table
    tail_k = st.tail_k if tail_k is None else tail_k
    heads = tail_k.shape[1]
    out = torch.full((q.shape[0], heads * G, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    work = torch.zeros(max(1, ops.work_size(q.shape[0], heads, n_splits, fused)), device="cuda")
    ops.decode(q, out, pool, block_table, st.seq_lens, st.tail_idx, tail_k, D ** -0.5, n_splits, work, fused=fused)
    torch.cuda.synchronize()
    assert not torch.isnan(out.float()).any()
    return out


def same_bits(a, b):
    return torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_relocated_pages_give_identical_outputs(config4):
    st, ops, q = config4
    ns = ops.splits(S, H, 131072 // P)
    assert ns > 1
    want = decode(ops, st, q, ns)
    perm = torch.randperm(st.pool.shape[0], generator=torch.Generator().manual_seed(7)).to("cuda")
    moved = torch.empty_like(st.pool)
    moved[perm] = st.pool
    assert same_bits(decode(ops, st, q, ns, pool=moved, block_table=perm.to(torch.int32)[st.block_table.long()]),
                     want)


def test_split_counts_and_fused_combine(config4):
    st, ops, q = config4
    ns = ops.splits(S, H, 131072 // P)
    base = decode(ops, st, q, ns)
    for other in (2, 37, 100):
        got = decode(ops, st, q, other)
        check_decode(got, base.float(), torch.bfloat16, f"{other} splits vs {ns}, all 32 units")
        if other != 2:
            assert same_bits(decode(ops, st, q, other, fused=True), got)


def test_kv_head_halves_equal_the_whole(config4):
    """The pool viewed at heads [h0, h0 + 4) (byte strides of the whole pool), those heads' tail rows and q heads:
    bit-identical to the same heads of the 8-head decode at the same split count."""
    st, ops, q = config4
    ns = ops.splits(S, H, 131072 // P)
    whole = decode(ops, st, q, ns)
    for h0 in (0, 4):
        half = decode(ops, st, q[:, h0 * G:(h0 + 4) * G].contiguous(), ns, pool=st.pool[:, h0:h0 + 4],
                      tail_k=st.tail_k[:, h0:h0 + 4].contiguous())
        assert same_bits(half, whole[:, h0 * G:(h0 + 4) * G])
