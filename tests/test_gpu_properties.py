"""Size-independent properties of the decode at BASELINE config 3's full size (256 x 4096 tokens, 8 kv heads, int4,
page 16), over every one of the 2048 (sequence, kv head) units rather than a sample: each unit reads only its own
pages, tail and query, so the outputs cannot depend on where the pages lie, on which other sequences share the
launch, on the launch order or (beyond the merge's rounding) on the split count.  The oracle checks a sample of
these units in tests/test_gpu_configs.py; these checks cover the rest of the batch."""
import pytest
import torch

from test_gpu_configs import build
from tolerance import check_decode

pytestmark = pytest.mark.gpu

G, D, P = 4, 128, 16


@pytest.fixture(scope="module")
def config3():
    st, ops, K, V, bt = build([4096] * 256, H=8, G=G, D=D, bits=4, P=P, seed=33, outliers=2, big=15.0, spread=2.0,
                              appends=3)
    del K, V
    gen = torch.Generator().manual_seed(34)
    q = torch.randn(256, 8 * G, D, generator=gen).to("cuda", torch.bfloat16)
    return st, ops, q


def decode(ops, st, q, pool=None, bt=None, n_splits=1, **kw):
    S, H = q.shape[0], st.tail_k.shape[1]
    out = torch.full((S, H * G, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    fused = kw.get("fused", False)
    work = torch.zeros(max(1, ops.work_size(S, H, n_splits, fused)), device="cuda")
    ops.decode(q, out, st.pool if pool is None else pool, st.block_table if bt is None else bt, st.seq_lens,
               st.tail_idx, st.tail_k, D ** -0.5, n_splits, work, **kw)
    torch.cuda.synchronize()
    assert not torch.isnan(out.float()).any()
    return out


def same_bits(a, b):
    return torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_relocated_pages_give_identical_outputs(config3):
    """Every record moved to another physical block (a random permutation of the pool) and the block table remapped:
    all 2048 units' outputs bit-identical."""
    st, ops, q = config3
    want = decode(ops, st, q)
    n = st.pool.shape[0]
    perm = torch.randperm(n, generator=torch.Generator().manual_seed(5)).to("cuda")
    moved = torch.empty_like(st.pool)
    moved[perm] = st.pool
    bt = perm.to(torch.int32)[st.block_table.long()]
    assert same_bits(decode(ops, st, q, pool=moved, bt=bt), want)


def test_subset_batch_gives_identical_outputs(config3):
    """The odd sequences decoded on their own (their table rows, lengths, tails and queries only): bit-identical to
    the same sequences' outputs in the full batch."""
    st, ops, q = config3
    want = decode(ops, st, q)
    idx = torch.arange(1, 256, 2, device="cuda")

    class Sub:
        pool, tail_k = st.pool, st.tail_k
        block_table = st.block_table[idx].contiguous()
        seq_lens = st.seq_lens[idx].contiguous()
        tail_idx = st.tail_idx[idx].contiguous()

    got = decode(ops, Sub, q[idx].contiguous())
    assert same_bits(got, want[idx])


def test_split_counts_and_fused_combine(config3):
    """Splitting every sequence's pages over 3 or 8 CTAs changes only the merge's rounding: within the decode bounds
    of the unsplit outputs over the whole batch; the fused combine equals the two-launch combine bit for bit."""
    st, ops, q = config3
    one = decode(ops, st, q)
    for ns in (3, 8):
        two = decode(ops, st, q, n_splits=ns)
        check_decode(two, one.float(), torch.bfloat16, f"{ns} splits vs unsplit, all 2048 units")
        assert same_bits(decode(ops, st, q, n_splits=ns, fused=True), two)


def test_launch_order_gives_identical_outputs(config3):
    st, ops, q = config3
    order = torch.randperm(256, generator=torch.Generator().manual_seed(6)).to(device="cuda", dtype=torch.int32)
    assert same_bits(decode(ops, st, q, order=order), decode(ops, st, q))
