"""GPU parity of the bulk write (quantize-on-write) on inputs chosen to reach every branch of the code arithmetic.

The fp16 / bf16 write is a persistent kernel with packed code arithmetic, a Markstein quotient for the scale and a
Newton-step reciprocal; the fp32 write keeps the per-token kernel.  Both must produce the oracle's pages byte for byte on
rows whose range is zero, rows whose fp16-rounded bias is off by more than half a step (codes that need the
clamp), ranges whose scale is an fp16 subnormal, and magnitudes near the fp16 limit; and the kernel's own scale
arithmetic is checked exhaustively against IEEE division and reciprocal."""
import pytest
import torch

from kushsim import fill, make_state
from oracle.kush_oracle import OracleOps

pytestmark = pytest.mark.gpu


def gpu_ops(D, bits, dtype, P):
    from kushkash_b200 import Ops
    return Ops(torch.device("cuda"), D, bits, 1, dtype, P)


def test_scale_arithmetic_selfcheck():
    from kushkash_b200._cuda import selfcheck
    assert selfcheck() == (0, 0, 0)


def edge_rows(n, D, g, dtype):
    """n rows of D values, cycling through kinds of rows: ordinary, constant, offset by 100 with a range of a few
    input ulps (the fp16 bias error exceeds half a step: clamped codes), tiny (scale an fp16 subnormal), huge
    (near the fp16 limit for fp16 inputs, 2e5 for the others), mixed sign with one outlier, and integer multiples of
    2^-24 in [-46, 45] (scale 6 * 2^-24: many codes land exactly on a rounding tie)."""
    big = 3e4 if dtype == torch.float16 else 2e5
    ulp = 100 * (2.0 ** -10 if dtype == torch.float16 else 2.0 ** -7)
    rows = []
    for r in range(n):
        kind = r % 7
        if kind == 0:
            x = torch.randn(D, generator=g)
        elif kind == 1:
            x = torch.full((D,), float(torch.randn(1, generator=g)))
        elif kind == 2:
            x = 100 + ulp * torch.randint(0, 4, (D,), generator=g).float()
        elif kind == 3:
            x = torch.randn(D, generator=g) * 1e-6
        elif kind == 4:
            x = big + big * 0.3 * torch.rand(D, generator=g)
        elif kind == 5:
            x = torch.randn(D, generator=g)
            x[int(torch.randint(0, D, (1,), generator=g))] = 40.0
        else:
            x = torch.randint(-46, 46, (D,), generator=g).float() * 2.0 ** -24
            x[0], x[1] = -46 * 2.0 ** -24, 45 * 2.0 ** -24
        rows.append(x)
    return torch.stack(rows)


def edge_inputs(D, bits, P, dtype, seed):
    """B=2, H=2, T=3P+3: K columns and V rows of every kind above (K per channel: the row kinds transposed)."""
    g = torch.Generator().manual_seed(seed)
    B, H, T = 2, 2, 3 * P + 3
    V = edge_rows(B * H * T, D, g, dtype).view(B, H, T, D)
    K = edge_rows(B * H * D, T, g, dtype).view(B, H, D, T).transpose(2, 3).contiguous()
    pages = -(-T // P)
    bt = torch.randperm(B * pages, generator=g).to(torch.int32).view(B, pages)
    return K.to(dtype).float(), V.to(dtype).float(), bt, B, H, T


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D,bits,P", [(D, b, P) for D in (64, 128, 256) for b in (4, 8) for P in (16, 32)])
@pytest.mark.parametrize("bulk", ["all", "split"])
def test_pages_edge_ranges(D, bits, P, dtype, bulk):
    K, V, bt, B, H, T = edge_inputs(D, bits, P, dtype, 10 * D + bits + P)
    nb = bt.numel()
    nbulk = T if bulk == "all" else P + 7
    ref = make_state(B, H, D, bits, P, bt, nb)
    fill(OracleOps(D, bits, 1, P), ref, K, V, nbulk, torch.float32, "cpu")
    st = make_state(B, H, D, bits, P, bt, nb, "cuda", dtype)
    fill(gpu_ops(D, bits, dtype, P), st, K, V, nbulk, dtype, "cuda")
    pool = st.pool.cpu()
    diff = (pool != ref.pool).nonzero()
    assert diff.numel() == 0, f"{diff.shape[0]} record bytes differ, first at (block, head, byte) {diff[0].tolist()}"
    assert torch.equal(st.tail_k.float().cpu(), ref.tail_k)


@pytest.mark.parametrize("bits", [4, 8])
def test_many_items_per_warp(bits):
    """More (page, head) items than 32 per resident warp (the metadata batches rotate), ragged lengths: full pages,
    partial last pages and pages that continue the tail of an earlier write, in one launch per chunk."""
    D, P, H, B = 128, 16, 8, 64
    g = torch.Generator().manual_seed(bits)
    first = torch.randint(1, 40, (B,), generator=g)
    second = torch.randint(1200, 1400, (B,), generator=g)
    pages = int((first + second).max()) // P + 1
    bt = torch.randperm(B * pages, generator=g).to(torch.int32).view(B, pages)
    from kushkash_b200 import Ops
    dtype = torch.bfloat16
    ops = Ops(torch.device("cuda"), D, bits, 1, dtype, P)
    ro = OracleOps(D, bits, 1, P)
    ref = make_state(B, H, D, bits, P, bt, B * pages)
    st = make_state(B, H, D, bits, P, bt, B * pages, "cuda", dtype)
    for lens in (first, second):
        total = lens.sum().item()
        k = torch.randn(total, H, D, generator=g).to(dtype)
        v = torch.randn(total, H, D, generator=g).to(dtype)
        qsl = torch.cat([torch.zeros(1, dtype=torch.int64), lens.cumsum(0)]).to(torch.int32)
        ctx = ref.seq_lens.clone()
        seq_lens = ctx + lens.to(torch.int32)
        jobs = [(s, p) for s in range(B) for p in range(int(ctx[s]) // P, (int(seq_lens[s]) - 1) // P + 1)]
        js = torch.tensor([j[0] for j in jobs], dtype=torch.int32)
        jp = torch.tensor([j[1] for j in jobs], dtype=torch.int32)
        ref.seq_lens.copy_(seq_lens)
        ro.write(k.float(), v.float(), qsl, ref.seq_lens, ref.tail_idx, js, jp, ref.pool, ref.block_table, ref.tail_k)
        st.seq_lens.copy_(seq_lens.cuda())
        ops.write(k.cuda(), v.cuda(), qsl.cuda(), st.seq_lens, st.tail_idx, js.cuda(), jp.cuda(), st.pool,
                  st.block_table, st.tail_k)
    assert torch.equal(st.pool.cpu(), ref.pool)
    assert torch.equal(st.tail_k.float().cpu(), ref.tail_k)
    from kushkash_b200._cuda import device_error
    assert device_error(clear=True) == 0
