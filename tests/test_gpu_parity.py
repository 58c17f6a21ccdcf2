"""GPU parity: the sm_100a kernels (through the C ABI, driven by kushkash_b200.Ops) against the CPU oracle on the
same seeded inputs, and against the golden fixtures from the reference's own pins.

Bars: page records, scales/biases and tails bit-exact (integer / byte work); FWHT and unpack bit-exact; decode
attention within the north-star bounds for bf16 outputs (max abs error 2e-3 and relative norm error 1e-2, each
asserted on its own) and the matching bounds for fp16 / fp32 (tests/tolerance.py)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from cases import DECODE_CASES, QUANT_CASES, decode_inputs, fwht_inputs, quant_inputs, unpack_inputs
from kushsim import fill, make_state, write_tokens
from oracle.kush_oracle import OracleOps
from tolerance import check_decode

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
ARR = np.load(GOLD / "golden.npz")
DTYPES = [torch.bfloat16, torch.float16, torch.float32]


def gpu_ops(D, bits, G, dtype, P=32):
    from kushkash_b200 import Ops
    return Ops(torch.device("cuda"), D, bits, G, dtype, P)


def exact(x, dtype):
    """The values the GPU sees for input x in `dtype`, as fp32 (what the oracle is given)."""
    return x.to(dtype).float()


def assert_close(got, want, dtype, what=""):
    """Decode bounds, max-abs and rel-norm asserted separately (tests/tolerance.py)."""
    check_decode(got, want, dtype, what)


# ---------------------------------------------------------------- quantize-on-write
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("D,bits,P", QUANT_CASES + [(256, 4, 32), (256, 8, 16)])
def test_pages_bit_exact(D, bits, P, dtype):
    c = quant_inputs(D, bits, P)
    K, V = exact(c["K"], dtype), exact(c["V"], dtype)
    ref = make_state(c["B"], c["H"], D, bits, P, c["block_table"], c["n_blocks"])
    fill(OracleOps(D, bits, 1, P), ref, K, V, c["bulk"], torch.float32, "cpu")
    st = make_state(c["B"], c["H"], D, bits, P, c["block_table"], c["n_blocks"], "cuda", dtype)
    fill(gpu_ops(D, bits, 1, dtype, P), st, K, V, c["bulk"], dtype, "cuda")
    pool = st.pool.cpu()
    diff = (pool != ref.pool).sum().item()
    assert diff == 0, f"{diff} record bytes differ from the oracle"
    if f"quant_{D}_{bits}_{P}" in ARR.files and dtype == torch.bfloat16:
        assert torch.equal(pool, torch.from_numpy(ARR[f"quant_{D}_{bits}_{P}"]))      # the reference's own pin
    assert torch.equal(st.tail_k.float().cpu(), ref.tail_k)
    assert torch.equal(st.seq_lens.cpu(), ref.seq_lens)


@pytest.mark.parametrize("bits", [4, 8])
def test_fused_write_equals_two_launches(bits):
    """mode 2 (one launch) leaves exactly the state of mode 0 then mode 1 (the reference's two launches), including
    chunks that start mid-page and end in a later partial page (the case where the two could race)."""
    D, P, H, B = 128, 16, 2, 3
    g = torch.Generator().manual_seed(5)
    bt = torch.randperm(B * 12, generator=g).to(torch.int32).view(B, 12)
    chunks = [(torch.randn(B, H, T, D, generator=g), torch.randn(B, H, T, D, generator=g)) for T in (5, 40, 1, 27, 16, 33)]
    states = []
    for fused in (True, False):
        ops = gpu_ops(D, bits, 1, torch.bfloat16, P)
        ops.fused_write = fused
        st = make_state(B, H, D, bits, P, bt, B * 12, "cuda", torch.bfloat16)
        n = 0
        for K, V in chunks:
            write_tokens(ops, st, K, V, n, torch.bfloat16, "cuda")
            n += K.shape[2]
        states.append(st)
    a, b = states
    assert torch.equal(a.pool, b.pool) and torch.equal(a.tail_k, b.tail_k)


# ---------------------------------------------------------------- decode
def decode_both(D, bits, G, P, B, H, n, dtype, n_splits=1, c=None):
    c = c or decode_inputs(D, bits, G, P, B, H, n)
    K, V, q = exact(c["K"], dtype), exact(c["V"], dtype), exact(c["q"], dtype)
    ref = make_state(B, H, D, bits, P, c["block_table"], c["n_blocks"])
    ro = OracleOps(D, bits, G, P)
    fill(ro, ref, K, V, n, torch.float32, "cpu")
    want = torch.empty(B, H * G, D)
    ro.decode(q.contiguous(), want, ref.pool, ref.block_table, ref.seq_lens, ref.tail_idx, ref.tail_k, D ** -0.5)
    ops = gpu_ops(D, bits, G, dtype, P)
    st = make_state(B, H, D, bits, P, c["block_table"], c["n_blocks"], "cuda", dtype)
    fill(ops, st, K, V, n, dtype, "cuda")
    assert torch.equal(st.pool.cpu(), ref.pool)
    out = torch.empty(B, H * G, D, dtype=dtype, device="cuda")
    work = torch.empty(ops.work_size(B, H, n_splits), device="cuda")
    ops.decode(q.to("cuda", dtype).contiguous(), out, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k,
               D ** -0.5, n_splits, work)
    return out, want, ops


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("D,bits,G,P,B,H,n", DECODE_CASES)
def test_decode_matches_oracle(D, bits, G, P, B, H, n, dtype):
    out, want, _ = decode_both(D, bits, G, P, B, H, n, dtype)
    assert_close(out, want, dtype, f"decode {D} {bits} {G} {P} {n}")


# kernel instantiations the golden-pinned cases above do not reach: D 256 int4 at pages 16 (G 8) and 32 (G 4), two
# n-tiles (G 12, 16) at int8 page 16 and D 64 page 32, one head per group at int8 page 16; each also split 3 ways
MORE_DECODE_CASES = [(256, 4, 8, 16, 1, 2, 70), (128, 8, 12, 16, 1, 2, 50), (64, 4, 16, 32, 1, 1, 40),
                     (128, 8, 1, 16, 2, 2, 33), (256, 4, 4, 32, 1, 2, 99)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D,bits,G,P,B,H,n", MORE_DECODE_CASES)
def test_decode_more_instantiations(D, bits, G, P, B, H, n, dtype):
    out, want, _ = decode_both(D, bits, G, P, B, H, n, dtype)
    assert_close(out, want, dtype, f"decode {D} {bits} {G} {P} {n}")
    out, want, _ = decode_both(D, bits, G, P, B, H, n, dtype, n_splits=3)
    assert_close(out, want, dtype, f"decode {D} {bits} {G} {P} {n} splits 3")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("G", [1, 4, 7, 8, 12])
def test_decode_gqa_groups(G, dtype):
    out, want, _ = decode_both(128, 4, G, 32, 2, 2, 333, dtype)
    assert_close(out, want, dtype, f"G={G}")


@pytest.mark.parametrize("n_splits", [2, 8, 64])
@pytest.mark.parametrize("P", [16, 32])
def test_decode_split_kv(n_splits, P):
    """Split-KV partials + combine equal the single-pass result (and the oracle), also with empty splits."""
    out, want, ops = decode_both(128, 4, 4, P, 2, 2, 40 * P + 7, torch.bfloat16, n_splits)
    assert_close(out, want, torch.bfloat16, f"splits={n_splits}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("n_splits", [1, 3, 8, 64])
def test_decode_ragged_splits(n_splits, dtype):
    """A ragged batch (0 tokens .. 200 pages, with and without tail pages) at split counts 1 to 64: the batch-wide
    page quota leaves the short sequences' later splits empty and moves each tail to the last split with pages; the
    outputs equal the oracle's at every split count (bf16: tensor-core kernel, fp32: CUDA-core kernel)."""
    D, bits, G, P, H = 128, 4, 4, 16, 2
    lens = [0, 1, 9, P, 3 * P + 5, 40 * P + 7, 200 * P, 17 * P + 15, 64 * P + 1]
    B = len(lens)
    pages = max(-(-n // P) for n in lens)
    g = torch.Generator().manual_seed(11)
    bt = torch.randperm(B * pages, generator=g).to(torch.int32).view(B, pages)
    T = sum(lens)
    k = exact(torch.randn(T, H, D, generator=g) + 3 * torch.randn(H, D, generator=g), dtype)
    v = exact(torch.randn(T, H, D, generator=g), dtype)
    q = exact(torch.randn(B, H * G, D, generator=g), dtype)
    qsl = torch.tensor([0] + lens, dtype=torch.int64).cumsum(0).to(torch.int32)
    jobs = [(s, p) for s in range(B) for p in range(-(-lens[s] // P))]
    js = torch.tensor([j[0] for j in jobs], dtype=torch.int32)
    jp = torch.tensor([j[1] for j in jobs], dtype=torch.int32)
    sl = torch.tensor(lens, dtype=torch.int32)
    ro, go = OracleOps(D, bits, G, P), gpu_ops(D, bits, G, dtype, P)
    ref = make_state(B, H, D, bits, P, bt, B * pages)
    st = make_state(B, H, D, bits, P, bt, B * pages, "cuda", dtype)
    ref.seq_lens.copy_(sl)
    st.seq_lens.copy_(sl.cuda())
    ro.write(k, v, qsl, ref.seq_lens, ref.tail_idx, js, jp, ref.pool, ref.block_table, ref.tail_k)
    go.write(k.to("cuda", dtype), v.to("cuda", dtype), qsl.cuda(), st.seq_lens, st.tail_idx, js.cuda(), jp.cuda(),
             st.pool, st.block_table, st.tail_k)
    assert torch.equal(st.pool.cpu(), ref.pool)
    want = torch.empty(B, H * G, D)
    ro.decode(q.contiguous(), want, ref.pool, ref.block_table, ref.seq_lens, ref.tail_idx, ref.tail_k, D ** -0.5)
    out = torch.full((B, H * G, D), float("nan"), dtype=dtype, device="cuda")
    work = torch.full((go.work_size(B, H, n_splits),), float("nan"), device="cuda")
    go.decode(q.to("cuda", dtype).contiguous(), out, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k,
              D ** -0.5, n_splits, work)
    assert_close(out, want, dtype, f"ragged splits={n_splits}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("n_splits", [1, 3])
def test_decode_longest_first_order(n_splits, dtype):
    """longest_first() is a permutation of the sequences by full pages, most first; a decode launched in that order
    gives the natural-order decode's outputs bit for bit (bf16: tensor-core kernel, fp32: CUDA-core kernel)."""
    D, bits, G, P, H = 128, 4, 4, 16, 2
    g = torch.Generator().manual_seed(21)
    lens = torch.randint(1, 40 * P, (37,), generator=g).tolist() + [0, 200 * P, 5 * P]
    B = len(lens)
    pages = max(-(-n // P) for n in lens)
    bt = torch.randperm(B * pages, generator=g).to(torch.int32).view(B, pages)
    ops = gpu_ops(D, bits, G, dtype, P)
    st = make_state(B, H, D, bits, P, bt, B * pages, "cuda", dtype)
    T = sum(lens)
    k = torch.randn(T, H, D, generator=g).to("cuda", dtype)
    v = torch.randn(T, H, D, generator=g).to("cuda", dtype)
    qsl = torch.tensor([0] + lens, dtype=torch.int64).cumsum(0).to(torch.int32).cuda()
    jobs = [(s, p) for s in range(B) for p in range(-(-lens[s] // P))]
    js = torch.tensor([j[0] for j in jobs], dtype=torch.int32).cuda()
    jp = torch.tensor([j[1] for j in jobs], dtype=torch.int32).cuda()
    st.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    ops.write(k, v, qsl, st.seq_lens, st.tail_idx, js, jp, st.pool, st.block_table, st.tail_k)
    order = ops.longest_first(st.seq_lens).cpu()
    assert sorted(order.tolist()) == list(range(B))
    full = [lens[s] // P for s in order.tolist()]
    assert full == sorted(full, reverse=True)
    q = torch.randn(B, H * G, D, generator=g).to("cuda", dtype)
    work = torch.empty(ops.work_size(B, H, n_splits), device="cuda")
    outs = []
    for o in (None, order.cuda()):
        out = torch.full((B, H * G, D), float("nan"), dtype=dtype, device="cuda")
        ops.decode(q, out, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5, n_splits, work,
                   order=o)
        outs.append(out)
    a, b = outs
    assert torch.equal(a.view(torch.int16 if dtype != torch.float32 else torch.int32),
                       b.view(torch.int16 if dtype != torch.float32 else torch.int32))


def test_longest_first_many_sequences():
    """5000 sequences (more than the kernel's 1024 threads), lengths up to past the 4095-page top key: a permutation,
    ranked by min(full pages, 4095) most first."""
    g = torch.Generator().manual_seed(5)
    P = 16
    lens = torch.randint(0, 70000, (5000,), generator=g, dtype=torch.int32)
    lens[:10] = 0
    ops = gpu_ops(128, 4, 4, torch.bfloat16, P)
    order = ops.longest_first(lens.cuda()).cpu().tolist()
    assert sorted(order) == list(range(5000))
    keys = [min(int(lens[s]) // P, 4095) for s in order]
    assert keys == sorted(keys, reverse=True)


def test_decode_tail_only_and_exact_page():
    for n in (1, 5, 31, 32, 33, 64):
        out, want, _ = decode_both(128, 4, 4, 32, 2, 2, n, torch.bfloat16)
        assert_close(out, want, torch.bfloat16, f"n={n}")


# ---------------------------------------------------------------- fwht / unpack
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("D", [64, 128, 256])
def test_fwht_bit_exact(D, dtype):
    x = fwht_inputs(D)
    x = x.clamp(-1e4, 1e4) if dtype == torch.float16 else x
    xd = x.to(dtype)
    want = OracleOps(D, 4, 1).fwht(xd.float()).to(dtype)
    got = gpu_ops(D, 4, 1, dtype).fwht(xd.cuda()).cpu()
    a = got.view(torch.int16) if dtype != torch.float32 else got.view(torch.int32)
    b = want.view(torch.int16) if dtype != torch.float32 else want.view(torch.int32)
    assert torch.equal(a, b), f"{(a != b).sum().item()} values differ"
    xc = xd.cuda()
    assert torch.equal(gpu_ops(D, 4, 1, dtype).fwht(xc, out=xc).cpu(), got)        # in place


def unpack_case(D, bits, P, dtype, rot, new_pad=0, out_shift=0):
    """Oracle and GPU unpack of one seeded case; new_pad > 0 gives k_new / v_new rows a stride of H * D + new_pad
    elements (views into wider buffers), which takes the element-wise copy of the new rows; out_shift > 0 starts kp and
    vp that many elements into their allocations (not 16-byte aligned: the element-wise kernel)."""
    c = unpack_inputs(D, bits, P)
    names = ("page_blk", "page_dst", "tail_blk", "tail_info", "tail_k", "k_new", "v_new", "new_dst")
    shape = (c["rows"], c["H"], D)
    args = {n: c[n] for n in names}
    for n in ("tail_k", "k_new", "v_new"):
        args[n] = exact(args[n], dtype)
    rk, rv = torch.full(shape, float("nan")), torch.full(shape, float("nan"))
    OracleOps(D, bits, 1, P).unpack(c["records"], *[args[n] for n in names], rk, rv, rot)
    # NaN-filled on the host so untouched rows carry the same NaN bit pattern as the reference's
    n_out = c["rows"] * c["H"] * D
    kp, vp = [torch.full((n_out + out_shift,), float("nan")).to(dtype).cuda()[out_shift:].view(shape) for _ in "kv"]
    gargs = [args[n].cuda().to(dtype) if n in ("tail_k", "k_new", "v_new") else args[n].cuda() for n in names]
    if new_pad:
        for i in (5, 6):
            x = gargs[i]
            wide = torch.zeros(x.shape[0], x.shape[1] * D + new_pad, dtype=dtype, device="cuda")
            wide[:, :x.shape[1] * D] = x.reshape(x.shape[0], -1)
            gargs[i] = wide[:, :x.shape[1] * D].view(x.shape[0], x.shape[1], D)
            assert gargs[i].stride(0) == x.shape[1] * D + new_pad
    gpu_ops(D, bits, 1, dtype, P).unpack(c["records"].cuda(), *gargs, kp, vp, rot)
    return kp, vp, rk, rv


@pytest.mark.parametrize("rot", [False, True])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("P", [16, 32])
@pytest.mark.parametrize("D,bits", [(64, 4), (128, 4), (256, 4), (128, 8), (64, 8), (256, 8)])
def test_unpack_bit_exact(D, bits, P, dtype, rot):
    kp, vp, rk, rv = unpack_case(D, bits, P, dtype, rot)
    for got, want in ((kp.cpu(), rk.to(dtype)), (vp.cpu(), rv.to(dtype))):
        a = got.view(torch.int16) if dtype != torch.float32 else got.view(torch.int32)
        b = want.view(torch.int16) if dtype != torch.float32 else want.view(torch.int32)
        assert torch.equal(a, b), f"{(a != b).sum().item()} of {a.numel()} values differ"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("pad", [1, 3, 8])
def test_unpack_strided_new_rows(pad, dtype):
    """New rows whose row stride is not a multiple of 16 bytes (pad 1, 3) and one that is (pad 8)."""
    kp, vp, rk, rv = unpack_case(128, 4, 16, dtype, False, new_pad=pad)
    for got, want in ((kp.cpu(), rk.to(dtype)), (vp.cpu(), rv.to(dtype))):
        a = got.view(torch.int16) if dtype != torch.float32 else got.view(torch.int32)
        b = want.view(torch.int16) if dtype != torch.float32 else want.view(torch.int32)
        assert torch.equal(a, b), f"{(a != b).sum().item()} of {a.numel()} values differ"


@pytest.mark.parametrize("rot", [False, True])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("D,bits,P", [(128, 4, 16), (64, 8, 32)])
def test_unpack_unaligned_output(D, bits, P, dtype, rot):
    """kp / vp one element off a 16-byte boundary: the element-wise kernel, same bits."""
    kp, vp, rk, rv = unpack_case(D, bits, P, dtype, rot, out_shift=1)
    assert kp.data_ptr() % 16 != 0
    for got, want in ((kp.cpu(), rk.to(dtype)), (vp.cpu(), rv.to(dtype))):
        a = got.view(torch.int16) if dtype != torch.float32 else got.view(torch.int32)
        b = want.view(torch.int16) if dtype != torch.float32 else want.view(torch.int32)
        assert torch.equal(a, b), f"{(a != b).sum().item()} of {a.numel()} values differ"


# ---------------------------------------------------------------- ragged, vLLM-style use
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("D,G,P", [(64, 3, 32), (128, 4, 16), (128, 7, 32)])
def test_ragged_mixed_batches(bits, D, G, P):
    """Sequences of different lengths; decodes (append with vLLM's pos_offset -1) and chunks mixed in one step;
    shuffled physical blocks, a padded block stride, permuted tail slots, a block-table row stride != width, and V
    as a strided view into a fused qkv buffer (the cases of the reference's tests/test_ragged.py).  GPU and oracle
    keep bit-identical pools and tails after every step; decode outputs agree."""
    import random
    dtype = torch.bfloat16
    rng = random.Random(2)
    H, n_req, W = 2, 5, 40
    n_blocks = n_req * W
    bt_all = torch.tensor(random.Random(0).sample(range(n_blocks), n_blocks), dtype=torch.int32).view(n_req, W)
    ti = torch.tensor(random.Random(1).sample(range(n_req + 3), n_req), dtype=torch.int32)
    lens = [0] * n_req
    ref = make_state(n_req, H, D, bits, P, bt_all, n_blocks, pad=48, slots=n_req + 3, tail_idx=ti, bt_pad=7)
    st = make_state(n_req, H, D, bits, P, bt_all, n_blocks, "cuda", dtype, pad=48, slots=n_req + 3, tail_idx=ti,
                    bt_pad=7)
    ro, go = OracleOps(D, bits, G, P), gpu_ops(D, bits, G, dtype, P)
    g = torch.Generator().manual_seed(3)

    def step(reqs, qlens):
        rows_k, rows_v, qsl, sl = [], [], [0], []
        for r, ql in zip(reqs, qlens):
            rows_k.append(exact(torch.randn(ql, H, D, generator=g), dtype))
            rows_v.append(exact(torch.randn(ql, H, D, generator=g), dtype))
            qsl.append(qsl[-1] + ql)
            sl.append(lens[r] + ql)
        k_all = torch.cat(rows_k)
        qkv = torch.zeros(k_all.shape[0], 3 * H * D)
        qkv[:, 2 * H * D:] = torch.cat(rows_v).flatten(1)
        q_all = exact(torch.randn(k_all.shape[0], H * G, D, generator=g), dtype)
        nd = next((i for i, ql in enumerate(qlens) if ql != 1), len(qlens))
        outs = {}
        for side, s, ops, dev, dt in (("ref", ref, ro, "cpu", torch.float32), ("gpu", st, go, "cuda", dtype)):
            kk = k_all.to(dev, dt)
            vv = qkv.to(dev, dt)[:, 2 * H * D:].view(-1, H, D)
            bt = torch.zeros(len(reqs), W + 7, dtype=torch.int32, device=dev)[:, :W]      # row stride != width
            bt.copy_(s.block_table[torch.tensor(reqs, device=dev)])
            sl_t = torch.tensor(sl, dtype=torch.int32, device=dev)
            ti_t = s.tail_idx[torch.tensor(reqs, device=dev)].contiguous()
            if nd:
                ops.append(kk[:nd], vv[:nd], sl_t[:nd], ti_t[:nd], s.pool, bt[:nd], s.tail_k, pos_offset=-1,
                           advance=False)
                o = torch.empty(nd, H * G, D, dtype=dt, device=dev)
                ops.decode(q_all[:nd].to(dev, dt).contiguous(), o, s.pool, bt[:nd], sl_t[:nd], ti_t[:nd], s.tail_k,
                           D ** -0.5)
                outs[side] = o
            if nd < len(reqs):
                jobs = [(i, p) for i in range(nd, len(reqs)) for p in range(lens[reqs[i]] // P, (sl[i] - 1) // P + 1)]
                js = torch.tensor([j[0] for j in jobs], dtype=torch.int32, device=dev)
                jp = torch.tensor([j[1] for j in jobs], dtype=torch.int32, device=dev)
                ops.write(kk, vv, torch.tensor(qsl, dtype=torch.int32, device=dev), sl_t, ti_t, js, jp, s.pool, bt,
                          s.tail_k)
        if nd:
            assert_close(outs["gpu"], outs["ref"], dtype, "ragged decode")
        assert torch.equal(st.pool.cpu(), ref.pool)
        assert torch.equal(st.tail_k.float().cpu(), ref.tail_k)
        for i, r in enumerate(reqs):
            lens[r] = sl[i]

    step([0, 1, 2], [70, 33, 5])
    step([3, 4], [31, 64])
    for _ in range(25):
        dec = [r for r in range(n_req) if rng.random() < 0.7 and lens[r] > 0]
        chk = [r for r in range(n_req) if r not in dec and rng.random() < 0.5]
        qls = [1] * len(dec) + [rng.randint(2, 40) for _ in chk]
        reqs = [r for r, ql in zip(dec + chk, qls) if lens[r] + ql <= W * P]
        qls = [ql for r, ql in zip(dec + chk, qls) if lens[r] + ql <= W * P]
        if reqs:
            step(reqs, qls)


# ---------------------------------------------------------------- rotation fused into the decode step
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("D,bits,P", [(128, 4, 16), (64, 8, 32), (256, 4, 32), (128, 8, 16)])
def test_append_rotated_equals_fwht_then_append(D, bits, P, dtype):
    """append(rotate=True) stores exactly what fwht() then append() store: pages (including the K pages the
    append completes from the tail) and tail rows, over 2 P + 3 steps."""
    H, B = 2, 3
    g = torch.Generator().manual_seed(D + bits + P)
    steps = 2 * P + 3
    pages = -(-steps // P)
    bt = torch.randperm(B * pages, generator=g).to(torch.int32).view(B, pages)
    ops = gpu_ops(D, bits, 1, dtype, P)
    st_a = make_state(B, H, D, bits, P, bt, B * pages, "cuda", dtype)
    st_b = make_state(B, H, D, bits, P, bt, B * pages, "cuda", dtype)
    off = torch.randn(H, D, generator=g) * 3
    for _ in range(steps):
        k = (torch.randn(B, H, D, generator=g) + off).to("cuda", dtype)
        v = torch.randn(B, H, D, generator=g).to("cuda", dtype)
        ops.append(ops.fwht(k), ops.fwht(v), st_a.seq_lens, st_a.tail_idx, st_a.pool, st_a.block_table, st_a.tail_k,
                   pos_offset=0, advance=True)
        ops.append(k, v, st_b.seq_lens, st_b.tail_idx, st_b.pool, st_b.block_table, st_b.tail_k, pos_offset=0,
                   advance=True, rotate=True)
    assert torch.equal(st_a.pool, st_b.pool)
    assert torch.equal(st_a.tail_k, st_b.tail_k) and torch.equal(st_a.seq_lens, st_b.seq_lens)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n_splits", [1, 3])
@pytest.mark.parametrize("D,bits,G,P,n", [(128, 4, 4, 16, 150), (64, 8, 3, 32, 77), (256, 4, 2, 32, 100)])
def test_decode_rotated(D, bits, G, P, n, n_splits, dtype):
    """decode(rotate=True) over a rotated cache equals the oracle's fwht(q) -> decode -> fwht(out) (fp32) within the
    decode tolerance, as the unfused GPU sequence does (bf16 / fp16: tensor-core kernel; fp32: CUDA-core kernel)."""
    B, H = 2, 2
    c = decode_inputs(D, bits, G, P, B, H, n)
    ro, ops = OracleOps(D, bits, G, P), gpu_ops(D, bits, G, dtype, P)
    K, V, q = exact(c["K"], dtype), exact(c["V"], dtype), exact(c["q"], dtype)
    Kr, Vr = exact(ro.fwht(K.contiguous()), dtype), exact(ro.fwht(V.contiguous()), dtype)   # the rotated cache
    ref = make_state(B, H, D, bits, P, c["block_table"], c["n_blocks"])
    fill(ro, ref, Kr, Vr, n, torch.float32, "cpu")
    want = torch.empty(B, H * G, D)
    ro.decode(ro.fwht(q.contiguous()), want, ref.pool, ref.block_table, ref.seq_lens, ref.tail_idx, ref.tail_k,
              D ** -0.5)
    want = ro.fwht(want)
    st = make_state(B, H, D, bits, P, c["block_table"], c["n_blocks"], "cuda", dtype)
    fill(ops, st, Kr, Vr, n, dtype, "cuda")
    assert torch.equal(st.pool.cpu(), ref.pool)
    work = torch.empty(ops.work_size(B, H, n_splits), device="cuda")
    qd = q.to("cuda", dtype).contiguous()
    out = torch.empty(B, H * G, D, dtype=dtype, device="cuda")
    ops.decode(qd, out, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5, n_splits, work,
               rotate=True)
    assert_close(out, want, dtype, f"rotated decode D{D} int{bits} P{P} splits {n_splits}")
    unfused = torch.empty_like(out)
    ops.decode(ops.fwht(qd), unfused, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5,
               n_splits, work)
    assert_close(ops.fwht(unfused), want, dtype, "unfused")


# ---------------------------------------------------------------- errors
def test_bad_arguments_raise():
    from kushkash_b200 import Ops
    with pytest.raises(ValueError):
        Ops(torch.device("cuda"), 96, 4, 1, torch.bfloat16)
    ops = Ops(torch.device("cuda"), 128, 4, 4, torch.bfloat16)
    raw = torch.zeros(4, 2 * 4736 + 8, dtype=torch.uint8, device="cuda")
    cache = raw[:, :2 * 4736].view(4, 2, 4736)                     # block stride not a multiple of 16
    q = torch.zeros(1, 8, 128, dtype=torch.bfloat16, device="cuda")
    z = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="16-byte"):
        ops.decode(q, torch.empty_like(q), cache, torch.zeros(1, 4, dtype=torch.int32, device="cuda"), z + 40, z,
                   torch.zeros(1, 2, 32, 128, dtype=torch.bfloat16, device="cuda"), 0.1)
    with pytest.raises(ValueError, match="work buffer"):
        ops.decode(q, torch.empty_like(q), torch.zeros(4, 2, 4736, dtype=torch.uint8, device="cuda"),
                   torch.zeros(1, 4, dtype=torch.int32, device="cuda"), z + 40, z,
                   torch.zeros(1, 2, 32, 128, dtype=torch.bfloat16, device="cuda"), 0.1, n_splits=2)


def test_no_decode_watchdog_fired():
    """None of the decode launches above gave up a bounded wait."""
    from kushkash_b200._cuda import device_error
    torch.cuda.synchronize()
    assert device_error(clear=True) == 0
