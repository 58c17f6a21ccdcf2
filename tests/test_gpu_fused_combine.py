"""The split-KV combine fused into the decode launch (Ops.decode(fused=True), kush_sm100_decode_fused_combine):
bit-identical to the decode followed by its combine launch, the counters back at 0 after every launch (two fused
launches in a row give the same bits), with and without rotation and a launch order, and within the decode
tolerance of the oracle."""
import pytest
import torch

from kushsim import make_state
from oracle.kush_oracle import OracleOps
from tolerance import check_decode

pytestmark = pytest.mark.gpu


def ragged_state(D, bits, G, P, dtype, lens, seed, H=2):
    """A written cache of ragged sequences (empty, tail-only, exact pages, long) on the GPU and its CPU twin."""
    from kushkash_b200 import Ops
    B = len(lens)
    pages = max(1, max(-(-n // P) for n in lens))
    g = torch.Generator().manual_seed(seed)
    bt = torch.randperm(B * pages, generator=g).to(torch.int32).view(B, pages)
    T = sum(lens)
    k = (torch.randn(T, H, D, generator=g) + 3 * torch.randn(H, D, generator=g)).to(dtype).float()
    v = torch.randn(T, H, D, generator=g).to(dtype).float()
    q = torch.randn(B, H * G, D, generator=g).to(dtype).float()
    qsl = torch.tensor([0] + lens, dtype=torch.int64).cumsum(0).to(torch.int32)
    jobs = [(s, p) for s in range(B) for p in range(-(-lens[s] // P))]
    js = torch.tensor([j[0] for j in jobs], dtype=torch.int32)
    jp = torch.tensor([j[1] for j in jobs], dtype=torch.int32)
    ops = Ops(torch.device("cuda"), D, bits, G, dtype, P)
    st = make_state(B, H, D, bits, P, bt, B * pages, "cuda", dtype)
    st.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    ops.write(k.to("cuda", dtype), v.to("cuda", dtype), qsl.cuda(), st.seq_lens, st.tail_idx, js.cuda(), jp.cuda(),
              st.pool, st.block_table, st.tail_k)
    ref = make_state(B, H, D, bits, P, bt, B * pages)
    ref.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    OracleOps(D, bits, G, P).write(k, v, qsl, ref.seq_lens, ref.tail_idx, js, jp, ref.pool, ref.block_table,
                                   ref.tail_k)
    return ops, st, ref, q, B, H


def bits_of(x):
    return x.view(torch.int32 if x.dtype == torch.float32 else torch.int16)


@pytest.mark.parametrize("D,bits,G,P,dtype", [
    (128, 4, 4, 16, torch.bfloat16),      # the BASELINE config 3 / 5 instantiation
    (128, 8, 7, 32, torch.float16),       # config 2's
    (128, 4, 7, 32, torch.bfloat16),      # configs 1 and 4
    (64, 4, 1, 16, torch.bfloat16),
    (256, 8, 8, 32, torch.float16),
    (128, 4, 12, 16, torch.bfloat16),     # two n-tiles of heads
    (128, 4, 4, 32, torch.float32),       # CUDA-core decode: its combine stays a second launch
])
@pytest.mark.parametrize("n_splits", [2, 5, 64])
def test_fused_combine_equals_two_launches(D, bits, G, P, dtype, n_splits):
    lens = [0, 1, P, 3 * P + 5, 40 * P + 7, 90 * P, 17 * P + P - 1, 2 * P]
    ops, st, ref, q, B, H = ragged_state(D, bits, G, P, dtype, lens, seed=D + bits + G + P + n_splits)
    qd = q.to("cuda", dtype).contiguous()
    args = (st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5, n_splits)
    want = torch.full((B, H * G, D), float("nan"), dtype=dtype, device="cuda")
    ops.decode(qd, want, *args, torch.empty(ops.work_size(B, H, n_splits), device="cuda"))
    work = torch.zeros(ops.work_size(B, H, n_splits, fused=True), device="cuda")
    counters = work[-B * H:].view(torch.int32)
    for call in range(2):                             # the counters start every call at 0
        got = torch.full_like(want, float("nan"))
        ops.decode(qd, got, *args, work, fused=True)
        torch.cuda.synchronize()
        assert torch.equal(bits_of(got), bits_of(want)), f"fused combine differs from decode + combine (call {call})"
        assert int(counters.abs().sum()) == 0, "fused decode left a counter non-zero"
    oracle = torch.empty(B, H * G, D)
    OracleOps(D, bits, G, P).decode(q.contiguous(), oracle, ref.pool, ref.block_table, ref.seq_lens, ref.tail_idx,
                                    ref.tail_k, D ** -0.5)
    check_decode(got, oracle, dtype, f"fused combine D{D} int{bits} G{G} P{P} splits {n_splits}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_combine_rotated_and_ordered(dtype):
    """Rotation (the merged rows rotated back by the last CTA) and a longest-first launch order."""
    D, bits, G, P, n_splits = 128, 4, 4, 16, 3
    lens = [5, 40 * P + 3, 7 * P, 0, 120 * P + 9, 33]
    ops, st, _, q, B, H = ragged_state(D, bits, G, P, dtype, lens, seed=5)
    qd = q.to("cuda", dtype).contiguous()
    args = (st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5, n_splits)
    order = ops.longest_first(st.seq_lens)
    for rotate, o in ((True, None), (False, order)):
        want = torch.empty(B, H * G, D, dtype=dtype, device="cuda")
        ops.decode(qd, want, *args, torch.empty(ops.work_size(B, H, n_splits), device="cuda"), rotate=rotate)
        work = torch.zeros(ops.work_size(B, H, n_splits, fused=True), device="cuda")
        for _ in range(2):
            got = torch.full_like(want, float("nan"))
            ops.decode(qd, got, *args, work, rotate=rotate, order=o, fused=True)
            assert torch.equal(bits_of(got), bits_of(want)), f"rotate={rotate} order={o is not None}"


def test_fused_combine_needs_counter_room():
    """The work buffer must hold the counters after the partials."""
    D, bits, G, P = 128, 4, 4, 16
    ops, st, _, q, B, H = ragged_state(D, bits, G, P, torch.bfloat16, [3 * P, 50], seed=1)
    out = torch.empty(B, H * G, D, dtype=torch.bfloat16, device="cuda")
    short = torch.zeros(ops.work_size(B, H, 4), device="cuda")
    with pytest.raises(ValueError):
        ops.decode(q.to("cuda", torch.bfloat16), out, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k,
                   D ** -0.5, 4, short, fused=True)


def test_fused_combine_many_splits():
    """16 heads x 300 splits: the unit's split factors do not fit the shared memory the fused merge stages them in,
    so its outputs are merged straight from global memory; still bit-identical to decode + combine."""
    D, bits, G, P, n_splits = 128, 4, 16, 16, 300
    ops, st, _, q, B, H = ragged_state(D, bits, G, P, torch.bfloat16, [400 * P + 3, 7, 90 * P], seed=9)
    qd = q.to("cuda", torch.bfloat16).contiguous()
    args = (st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5, n_splits)
    want = torch.empty(B, H * G, D, dtype=torch.bfloat16, device="cuda")
    ops.decode(qd, want, *args, torch.empty(ops.work_size(B, H, n_splits), device="cuda"))
    work = torch.zeros(ops.work_size(B, H, n_splits, fused=True), device="cuda")
    got = torch.full_like(want, float("nan"))
    ops.decode(qd, got, *args, work, fused=True)
    assert torch.equal(bits_of(got), bits_of(want))
