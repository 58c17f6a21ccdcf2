"""Per-step metadata built on the device (kush_sm100_write_jobs, kush_sm100_unpack_plan) against the host-side
construction kushkash's serving backends use (one job per (sequence, logical page touched) over pages_touched,
kushkash/_ops.py:343-344, sequence-major), and the writes / unpacks driven by the device lists (with their padding)
against the same launches driven by exact host lists: records, tails and packed K/V bit-identical."""
import pytest
import torch

from kushsim import make_state

pytestmark = pytest.mark.gpu


def host_jobs(qsl, lens, P):
    """The reference's job list: [(s, p) for s ... for p in pages_touched(ctx, total)] (kushkash/_ops.py:343-344)."""
    jobs = []
    for s, total in enumerate(lens):
        ctx = total - (qsl[s + 1] - qsl[s])
        if total > ctx:
            jobs += [(s, p) for p in range(ctx // P, (total - 1) // P + 1)]
    return jobs


def step_case(S, P, seed, max_ctx=300, max_new=70):
    """A chunked-prefill / decode step: per sequence a history (ctx, possibly 0) and new rows (possibly 0)."""
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(0, max_ctx, (S,), generator=g)
    new = torch.randint(0, max_new, (S,), generator=g)
    new[torch.rand(S, generator=g) < 0.3] = 1                      # decode rows
    ctx[torch.rand(S, generator=g) < 0.1] = 0                      # fresh prompts
    ctx[:3] = torch.tensor([0, P, 2 * P + 3])[:min(3, S)]
    lens = (ctx + new).tolist()
    qsl = [0]
    for n in new.tolist():
        qsl.append(qsl[-1] + n)
    return qsl, lens


@pytest.mark.parametrize("S,P", [(1, 16), (7, 32), (300, 16), (2500, 16), (1500, 32)])
def test_write_jobs_match_host_list(S, P):
    from kushkash_b200 import Ops
    ops = Ops(torch.device("cuda"), 128, 4, 4, torch.bfloat16, P)
    qsl, lens = step_case(S, P, seed=S + P)
    want = host_jobs(qsl, lens, P)
    q, sl = torch.tensor(qsl, dtype=torch.int32, device="cuda"), torch.tensor(lens, dtype=torch.int32, device="cuda")
    bound = qsl[-1] // P + 2 * S
    assert len(want) <= bound
    for cap in (len(want), bound):
        js, jp, n = ops.write_jobs(q, sl, cap)
        torch.cuda.synchronize()
        assert int(n) == len(want)
        got = list(zip(js.tolist(), jp.tolist()))
        assert got[:len(want)] == want and all(s == -1 for s, _ in got[len(want):])
    if want:                                            # a capacity below the count: the lists are cut, n says so
        js, jp, n = ops.write_jobs(q, sl, max(0, len(want) - 5))
        torch.cuda.synchronize()
        assert int(n) == len(want) and list(zip(js.tolist(), jp.tolist())) == want[:max(0, len(want) - 5)]


@pytest.mark.parametrize("bits,P,fused", [(4, 16, True), (8, 32, True), (4, 32, False)])
def test_write_with_device_jobs_equals_host_jobs(bits, P, fused):
    """Two steps (a first chunk, then chunks continuing mid-page and decode rows) written once with the host's exact
    job lists and once with device-built lists padded to their bound: every record and tail byte equal."""
    from kushkash_b200 import Ops
    D, H, S = 128, 2, 40
    g = torch.Generator().manual_seed(bits + P)
    pages = 24
    bt = torch.randperm(S * pages, generator=g).to(torch.int32).view(S, pages)
    states = [make_state(S, H, D, bits, P, bt, S * pages, "cuda", torch.bfloat16) for _ in range(2)]
    ops = Ops(torch.device("cuda"), D, bits, 4, torch.bfloat16, P)
    ops.fused_write = fused
    lens = torch.zeros(S, dtype=torch.int64)
    for step in range(3):
        new = torch.randint(0, 90, (S,), generator=g) if step < 2 else torch.ones(S, dtype=torch.int64)
        qsl = torch.cat([torch.zeros(1, dtype=torch.int64), new.cumsum(0)]).to(torch.int32)
        lens = lens + new
        T = int(qsl[-1])
        k = torch.randn(T, H, D, generator=g).to("cuda", torch.bfloat16)
        v = torch.randn(T, H, D, generator=g).to("cuda", torch.bfloat16)
        jobs = host_jobs(qsl.tolist(), lens.tolist(), P)
        for i, st in enumerate(states):
            st.seq_lens.copy_(lens.to(torch.int32))
            q = qsl.cuda()
            if i == 0:
                js = torch.tensor([j[0] for j in jobs], dtype=torch.int32, device="cuda")
                jp = torch.tensor([j[1] for j in jobs], dtype=torch.int32, device="cuda")
            else:
                js, jp, _ = ops.write_jobs(q, st.seq_lens, T // P + 2 * S)
            ops.write(k, v, q, st.seq_lens, st.tail_idx, js, jp, st.pool, st.block_table, st.tail_k)
        torch.cuda.synchronize()
        assert torch.equal(states[0].pool, states[1].pool), f"records differ after step {step}"
        assert torch.equal(states[0].tail_k.view(torch.int16), states[1].tail_k.view(torch.int16))


def test_write_jobs_and_write_in_a_cuda_graph():
    """The device-built jobs and the write they drive, captured together and replayed: the same records as eager."""
    from kushkash_b200 import Ops
    D, H, S, P, bits = 128, 2, 16, 16, 4
    g = torch.Generator().manual_seed(3)
    bt = torch.randperm(S * 16, generator=g).to(torch.int32).view(S, 16)
    new = torch.randint(1, 60, (S,), generator=g)
    qsl = torch.cat([torch.zeros(1, dtype=torch.int64), new.cumsum(0)]).to(torch.int32).cuda()
    T = int(qsl[-1])
    k = torch.randn(T, H, D, generator=g).to("cuda", torch.bfloat16)
    v = torch.randn(T, H, D, generator=g).to("cuda", torch.bfloat16)
    ops = Ops(torch.device("cuda"), D, bits, 4, torch.bfloat16, P)
    cap = T // P + 2 * S
    bufs = [torch.empty(cap, dtype=torch.int32, device="cuda") for _ in range(2)] + [torch.empty(1, dtype=torch.int32,
                                                                                                  device="cuda")]
    eager, graphed = (make_state(S, H, D, bits, P, bt, S * 16, "cuda", torch.bfloat16) for _ in range(2))
    for st in (eager, graphed):
        st.seq_lens.copy_(new.to(torch.int32))

    def step(st):
        js, jp, _ = ops.write_jobs(qsl, st.seq_lens, cap, *bufs)
        ops.write(k, v, qsl, st.seq_lens, st.tail_idx, js, jp, st.pool, st.block_table, st.tail_k)

    step(eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step(graphed)                                    # warm the stream once, then start from zero again
    torch.cuda.current_stream().wait_stream(s)
    graphed.pool.zero_()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        step(graphed)
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(eager.pool, graphed.pool)


@pytest.mark.parametrize("P,bits,rot", [(16, 4, False), (32, 8, True)])
def test_unpack_plan_matches_host_plan(P, bits, rot):
    """The device plan (packed history + new rows per sequence) against the same plan built on the host, and the
    unpack it drives (with its padding) against the unpack driven by the exact host lists: kp / vp bit-identical."""
    from kushkash_b200 import Ops
    D, H, S = 128, 2, 30
    g = torch.Generator().manual_seed(P + bits)
    qsl, lens = step_case(S, P, seed=P + 1, max_ctx=200, max_new=40)
    pages = max(-(-n // P) for n in lens) + 1
    bt = torch.randperm(S * pages, generator=g).to(torch.int32).view(S, pages)
    ops = Ops(torch.device("cuda"), D, bits, 4, torch.bfloat16, P)
    st = make_state(S, H, D, bits, P, bt, S * pages, "cuda", torch.bfloat16)
    # fill the history (ctx tokens per sequence) with one bulk write
    ctx = [n - (qsl[s + 1] - qsl[s]) for s, n in enumerate(lens)]
    hq = [0]
    for c in ctx:
        hq.append(hq[-1] + c)
    Th = hq[-1]
    kh = torch.randn(Th, H, D, generator=g).to("cuda", torch.bfloat16)
    vh = torch.randn(Th, H, D, generator=g).to("cuda", torch.bfloat16)
    st.seq_lens.copy_(torch.tensor(ctx, dtype=torch.int32))
    jobs = host_jobs(hq, ctx, P)
    ops.write(kh, vh, torch.tensor(hq, dtype=torch.int32, device="cuda"), st.seq_lens, st.tail_idx,
              torch.tensor([j[0] for j in jobs], dtype=torch.int32, device="cuda"),
              torch.tensor([j[1] for j in jobs], dtype=torch.int32, device="cuda"), st.pool, st.block_table, st.tail_k)
    st.seq_lens.copy_(torch.tensor(lens, dtype=torch.int32))
    T = qsl[-1]
    kn = torch.randn(T, H, D, generator=g).to("cuda", torch.bfloat16)
    vn = torch.randn(T, H, D, generator=g).to("cuda", torch.bfloat16)
    # host plan
    base, pb, pd, tb, ti, nd = [], [], [], [], [], []
    row = 0
    for s in range(S):
        base.append(row)
        full, rem = divmod(ctx[s], P)
        pb += bt[s, :full].tolist()
        pd += [row + p * P for p in range(full)]
        if rem:
            tb.append(int(bt[s, full]))
            ti += [row + full * P, rem, int(st.tail_idx[s])]
        nd += [row + ctx[s] + t for t in range(qsl[s + 1] - qsl[s])]
        row += lens[s]
    base.append(row)
    plan = ops.unpack_plan(torch.tensor(qsl, dtype=torch.int32, device="cuda"), st.seq_lens, st.tail_idx,
                           st.block_table, len(pb) + 7, S, T)
    torch.cuda.synchronize()
    assert plan["counts"].tolist() == [len(pb), len(tb), T, row]
    assert plan["kv_start"].tolist() == base
    assert plan["page_blk"][:len(pb)].tolist() == pb and (plan["page_blk"][len(pb):] == -1).all()
    assert plan["page_dst"][:len(pd)].tolist() == pd
    assert plan["tail_blk"][:len(tb)].tolist() == tb and (plan["tail_blk"][len(tb):] == -1).all()
    assert plan["tail_info"][:len(ti)].tolist() == ti
    assert plan["new_dst"].tolist() == nd
    i32 = dict(dtype=torch.int32, device="cuda")
    outs = []
    for lists in ((torch.tensor(pb, **i32), torch.tensor(pd, **i32), torch.tensor(tb, **i32), torch.tensor(ti, **i32),
                   torch.tensor(nd, **i32)),
                  (plan["page_blk"], plan["page_dst"], plan["tail_blk"], plan["tail_info"], plan["new_dst"])):
        kp = torch.full((row, H, D), float("nan"), dtype=torch.bfloat16, device="cuda")
        vp = torch.full_like(kp, float("nan"))
        ops.unpack(st.pool, lists[0], lists[1], lists[2], lists[3], st.tail_k, kn, vn, lists[4], kp, vp, rot)
        outs.append((kp, vp))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert not torch.isnan(a.float()).any()
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
