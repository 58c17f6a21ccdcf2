"""GPU parity at the BASELINE configurations' own sizes.

Config 1 (8 x 2048, int4, page 32, Qwen2.5-7B heads) and config 2 (64 sequences with lengths U[256, 8192], int8,
page 32, appends after a bulk prefill) are checked in full against the CPU oracle.  Configs 3 (256 x 4096, int4,
page 16, Llama-3.1-8B heads) and 4 (4 x 131072, int4, page 32, Qwen3-8B heads) are run at full size on the GPU
and checked on a sample of (sequence, kv head) units: every unit is independent (its own pages, tail and output),
so the oracle reproduces a unit from that unit's inputs alone -- a size-independent property of the path.  Pages
must be bit-exact, decode outputs within the bf16 bounds of the other GPU tests (max abs 2e-3, rel-norm 1e-2)."""
import random

import pytest
import torch

from kushsim import make_state
from oracle.kush_oracle import OracleOps
from tolerance import check_decode

pytestmark = pytest.mark.gpu

DT = torch.bfloat16


def assert_close(got, want, what):
    check_decode(got, want, DT, what)


def key_offsets(H, D, gen, outliers, big, spread):
    off = torch.randn(H, D, generator=gen) * spread
    for h in range(H):
        idx = torch.randperm(D, generator=gen)[:outliers]
        off[h, idx] = big * torch.sign(torch.randn(outliers, generator=gen))
    return off


def gpu_ops(D, bits, G, P):
    from kushkash_b200 import Ops
    return Ops(torch.device("cuda"), D, bits, G, DT, P)


def build(lens, H, G, D, bits, P, seed, outliers=4, big=20.0, spread=0.5, appends=0, make_ops=gpu_ops, dev="cuda",
          dt=DT):
    """Device state with len_s tokens per sequence: one ragged bulk write of len_s - appends tokens, then `appends`
    single-token append steps; returns the state, the ops and the (bf16-exact) inputs."""
    gen = torch.Generator().manual_seed(seed)
    S = len(lens)
    pages = [-(-n // P) for n in lens]
    W = max(pages)
    perm = torch.randperm(sum(pages), generator=gen).to(torch.int32)
    bt = torch.zeros(S, W, dtype=torch.int32)
    o = 0
    for s, p in enumerate(pages):
        bt[s, :p] = perm[o:o + p]
        o += p
    off = key_offsets(H, D, gen, outliers, big, spread)
    K = [(torch.randn(n, H, D, generator=gen) + off).to(DT) for n in lens]
    V = [torch.randn(n, H, D, generator=gen).to(DT) for n in lens]
    ops = make_ops(D, bits, G, P)
    st = make_state(S, H, D, bits, P, bt, sum(pages), dev, dt)
    bulk = [n - appends for n in lens]
    qsl = torch.tensor([0] + list(torch.tensor(bulk).cumsum(0)), dtype=torch.int32)
    jobs = [(s, p) for s in range(S) for p in range(0, -(-bulk[s] // P))]
    st.seq_lens.copy_(torch.tensor(bulk, dtype=torch.int32))
    put = lambda x: x.to(device=dev, dtype=dt if x.is_floating_point() else x.dtype)  # noqa: E731
    ops.write(put(torch.cat([k[:b] for k, b in zip(K, bulk)])), put(torch.cat([v[:b] for v, b in zip(V, bulk)])),
              put(qsl), st.seq_lens, st.tail_idx, put(torch.tensor([j[0] for j in jobs], dtype=torch.int32)),
              put(torch.tensor([j[1] for j in jobs], dtype=torch.int32)), st.pool, st.block_table, st.tail_k)
    for a in range(appends):
        ops.append(put(torch.stack([k[b + a] for k, b in zip(K, bulk)])),
                   put(torch.stack([v[b + a] for v, b in zip(V, bulk)])), st.seq_lens, st.tail_idx, st.pool,
                   st.block_table, st.tail_k, pos_offset=0, advance=True)
    return st, ops, K, V, bt


def oracle_unit(K, V, q, n, h, G, D, bits, P):
    """The oracle's records and decode output of one (sequence, kv head) unit, built from its inputs alone."""
    pages = -(-n // P)
    ro = OracleOps(D, bits, G, P)
    st = make_state(1, 1, D, bits, P, torch.arange(pages, dtype=torch.int32).view(1, pages), pages)
    k = K[:n, h:h + 1].float().contiguous()
    v = V[:n, h:h + 1].float().contiguous()
    st.seq_lens.fill_(n)
    ro.write(k, v, torch.tensor([0, n], dtype=torch.int32), st.seq_lens, st.tail_idx,
             torch.zeros(pages, dtype=torch.int32), torch.arange(pages, dtype=torch.int32), st.pool, st.block_table,
             st.tail_k)
    out = torch.empty(1, G, D)
    ro.decode(q.float().view(1, G, D).contiguous(), out, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k,
              D ** -0.5)
    return st.pool[:, 0], st.tail_k[0, 0], out[0]


def check_units(st, ops, K, V, bt, units, G, D, bits, P, seed, dev="cuda", dt=DT):
    S, H = bt.shape[0], st.tail_k.shape[1]
    gen = torch.Generator().manual_seed(seed + 1)
    q = torch.randn(S, H * G, D, generator=gen).to(DT)
    n_splits = ops.splits(S, H, int(st.seq_lens.max()) // P)
    out = torch.empty(S, H * G, D, dtype=dt, device=dev)
    work = torch.empty(max(1, ops.work_size(S, H, n_splits)), device=dev)
    ops.decode(q.to(device=dev, dtype=dt), out, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k,
               D ** -0.5, n_splits, work)
    lens = st.seq_lens.cpu().tolist()
    for s, h in units:
        check_unit(st, bt, out, s, h, lens[s], K[s], V[s], q[s, h * G:(h + 1) * G], G, D, bits, P)


def check_unit(st, bt, out, s, h, n, Ks, Vs, qs, G, D, bits, P):
    """Pages, tail rows and decode output of unit (s, h) on the device against the oracle run on that unit's inputs
    alone (Ks, Vs: [>= n, H, D] rows of sequence s; qs: its G query rows of kv head h)."""
    rec, tk, o = oracle_unit(Ks, Vs, qs, n, h, G, D, bits, P)
    pages = -(-n // P)
    got = st.pool[bt[s, :pages].long().to(st.pool.device), h].cpu()
    full = n // P
    assert torch.equal(got[:full], rec[:full]), (s, h, "full pages")
    if n % P:                                                       # partial page: V rows and their scales
        dc = D if bits == 8 else D // 2
        F = 2 * P * dc
        r = n % P
        assert torch.equal(got[full, P * dc:P * dc + r * dc], rec[full, P * dc:P * dc + r * dc]), (s, h)
        for a in (F + 4 * D, F + 4 * D + 2 * P):                  # vs, vb of the r rows
            assert torch.equal(got[full, a:a + 2 * r], rec[full, a:a + 2 * r]), (s, h, "v scales")
        assert torch.equal(st.tail_k[st.tail_idx[s].item(), h, :r].float().cpu(), tk[:r]), (s, h, "tail")
    assert_close(out[s, h * G:(h + 1) * G].cpu(), o, f"decode unit {(s, h)} n={n}")


def test_config1_full():
    """Qwen2.5-7B heads (28 q / 4 kv, D 128), int4, 8 sequences of 2048 tokens, page 32, 4 key
    channels per kv head at +-20, the rest N(0, 0.5); bulk write then one decode step."""
    st, ops, K, V, bt = build([2048] * 8, H=4, G=7, D=128, bits=4, P=32, seed=1)
    check_units(st, ops, K, V, bt, [(s, h) for s in range(8) for h in range(4)], 7, 128, 4, 32, 1)


def test_config2_full():
    """same heads, int8, 64 sequences with lengths U[256, 8192], page 32; bulk write then 16
    decode appends (the config's 16 steps), then attention."""
    rng = random.Random(2)
    lens = [rng.randint(256, 8192) for _ in range(64)]
    st, ops, K, V, bt = build(lens, H=4, G=7, D=128, bits=8, P=32, seed=2, appends=16)
    check_units(st, ops, K, V, bt, [(s, h) for s in range(64) for h in range(4)], 7, 128, 8, 32, 2)


def test_config3_full_size_sampled():
    """BASELINE config 3 at full size (256 x 4096, Llama-3.1-8B heads 32 / 8, int4, page 16, key offsets N(0, 2) and
    2 outlier channels at +-15), 5 decode appends; 24 sampled (sequence, kv head) units checked."""
    st, ops, K, V, bt = build([4096] * 256, H=8, G=4, D=128, bits=4, P=16, seed=3, outliers=2, big=15.0, spread=2.0,
                              appends=5)
    rng = random.Random(3)
    units = sorted({(rng.randrange(256), rng.randrange(8)) for _ in range(24)})
    check_units(st, ops, K, V, bt, units, 4, 128, 4, 16, 3)


def test_config4_full_size_sampled():
    """BASELINE config 4 at full size (4 x 131072, Qwen3-8B heads 32 / 8, int4, page 32, key offsets N(0, 4)),
    split-KV decode; 3 sampled units checked."""
    st, ops, K, V, bt = build([131072] * 4, H=8, G=4, D=128, bits=4, P=32, seed=4, outliers=0, big=0.0, spread=4.0,
                              appends=3)
    assert ops.splits(4, 8, 131072 // 32) > 1
    check_units(st, ops, K, V, bt, [(0, 0), (1, 5), (3, 7)], 4, 128, 4, 32, 4)


def test_config5_full_size_sampled():
    """BASELINE config 5 at its own shape: 2048 decode sequences with lognormal lengths (median 2048, sigma 0.8, cap
    16384), Llama-3.1-8B heads (32 q / 8 kv, D 128), int4, page 16, key offsets N(0, 2) plus 2 outlier channels at
    +-15 per kv head.  The caches are filled by ragged bulk writes; then one serving step as bench.py runs it: a bulk
    prefill-quantize of 32 new 2048-token prompts, a one-token append to every decode sequence and the split-KV
    decode of all 2048 in longest-first launch order.  64 sampled decode units (the longest and the shortest sequence
    among them) and 8 prompt units are checked against the oracle run on each unit's inputs alone."""
    import math
    S, H, G, D, bits, P, NPR, PL = 2048, 8, 4, 128, 4, 16, 32, 2048
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(S, generator=gen) * 0.8 + math.log(2048)
    lens = [int(min(16384, max(1, round(math.exp(v))))) for v in x.tolist()]
    off = key_offsets(H, D, gen, 2, 15.0, 2.0)
    rng = random.Random(5)
    picks = set(rng.sample(range(S), 62)) | {max(range(S), key=lens.__getitem__), min(range(S), key=lens.__getitem__)}
    units = {s: rng.randrange(H) for s in sorted(picks)}
    pr_units = {p: rng.randrange(H) for p in rng.sample(range(NPR), 8)}
    pages = [-(-(n + 1) // P) for n in lens]
    ppr = PL // P
    n_blocks = sum(pages) + NPR * ppr
    perm = torch.randperm(n_blocks, generator=gen).to(torch.int32)
    bt = torch.zeros(S, max(pages), dtype=torch.int32)
    o = 0
    for s, p in enumerate(pages):
        bt[s, :p] = perm[o:o + p]
        o += p
    bt_pr = perm[o:].view(NPR, ppr).contiguous()
    ops = gpu_ops(D, bits, G, P)
    st = make_state(S, H, D, bits, P, bt, n_blocks, "cuda", DT)
    pr = make_state(NPR, H, D, bits, P, bt_pr, 1, "cuda", DT)
    pr.pool = st.pool                                               # prompts and decode sequences share one pool
    offd = off.cuda()
    dgen = torch.Generator(device="cuda").manual_seed(55)
    kept = {}                                                       # sampled units' inputs, on the CPU

    def chunk_write(state, seqs, n_of, tag):
        s0, s1 = seqs[0], seqs[-1] + 1
        rows = [n_of(s) for s in range(s0, s1)]
        T = sum(rows)
        k = (torch.randn(T, H, D, generator=dgen, device="cuda") + offd).to(DT)
        v = torch.randn(T, H, D, generator=dgen, device="cuda").to(DT)
        qsl = torch.tensor([0] + rows, dtype=torch.int64).cumsum(0)
        npg = [-(-r // P) for r in rows]
        js = torch.tensor([i for i, m in enumerate(npg) for _ in range(m)], dtype=torch.int32)
        jp = torch.tensor([j for m in npg for j in range(m)], dtype=torch.int32)
        state.seq_lens[s0:s1] = torch.tensor(rows, dtype=torch.int32, device="cuda")
        ops.write(k, v, qsl.to(torch.int32).cuda(), state.seq_lens[s0:s1], state.tail_idx[s0:s1], js.cuda(),
                  jp.cuda(), state.pool, state.block_table[s0:s1], state.tail_k)
        for s in range(s0, s1):
            if (tag, s) in want_rows:
                a, b = int(qsl[s - s0]), int(qsl[s - s0 + 1])
                kept[(tag, s)] = (k[a:b].cpu(), v[a:b].cpu())

    want_rows = {("dec", s) for s in units} | {("pr", p) for p in pr_units}
    chunk, tok = [], 0
    for s in range(S):                                              # caches: ragged bulk writes of <= 256k tokens
        if chunk and tok + lens[s] > 262144:
            chunk_write(st, chunk, lens.__getitem__, "dec")
            chunk, tok = [], 0
        chunk.append(s)
        tok += lens[s]
    chunk_write(st, chunk, lens.__getitem__, "dec")
    # the serving step
    chunk_write(pr, list(range(NPR)), lambda p: PL, "pr")
    k_new = (torch.randn(S, H, D, generator=dgen, device="cuda") + offd).to(DT)
    v_new = torch.randn(S, H, D, generator=dgen, device="cuda").to(DT)
    ops.append(k_new, v_new, st.seq_lens, st.tail_idx, st.pool, st.block_table, st.tail_k, pos_offset=0, advance=True)
    q = torch.randn(S, H * G, D, generator=dgen, device="cuda").to(DT)
    ns = ops.splits(S, H, (max(lens) + 1) // P)
    work = torch.empty(max(1, ops.work_size(S, H, ns)), device="cuda")
    out = torch.full((S, H * G, D), float("nan"), dtype=DT, device="cuda")
    order = ops.longest_first(st.seq_lens)
    ops.decode(q, out, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5, ns, work, order=order)
    torch.cuda.synchronize()
    assert st.seq_lens.cpu().tolist() == [n + 1 for n in lens]
    bt_c = st.block_table.cpu()
    kn, vn, qc = k_new.cpu(), v_new.cpu(), q.cpu()
    for s, h in units.items():
        ks, vs = kept[("dec", s)]
        Ks, Vs = torch.cat([ks, kn[s:s + 1]]), torch.cat([vs, vn[s:s + 1]])
        check_unit(st, bt_c, out, s, h, lens[s] + 1, Ks, Vs, qc[s, h * G:(h + 1) * G], G, D, bits, P)
    btp = pr.block_table.cpu()
    for p, h in pr_units.items():                                  # prompt pages: bit-exact records
        ks, vs = kept[("pr", p)]
        rec, _, _ = oracle_unit(ks, vs, torch.zeros(G, D), PL, h, G, D, bits, P)
        got = st.pool[btp[p].long().cuda(), h].cpu()
        assert torch.equal(got, rec), ("prompt", p, h)
