"""GPU tests of the peer-memory output gather of KV-head sharding (kushkash_b200.shard.PeerGather).

One GPU: the gather of a single rank equals Ops.decode bit for bit (the same combine arithmetic), several slots
keep their own outputs, and the gather count advances once per gather with no wait giving up; a wait on a peer
that never gathers gives up after its limit and reports (failure detection without a fault).  Two GPUs (skipped
with fewer): each of two processes decodes half of the kv heads, and every rank's gathered [S, Hq, D] output equals
the unsharded decode bit for bit, eagerly and replayed from one CUDA graph."""
import multiprocessing as mp
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _state(D, bits, G, P, B, H, n, seed):
    from kushsim import fill, make_state
    from cases import decode_inputs
    from kushkash_b200 import Ops
    c = decode_inputs(D, bits, G, P, B, H, n)
    dtype = torch.bfloat16
    ops = Ops(torch.device("cuda"), D, bits, G, dtype, P)
    st = make_state(B, H, D, bits, P, c["block_table"], c["n_blocks"], "cuda", dtype)
    fill(ops, st, c["K"].to(dtype).float(), c["V"].to(dtype).float(), n, dtype, "cuda")
    q = c["q"].to("cuda", dtype).contiguous()
    return ops, st, q


def test_single_rank_gather_equals_decode():
    from kushkash_b200._cuda import device_error
    from kushkash_b200.shard import PeerGather, decode_gathered
    D, bits, G, P, B, H, n, ns = 128, 4, 4, 32, 3, 2, 40 * 32 + 9, 4
    ops, st, q = _state(D, bits, G, P, B, H, n, 0)
    want = torch.empty(B, H * G, D, dtype=torch.bfloat16, device="cuda")
    work = torch.empty(ops.work_size(B, H, ns), device="cuda")
    ops.decode(q, want, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5, ns, work)
    pg = PeerGather(B, H * G, D, torch.bfloat16, slots=2)
    try:
        assert pg.world == 1 and pg.rank == 0
        got = decode_gathered(ops, q, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5, ns,
                              work, pg, slot=1)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
        assert not pg.outs[0].view(torch.int16).any()                    # the other slot untouched (zero-filled)
        decode_gathered(ops, q * 2, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5, ns,
                        work, pg, slot=0)
        torch.cuda.synchronize()
        assert pg.outs[0].float().abs().sum() > 0 and torch.equal(pg.outs[1].view(torch.int16), want.view(torch.int16))
        assert pg.count.tolist() == [0, 2]                               # blocks reset, two gathers counted
        assert device_error(clear=True) == 0
    finally:
        pg.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q_out):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent
    sys.path[:0] = [str(root), str(root / "golden"), str(root.parent)]
    try:
        import datetime
        import torch.distributed as dist
        from kushkash_b200._cuda import device_error
        from kushkash_b200.shard import PeerGather, decode_gathered, kv_head_range
        from kushsim import fill, make_state
        from cases import decode_inputs
        from kushkash_b200 import Ops
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        D, bits, G, P, B, H, n, ns = 128, 4, 4, 32, 3, 4, 50 * 32 + 5, 4
        dtype = torch.bfloat16
        c = decode_inputs(D, bits, G, P, B, H, n)
        K, V = c["K"].to(dtype).float(), c["V"].to(dtype).float()
        q = c["q"].to(dev, dtype).contiguous()
        ops = Ops(dev, D, bits, G, dtype, P)
        full = make_state(B, H, D, bits, P, c["block_table"], c["n_blocks"], dev, dtype)
        fill(ops, full, K, V, n, dtype, dev)
        want = torch.empty(B, H * G, D, dtype=dtype, device=dev)
        work_f = torch.empty(ops.work_size(B, H, ns), device=dev)
        ops.decode(q, want, full.pool, full.block_table, full.seq_lens, full.tail_idx, full.tail_k, D ** -0.5, ns,
                   work_f)
        h0, h1 = kv_head_range(H, rank, world)
        mine = make_state(B, h1 - h0, D, bits, P, c["block_table"], c["n_blocks"], dev, dtype)
        fill(ops, mine, K[:, h0:h1], V[:, h0:h1], n, dtype, dev)
        qm = q[:, h0 * G:h1 * G].contiguous()
        work = torch.empty(ops.work_size(B, h1 - h0, ns), device=dev)
        pg = PeerGather(B, H * G, D, dtype, slots=2)
        ok = []

        def run(slot):
            return decode_gathered(ops, qm, mine.pool, mine.block_table, mine.seq_lens, mine.tail_idx, mine.tail_k,
                                   D ** -0.5, ns, work, pg, slot)

        got = run(0)
        torch.cuda.synchronize(dev)
        ok.append(torch.equal(got.view(torch.int16), want.view(torch.int16)))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run(1)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize(dev)
        ok.append(torch.equal(pg.outs[1].view(torch.int16), want.view(torch.int16)))
        ok.append(pg.count.tolist()[1] == 4 and device_error(clear=True) == 0)
        del g
        pg.close()
        dist.barrier()
        dist.destroy_process_group()
        q_out.put((rank, ok))
    except Exception as e:                                      # report, do not hang the parent
        q_out.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_gather_equals_unsharded_decode():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            r, v = q.get(timeout=240)
            results[r] = v
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(2):
        assert results.get(r) == [True, True, True], f"rank {r}: {results.get(r)}"


def test_gather_wait_gives_up_and_reports():
    """A wait for a peer that never gathers (world 2 on a one-rank buffer: rank 1's count stays 0) gives up after
    its limit (2 s) instead of hanging, sets bit 2 of device_error, and leaves the context usable."""
    import time
    from kushkash_b200 import _cuda
    from kushkash_b200.shard import PeerGather
    pg = PeerGather(1, 4, 64, torch.bfloat16, slots=1)
    try:
        _cuda.device_error(clear=True)
        pg.count[1] = 1                                            # this rank has made one gather
        t0 = time.monotonic()
        _cuda.check(_cuda.lib().kush_sm100_gather_wait(pg.base + pg.flags_off, 2, pg.base + pg.ctr_off,
                                                        _cuda.raw_stream(pg.device.index)), "gather_wait")
        torch.cuda.synchronize()
        waited = time.monotonic() - t0
        assert 1.5 < waited < 30, waited
        assert _cuda.device_error(clear=True) == 4
        x = torch.ones(4, device="cuda")                           # the context still works
        assert float((x * 2).sum()) == 8.0
    finally:
        pg.close()
