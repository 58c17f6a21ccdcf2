"""Multi-rank host logic on CPU with gloo (world size 2): request partitioning and KV-head sharding with the output
gather.  Each rank runs the decode of its own shard with the CPU oracle (test infrastructure) and the gathered
result must equal the single-process decode over all heads bit for bit; request shards must cover every sequence
once and balance the tokens."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from kushkash_b200.shard import gather_heads, kv_head_range, partition_requests


def test_partition_requests_covers_and_balances():
    import random
    rng = random.Random(0)
    lens = [int(rng.lognormvariate(7.6, 0.8)) + 1 for _ in range(2048)]
    for world in (1, 2, 4, 8):
        parts = partition_requests(lens, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(lens)))
        loads = [sum(lens[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lens)
        assert parts == partition_requests(lens, world)            # deterministic on every rank
    with pytest.raises(ValueError):
        partition_requests(lens, 0)


def test_kv_head_range():
    assert [kv_head_range(8, r, 4) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert kv_head_range(8, 0, 1) == (0, 8)
    with pytest.raises(ValueError):
        kv_head_range(8, 0, 3)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q):
    import torch.distributed as dist
    from cases import decode_inputs
    from kushsim import fill, make_state
    from oracle.kush_oracle import OracleOps
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        D, bits, G, P, B, H, n = 64, 4, 2, 32, 2, 4, 100
        c = decode_inputs(D, bits, G, P, B, H, n)
        h0, h1 = kv_head_range(H, rank, world)
        hs = h1 - h0
        st = make_state(B, hs, D, bits, P, c["block_table"], c["n_blocks"])
        ops = OracleOps(D, bits, G, P)
        fill(ops, st, c["K"][:, h0:h1], c["V"][:, h0:h1], n, torch.float32, "cpu")
        out = torch.empty(B, hs * G, D)
        ops.decode(c["q"][:, h0 * G:h1 * G].contiguous(), out, st.pool, st.block_table, st.seq_lens, st.tail_idx,
                   st.tail_k, D ** -0.5)
        full = gather_heads(out)
        if rank == 0:
            q.put(full)
    finally:
        dist.destroy_process_group()


def test_kv_head_sharded_decode_gathers_to_the_unsharded_result():
    from cases import decode_inputs
    from kushsim import fill, make_state
    from oracle.kush_oracle import OracleOps
    D, bits, G, P, B, H, n = 64, 4, 2, 32, 2, 4, 100
    c = decode_inputs(D, bits, G, P, B, H, n)
    st = make_state(B, H, D, bits, P, c["block_table"], c["n_blocks"])
    ops = OracleOps(D, bits, G, P)
    fill(ops, st, c["K"], c["V"], n, torch.float32, "cpu")
    want = torch.empty(B, H * G, D)
    ops.decode(c["q"], want, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5)

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert torch.equal(got, want)
