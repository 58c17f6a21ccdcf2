"""Test driver shared by the CPU-oracle tests and the GPU parity tests: one layer of cache state and the host side
of a write step, identical for the oracle (oracle/kush_oracle.py OracleOps, CPU fp32) and for the CUDA library
(kushkash_b200 Ops), so both see the same inputs and the same call sequence."""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class State:
    pool: torch.Tensor          # [n_blocks, H, RB] uint8 (possibly a view with a padded block stride)
    block_table: torch.Tensor   # [B, W] int32 (possibly a view with row stride > W)
    tail_k: torch.Tensor        # [slots, H, P, D]
    tail_idx: torch.Tensor      # [B] int32
    seq_lens: torch.Tensor      # [B] int32
    P: int


def make_state(B: int, H: int, D: int, bits: int, P: int, block_table: torch.Tensor, n_blocks: int,
               device="cpu", dtype=torch.float32, pad: int = 0, slots: int | None = None,
               tail_idx: torch.Tensor | None = None, bt_pad: int = 0) -> State:
    dc = D if bits == 8 else D // 2
    rb = 2 * P * dc + 4 * D + 4 * P
    raw = torch.zeros(n_blocks, H * rb + pad, dtype=torch.uint8, device=device)
    pool = raw[:, :H * rb].view(n_blocks, H, rb)
    W = block_table.shape[1]
    bt = torch.zeros(B, W + bt_pad, dtype=torch.int32, device=device)[:, :W]
    bt.copy_(block_table.to(device))
    slots = slots or B
    tail = torch.zeros(slots, H, P, D, dtype=dtype, device=device)
    ti = (tail_idx if tail_idx is not None else torch.arange(B, dtype=torch.int32)).to(device)
    return State(pool, bt, tail, ti, torch.zeros(B, dtype=torch.int32, device=device), P)


def rows_of(x: torch.Tensor, dtype, device) -> torch.Tensor:
    """[B, H, T, D] -> kernel rows [B*T, H, D] (head stride D), contiguous."""
    B, H, T, D = x.shape
    return x.transpose(1, 2).contiguous().reshape(B * T, H, D).to(device=device, dtype=dtype)


def write_tokens(ops, st: State, K: torch.Tensor, V: torch.Tensor, n0: int, dtype, device) -> None:
    """Append tokens n0 .. n0+T of every sequence (equal lengths), the way KushCache.write does
    (kushkash/cache.py:132-162): T == 1 -> append with advance, else one ragged write with one job per page."""
    B, H, T, D = K.shape
    P = st.P
    k, v = rows_of(K, dtype, device), rows_of(V, dtype, device)
    if T == 1:
        ops.append(k, v, st.seq_lens, st.tail_idx, st.pool, st.block_table, st.tail_k, pos_offset=0, advance=True)
        return
    st.seq_lens.fill_(n0 + T)
    pages = torch.arange(n0 // P, (n0 + T - 1) // P + 1, dtype=torch.int32)
    job_seq = torch.arange(B, dtype=torch.int32).repeat_interleave(pages.numel()).to(device)
    qsl = (torch.arange(B + 1, dtype=torch.int32) * T).to(device)
    ops.write(k, v, qsl, st.seq_lens, st.tail_idx, job_seq, pages.repeat(B).to(device), st.pool, st.block_table,
              st.tail_k)


def fill(ops, st: State, K: torch.Tensor, V: torch.Tensor, bulk: int, dtype, device) -> None:
    """Bulk-write the first `bulk` tokens, then append the rest one token at a time."""
    T = K.shape[2]
    if bulk:
        write_tokens(ops, st, K[:, :, :bulk], V[:, :, :bulk], 0, dtype, device)
    for t in range(bulk, T):
        write_tokens(ops, st, K[:, :, t:t + 1], V[:, :, t:t + 1], t, dtype, device)
