"""Seeded inputs shared by the golden-fixture generator (make_golden.py) and the tests.

Everything here is plain PyTorch on the CPU with explicit torch.Generator seeds, so the same tensors come out
wherever the tests run.  Float inputs are rounded to bf16 first: the values are then exact in bf16, fp16-free
fp32 and the kernels' bf16 path alike, so one fixture pins every input dtype.
"""
from __future__ import annotations

import torch

# (D, bits, P) grid of the quantize-on-write fixtures; P = 32 is kushkash's page, P = 16 the same layout at 16 rows
QUANT_CASES = [(D, bits, P) for D in (64, 128) for bits in (4, 8) for P in (16, 32)]
# (D, bits, G, P, B, H, n) decode fixtures: full pages + a partial page, tail-only, one page exactly, GQA groups
DECODE_CASES = [
    (128, 4, 4, 32, 2, 2, 150),
    (128, 8, 7, 32, 2, 2, 77),
    (64, 4, 1, 32, 1, 2, 31),
    (128, 4, 8, 32, 1, 2, 64),
    (256, 8, 2, 32, 1, 2, 100),
    (128, 4, 4, 16, 2, 2, 150),
    (64, 8, 3, 16, 2, 2, 45),
]


def bf16_exact(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


def record_bytes(D: int, bits: int, P: int) -> int:
    dc = D if bits == 8 else D // 2
    return 2 * P * dc + 4 * D + 4 * P


def quant_inputs(D: int, bits: int, P: int):
    """B=2 sequences, H=2 kv heads, T = 2P + 5 tokens (two full pages, one partial), K with an outlier channel;
    the first P + 7 tokens are one bulk write, the rest single-token appends.  Pages of the pool are a seeded
    permutation."""
    g = torch.Generator().manual_seed(1000 * D + 10 * bits + P)
    B, H, T = 2, 2, 2 * P + 5
    K = torch.randn(B, H, T, D, generator=g) * 3
    K[..., 1] += 50
    V = torch.randn(B, H, T, D, generator=g)
    pages = -(-T // P)
    perm = torch.randperm(B * pages, generator=g).to(torch.int32).view(B, pages)
    return dict(K=bf16_exact(K), V=bf16_exact(V), B=B, H=H, T=T, bulk=P + 7, block_table=perm, n_blocks=B * pages)


def decode_inputs(D: int, bits: int, G: int, P: int, B: int, H: int, n: int):
    """K with per-channel offsets (4 channels at +-20 like BASELINE config 1, the rest N(0, 0.5)), V N(0,1),
    q N(0,1); seeded page permutation with room for ceil(n/P) pages per sequence."""
    g = torch.Generator().manual_seed(7 * D + 3 * bits + 11 * G + P + 13 * n)
    off = torch.randn(H, 1, D, generator=g) * 0.5
    idx = torch.randperm(D, generator=g)[:4]
    off[:, :, idx] = 20 * torch.sign(torch.randn(H, 1, 4, generator=g))
    K = torch.randn(B, H, n, D, generator=g) + off
    V = torch.randn(B, H, n, D, generator=g)
    q = torch.randn(B, H * G, D, generator=g)
    pages = -(-n // P)
    perm = torch.randperm(B * pages, generator=g).to(torch.int32).view(B, pages)
    return dict(K=bf16_exact(K), V=bf16_exact(V), q=bf16_exact(q), block_table=perm, n_blocks=B * pages)


def fwht_inputs(D: int) -> torch.Tensor:
    """Rows with magnitudes far apart, a zero row, a huge outlier and rounding-heavy sums (the kinds of rows the
    reference's FWHT test uses, tests/test_cpu.py:429-437, regenerated from this file's own seed)."""
    g = torch.Generator().manual_seed(D)
    x = torch.randn(203, D, generator=g)
    x[:50] *= torch.logspace(-6, 6, 50)[:, None]
    x[50, :] = 0
    x[51, 7] = 1e30
    x[52] = torch.arange(D, dtype=torch.float32) * 1e-3 + 1
    return x


def pack_records(kq, ks, kb, vq, vs, vb, D: int, bits: int, P: int) -> torch.Tensor:
    """Assemble one record [RB] uint8 from its parts (kushkash/kush/quant.mojo:53-87 layout):
    kq/vq int8 [P, D] codes, ks/kb fp16 [D], vs/vb fp16 [P]."""
    def rows(c):
        c = c.to(torch.int8)
        if bits == 4:
            lo, hi = c[:, :D // 2], c[:, D // 2:]
            c = ((lo & 0x0F) | (hi << 4)).to(torch.int8)
        return c.contiguous().view(torch.uint8).reshape(-1)
    meta = torch.cat([ks.half(), kb.half(), vs.half(), vb.half()]).contiguous().view(torch.uint8)
    return torch.cat([rows(kq), rows(vq), meta])


def unpack_inputs(D: int, bits: int, P: int = 32, seed: int = 0):
    """Seeded records with small fp16 scales / signed biases, 4 full history pages, 3 partial pages (1, P/2 + 1 and
    P - 1 tokens, K from a tail slot), 40 new rows (one full block of 32 and a partial one); one never-written row
    between every group so a stray write shows up as a non-NaN."""
    g = torch.Generator().manual_seed(100 + 17 * D + bits + P + seed)
    H, n_blk, slots = 2, 10, 3
    rb = record_bytes(D, bits, P)
    dc = D if bits == 8 else D // 2
    rec = torch.randint(0, 256, (n_blk, H, rb), dtype=torch.uint8, generator=g)
    m = rec[:, :, 2 * P * dc:].view(torch.float16)                     # [n_blk, H, 2D + 2P]
    m[:, :, :D] = (torch.rand(n_blk, H, D, generator=g) * 0.08 + 0.001).half()          # K scales
    m[:, :, D:2 * D] = ((torch.rand(n_blk, H, D, generator=g) - 0.5) * 0.5).half()       # K biases
    m[:, :, 2 * D:2 * D + P] = (torch.rand(n_blk, H, P, generator=g) * 0.08 + 0.001).half()   # V scales
    m[:, :, 2 * D + P:] = ((torch.rand(n_blk, H, P, generator=g) - 0.5) * 0.5).half()    # V biases
    tail_k = bf16_exact(torch.randn(slots, H, P, D, generator=g) * 0.7)
    page_blk = torch.tensor([3, 8, 0, 5], dtype=torch.int32)
    page_dst = torch.tensor([1, 1 + P, 2 + 2 * P, 2 + 3 * P], dtype=torch.int32)       # gaps at rows 0, 1 + 2P
    r0 = 3 + 4 * P
    tails = [(r0, 1, 2, 6), (r0 + 2, P // 2 + 1, 0, 1), (r0 + 4 + P // 2, P - 1, 1, 9)]   # (first row, n, slot, blk)
    tail_blk = torch.tensor([t[3] for t in tails], dtype=torch.int32)
    tail_info = torch.tensor([x for t in tails for x in t[:3]], dtype=torch.int32)
    n0 = r0 + 4 + P // 2 + P                                            # first row after the tails (+ a gap)
    new_dst = torch.cat([torch.arange(n0, n0 + 32), torch.arange(n0 + 33, n0 + 41)]).to(torch.int32)
    rows = n0 + 42
    k_new = bf16_exact(torch.randn(40, H, D, generator=g))
    v_new = bf16_exact(torch.randn(40, H, D, generator=g))
    return dict(records=rec, page_blk=page_blk, page_dst=page_dst, tail_blk=tail_blk, tail_info=tail_info,
                tail_k=tail_k, k_new=k_new, v_new=v_new, new_dst=new_dst, rows=rows, H=H)
