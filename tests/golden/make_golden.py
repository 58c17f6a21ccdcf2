"""Generates tests/golden/golden.npz and golden.json from the REFERENCE's own PyTorch pins.

Run where a checkout of the reference is available (nothing at test time reads it), naming its directory:

    python tests/golden/make_golden.py <kushkash checkout>        # or KUSHKASH_REF=<checkout> python ...

What it pins, and with which reference function:
  quant   pages written by bulk writes + token appends == the reference's torch quantizer
          (tests/test_cpu.py:16-24 ref_quantize) applied per page / per token, assembled into the record layout
          of kushkash/kush/quant.mojo:53-87
  decode  attention over those pages == torch SDPA over the reference's dequantization
          (kushkash/_ops.py:295-306 cached_kv, :217-251 dequant_records), in fp64
  unpack  kushkash/_ops.py:398-436 unpack_reference on seeded records, bit patterns hashed
  fwht    kushkash/_ops.py:383-395 fwht_reference (the canonical butterfly order), bit patterns hashed
P = 16 fixtures run the same reference functions with kushkash._ops.PAGE set to 16 (the reference hard-codes 32;
its arithmetic per page is unchanged).
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from cases import (DECODE_CASES, QUANT_CASES, decode_inputs, fwht_inputs, pack_records, quant_inputs,  # noqa: E402
                   record_bytes, unpack_inputs)

def reference_dir() -> Path:
    """The reference checkout: the first command-line argument, else $KUSHKASH_REF; there is no default."""
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KUSHKASH_REF")
    if not ref:
        raise SystemExit("usage: make_golden.py <kushkash checkout>  (or set KUSHKASH_REF)")
    return Path(ref)


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def reference_pool(K, V, n, block_table, n_blocks, D, bits, P, ref_quantize):
    """Pool [n_blocks, H, RB] holding the first n tokens of K, V [B, H, T, D] as the reference quantizes them:
    full pages per page, the partial page's V rows per token (its K stays in the exact tail, its K part and K
    meta stay zero as in a fresh pool)."""
    B, H = K.shape[0], K.shape[1]
    rb = record_bytes(D, bits, P)
    pool = torch.zeros(n_blocks, H, rb, dtype=torch.uint8)
    for b in range(B):
        for p in range(-(-n // P)):
            lo, hi = p * P, min(n, (p + 1) * P)
            for h in range(H):
                kq = torch.zeros(P, D, dtype=torch.int8)
                ks = torch.zeros(D)
                kb = torch.zeros(D)
                if hi - lo == P:
                    ck, sk, bk = ref_quantize(K[b, h, lo:hi], bits, dim=0)
                    kq, ks, kb = ck, sk[0], bk[0]
                vq = torch.zeros(P, D, dtype=torch.int8)
                vs = torch.zeros(P)
                vb = torch.zeros(P)
                cv, sv, bv = ref_quantize(V[b, h, lo:hi], bits, dim=1)
                vq[:hi - lo], vs[:hi - lo], vb[:hi - lo] = cv, sv[:, 0], bv[:, 0]
                pool[int(block_table[b, p]), h] = pack_records(kq, ks, kb, vq, vs, vb, D, bits, P)
    return pool


def main() -> None:
    ref = reference_dir()
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "tests"))
    import kushkash._ops as kops
    from kushkash._ops import cached_kv, fwht_reference, unpack_reference
    from test_cpu import ref_quantize

    arrays: dict[str, np.ndarray] = {}
    meta: dict = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__, "quant": {}, "decode": {},
                  "unpack": {}, "fwht": {}}

    for D, bits, P in QUANT_CASES:
        c = quant_inputs(D, bits, P)
        pool = reference_pool(c["K"], c["V"], c["T"], c["block_table"], c["n_blocks"], D, bits, P, ref_quantize)
        key = f"quant_{D}_{bits}_{P}"
        arrays[key] = pool.numpy()
        meta["quant"][key] = {"sha256": sha(pool), "shape": list(pool.shape)}

    for D, bits, G, P, B, H, n in DECODE_CASES:
        c = decode_inputs(D, bits, G, P, B, H, n)
        pool = reference_pool(c["K"], c["V"], n, c["block_table"], c["n_blocks"], D, bits, P, ref_quantize)
        tail = torch.zeros(B, H, P, D)
        r = n % P
        if r:
            tail[:, :, :r] = c["K"][:, :, n - r:n]
        kops.PAGE = P
        try:
            hk, hv = cached_kv(pool, c["block_table"], n, tail, D, bits, torch.float64)
        finally:
            kops.PAGE = 32
        q = c["q"].double()
        out = F.scaled_dot_product_attention(q[:, :, None], hk, hv, enable_gqa=G > 1, scale=D ** -0.5)[:, :, 0]
        key = f"decode_{D}_{bits}_{G}_{P}_{B}_{H}_{n}"
        arrays[key] = out.float().numpy()
        meta["decode"][key] = {"pool_sha256": sha(pool)}

    for D, bits, rot in ((64, 4, False), (64, 4, True), (128, 8, True), (256, 4, False)):
        c = unpack_inputs(D, bits)
        shape = (c["rows"], c["H"], D)
        kp, vp = torch.full(shape, float("nan")), torch.full(shape, float("nan"))
        unpack_reference(c["records"], c["page_blk"], c["page_dst"], c["tail_blk"], c["tail_info"], c["tail_k"],
                         c["k_new"], c["v_new"], c["new_dst"], kp, vp, D, bits, rot)
        key = f"unpack_{D}_{bits}_{int(rot)}"
        meta["unpack"][key] = {"kp_sha256": sha(kp), "vp_sha256": sha(vp),
                               "kp_sample": kp[0, 0, :4].tolist(), "vp_sample": vp[0, 0, :4].tolist()}

    for D in (64, 128, 256):
        y = fwht_reference(fwht_inputs(D))
        meta["fwht"][f"fwht_{D}"] = {"sha256": sha(y), "sample": y[0, :4].tolist()}

    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(f"wrote {HERE / 'golden.npz'} ({(HERE / 'golden.npz').stat().st_size} bytes) and golden.json")


if __name__ == "__main__":
    main()
