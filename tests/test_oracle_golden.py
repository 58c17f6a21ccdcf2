"""The CPU oracle (oracle/kush_oracle.c, test infrastructure) against the golden fixtures generated from the
reference's own PyTorch pins (tests/golden/make_golden.py).  No GPU needed.

Pins: pages bit-exact vs tests/test_cpu.py:16-24 ref_quantize of the reference; decode within 1e-5 (rel-norm, the
reference's CPU tolerance, tests/test_cpu.py:96) of SDPA over the reference's dequantization (cached_kv); unpack and
FWHT bit patterns equal to the reference's unpack_reference / fwht_reference."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from cases import DECODE_CASES, QUANT_CASES, decode_inputs, fwht_inputs, quant_inputs, unpack_inputs
from kushsim import fill, make_state
from oracle.kush_oracle import OracleOps, lib

GOLD = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLD / "golden.json").read_text())
ARR = np.load(GOLD / "golden.npz")


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def test_fp16_rounding_matches_numpy():
    """The oracle's own fp32 -> fp16 conversion (round to nearest even, subnormals, overflow) == numpy's."""
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2 ** 32, 200_000, dtype=np.uint64).astype(np.uint32)
    special = np.array([0x00000000, 0x80000000, 0x477FE000, 0x477FF000, 0x477FEFFF, 0x38800000, 0x387FFFFF,
                        0x33000000, 0x33000001, 0x32FFFFFF, 0x7F800000, 0x3F800000, 0x3DCCCCCD], dtype=np.uint32)
    vals = np.concatenate([bits, special]).view(np.float32)
    vals = vals[np.isfinite(vals)]
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    f2h = lib().kush_oracle_f2h
    got = np.array([f2h(float(v)) for v in vals[:20000]] + [f2h(float(v)) for v in vals[-len(special):]],
                   dtype=np.uint16)
    ref = np.concatenate([want[:20000], want[-len(special):]])
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("D,bits,P", QUANT_CASES)
def test_pages_match_reference_quantizer(D, bits, P):
    """Bulk write + single-token appends produce exactly the reference quantizer's pages; tails hold exact K."""
    c = quant_inputs(D, bits, P)
    st = make_state(c["B"], c["H"], D, bits, P, c["block_table"], c["n_blocks"])
    fill(OracleOps(D, bits, 1, P), st, c["K"], c["V"], c["bulk"], torch.float32, "cpu")
    key = f"quant_{D}_{bits}_{P}"
    want = torch.from_numpy(ARR[key])
    assert sha(want) == META["quant"][key]["sha256"]
    diff = (st.pool != want).sum().item()
    assert diff == 0, f"{diff} record bytes differ from the reference quantizer"
    r = c["T"] % P
    assert torch.equal(st.tail_k[:, :, :r], c["K"][:, :, c["T"] - r:])


@pytest.mark.parametrize("D,bits,G,P,B,H,n", DECODE_CASES)
def test_decode_matches_reference_dequant(D, bits, G, P, B, H, n):
    c = decode_inputs(D, bits, G, P, B, H, n)
    st = make_state(B, H, D, bits, P, c["block_table"], c["n_blocks"])
    ops = OracleOps(D, bits, G, P)
    fill(ops, st, c["K"], c["V"], n, torch.float32, "cpu")
    key = f"decode_{D}_{bits}_{G}_{P}_{B}_{H}_{n}"
    assert sha(st.pool) == META["decode"][key]["pool_sha256"]
    out = torch.empty(B, H * G, D)
    ops.decode(c["q"].contiguous(), out, st.pool, st.block_table, st.seq_lens, st.tail_idx, st.tail_k, D ** -0.5)
    ref = torch.from_numpy(ARR[key])
    assert ((out - ref).norm() / ref.norm()).item() < 1e-5


@pytest.mark.parametrize("key", sorted(META["unpack"]))
def test_unpack_matches_reference(key):
    _, D, bits, rot = key.split("_")
    D, bits, rot = int(D), int(bits), bool(int(rot))
    c = unpack_inputs(D, bits)
    shape = (c["rows"], c["H"], D)
    kp, vp = torch.full(shape, float("nan")), torch.full(shape, float("nan"))
    OracleOps(D, bits, 1).unpack(c["records"], c["page_blk"], c["page_dst"], c["tail_blk"], c["tail_info"], c["tail_k"],
                                 c["k_new"], c["v_new"], c["new_dst"], kp, vp, rot)
    assert sha(kp) == META["unpack"][key]["kp_sha256"]
    assert sha(vp) == META["unpack"][key]["vp_sha256"]
    assert kp[0].isnan().all() and vp[-1].isnan().all()                           # gap rows untouched


@pytest.mark.parametrize("D", [64, 128, 256])
def test_fwht_matches_reference(D):
    y = OracleOps(D, 4, 1).fwht(fwht_inputs(D))
    assert sha(y) == META["fwht"][f"fwht_{D}"]["sha256"]


def test_oracle_rejects_unsupported_shapes():
    with pytest.raises(ValueError):
        OracleOps(96, 4, 1)
    ops = OracleOps(64, 4, 1)
    ops.D = 96                                       # the C ABI itself returns -1 -> ValueError
    with pytest.raises(ValueError):
        ops.fwht(torch.zeros(2, 96))
