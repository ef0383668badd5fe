"""Pin the numpy oracle to the reference: its outputs on the fixture cases must
equal atflash.reference.ref_window_attn (and gates/g2_correctness.ref_decode_sliced)
outputs recorded by tests/golden/make_golden.py, and the test inputs must be the
reference's own tensors (sha256)."""
import json
import math
import os

import numpy as np
import pytest

from _inputs import make_bhsd, sha_bf16, to_np
from oracle import attention as OA
from oracle import window_table as OWT

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = json.load(open(os.path.join(HERE, "golden", "attn_cases.json")))


def _k(x):
    return float("inf") if x == "inf" else float(x)


def golden_rows(case):
    """Output rows a prefill fixture holds: all of them, or the rows of the
    128-row query tiles listed under "tiles"."""
    if "tiles" not in case:
        return np.arange(case["N"])
    return np.concatenate([np.arange(t * 128, min((t + 1) * 128, case["N"])) for t in case["tiles"]])


@pytest.mark.parametrize("case", CASES["prefill"], ids=lambda c: c["name"])
def test_oracle_prefill_matches_reference(case):
    q, k, v, _ = make_bhsd(case["hq"], case["hkv"], case["N"], case["d"], case["base"], case["seed"])
    assert sha_bf16(q) == case["sha_q"] and sha_bf16(k) == case["sha_k"] and sha_bf16(v) == case["sha_v"]
    gold = np.load(os.path.join(HERE, "golden", f"attn_{case['name']}.npz"))
    rows = golden_rows(case)
    for kr in case["k_rets"]:
        tag = "inf" if kr == "inf" else f"{kr:g}"
        w = OWT.wavelengths_sorted(case["d"], case["base"], _k(kr))
        kw = {"q_tiles": case["tiles"]} if "tiles" in case else {}
        o32 = OA.ref_window_attn(to_np(q), to_np(k), to_np(v), w, phase="prefill",
                                 block_m=case["block_m"], block_n=case["block_n"], mode="fp32", **kw)[:, :, rows]
        np.testing.assert_allclose(o32, gold[f"out32_k{tag}"], rtol=0, atol=2e-5)
        o16 = OA.ref_window_attn(to_np(q), to_np(k), to_np(v), w, phase="prefill",
                                 block_m=case["block_m"], block_n=case["block_n"], mode="bf16", **kw)[:, :, rows]
        anchor = float(np.abs(o16 - o32).max())
        # the bf16 anchor is an emulation; it must be of the reference's magnitude
        assert 0.25 * float(gold[f"anchor_k{tag}"]) <= anchor <= 4.0 * float(gold[f"anchor_k{tag}"])


@pytest.mark.parametrize("case", CASES["decode"], ids=lambda c: c["name"])
def test_oracle_decode_matches_reference(case):
    q, k, v, _ = make_bhsd(case["hq"], case["hkv"], case["N"], case["d"], case["base"], case["seed"],
                           phase="decode")
    assert sha_bf16(q) == case["sha_q"] and sha_bf16(k) == case["sha_k"] and sha_bf16(v) == case["sha_v"]
    gold = np.load(os.path.join(HERE, "golden", f"attn_{case['name']}.npz"))
    for kr in case["k_rets"]:
        tag = "inf" if kr == "inf" else f"{kr:g}"
        w = OWT.wavelengths_sorted(case["d"], case["base"], _k(kr))
        o32 = OA.ref_window_attn(to_np(q), to_np(k), to_np(v), w, phase="decode", block_m=1,
                                 block_n=1, mode="fp32")
        np.testing.assert_allclose(o32, gold[f"out32_k{tag}"], rtol=0, atol=2e-5)
        zs = OWT.zhi_slice_vec8(case["d"], case["base"], _k(kr))
        q2 = to_np(q)[0, :, 0, :]
        k2 = np.transpose(to_np(k)[0], (1, 0, 2))
        v2 = np.transpose(to_np(v)[0], (1, 0, 2))
        ov8 = OA.ref_decode_sliced(q2, k2, v2, zs, 8)
        np.testing.assert_allclose(ov8, gold[f"vec8_k{tag}"], rtol=0, atol=2e-5)


def test_window_is_active_in_fixtures():
    """The fixture cases really cut levels (otherwise they would pin nothing)."""
    for case in CASES["prefill"]:
        for kr in case["k_rets"]:
            if kr == "inf":
                continue
            w = OWT.wavelengths_sorted(case["d"], case["base"], _k(kr))
            st = OWT.mma_slice_stats("prefill", case["N"], case["N"], 128, 128, w, case["d"])
            assert st["qk_slice_ratio"] < 1.0
            if "tiles" in case:  # the recorded tiles themselves cut levels
                last = max(case["tiles"]) * 128
                segs = OWT.deff_segments("prefill", last, last + 128, 128, 128, case["N"], w, case["d"])
                assert min(dd for (_, _, dd) in segs) < case["d"]
    for case in CASES["decode"]:
        for kr in case["k_rets"]:
            if kr == "inf":
                continue
            w = OWT.wavelengths_sorted(case["d"], case["base"], _k(kr))
            assert OWT.deff_of_zmin(case["N"] - 1, w, case["d"]) < case["d"]


def test_lse_merge_identity():
    """Splitting the keys and merging partial states equals the full softmax."""
    rng = np.random.default_rng(0)
    N, d = 300, 16
    s = rng.standard_normal(N).astype(np.float32)
    vv = rng.standard_normal((N, d)).astype(np.float32)
    p = np.exp(s - s.max())
    full = (p / p.sum()) @ vv
    parts_o, parts_l = [], []
    for a, b in ((0, 100), (100, 120), (120, 300)):
        ss = s[a:b]
        m = ss.max()
        e = np.exp(ss - m)
        parts_o.append((e / e.sum()) @ vv[a:b])
        parts_l.append(m + math.log(e.sum()))
    o, l = OA.merge_states(np.stack(parts_o), np.array(parts_l, dtype=np.float32))
    np.testing.assert_allclose(o, full, atol=1e-6)
    assert abs(l - (s.max() + math.log(np.exp(s - s.max()).sum()))) < 1e-5


def test_oracle_chunk_offset_consistency():
    """q_offset extension: the rows of a bottom-right chunk equal the same rows
    of the full run when the chunk starts on the tile grid."""
    q, k, v, _ = make_bhsd(3, 1, 384, 128, 1e4, 5)
    w = OWT.wavelengths_sorted(128, 1e4, 2.0)
    full = OA.ref_window_attn(to_np(q), to_np(k), to_np(v), w, phase="prefill", block_m=128, block_n=128)
    part = OA.ref_window_attn(to_np(q)[:, :, 256:], to_np(k), to_np(v), w, phase="prefill",
                              block_m=128, block_n=128, q_offset=256)
    np.testing.assert_allclose(part, full[:, :, 256:], atol=1e-6)
    sub = OA.ref_window_attn(to_np(q), to_np(k), to_np(v), w, phase="prefill", block_m=128,
                             block_n=128, q_tiles=[2])
    np.testing.assert_allclose(sub[:, :, 256:], full[:, :, 256:], atol=0)
