"""Window rule: product tables (Python and C ABI) and the oracle restatement, all
checked bit for bit against fixtures generated from the reference itself
(tests/golden/window_tables.json; generator tests/golden/make_golden.py).

Mirrors the reference's CPU checks (tools/cpu_checks.py:56-117): twin widths and
D_eff, zhi level boundaries, and the recorded C1 tables."""
import ctypes
import json
import math
import os
import struct

import pytest

from oracle import window_table as OWT
from atflash import window_table as WT

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "window_tables.json")))


def _bits(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def _k(rec):
    return float("inf") if rec["k_ret"] == "inf" else float(rec["k_ret"])


@pytest.mark.parametrize("rec", GOLD["tables"], ids=lambda r: f"d{r['head_dim']}-b{r['base']:g}-k{r['k_ret']}")
def test_tables_match_reference(rec):
    d, base, k = rec["head_dim"], rec["base"], _k(rec)
    w_prod = WT.wavelengths_sorted(d, base, k).tolist()
    w_orc = OWT.wavelengths_sorted(d, base, k)
    assert [_bits(x) for x in w_prod] == rec["wvec_bits"]
    assert [_bits(x) for x in w_orc] == rec["wvec_bits"]
    for z, deff in rec["deff"]:
        assert WT.deff_of_zmin(z, w_prod, d) == deff
        assert OWT.deff_of_zmin(z, w_orc, d) == deff
    for z, na in rec["n_active"]:
        assert WT.n_active(z, w_prod) == na
        assert OWT.n_active(z, w_orc) == na
    for cap, zhi in rec["zhi16"].items():
        assert list(WT.window_zhi_from_kret(d, base, k, int(cap))) == zhi
        assert list(OWT.window_zhi_from_kret(d, base, k, int(cap))) == zhi
        # D_eff through the zhi levels equals the per-pair rule at every checked z
        for z, deff in rec["deff"]:
            if z <= int(cap):
                assert WT.deff_from_zhi(zhi, z) == deff
    assert WT.zhi_slice_vec8(d, base, k, device="cpu").tolist() == rec["zhi8"]
    assert OWT.zhi_slice_vec8(d, base, k) == rec["zhi8"]
    for n, sv in rec["s_vec8"].items():
        assert WT.theory_s_vec8(d, base, k, int(n)) == tuple(sv)
        assert OWT.theory_s_vec8(d, base, k, int(n)) == tuple(sv)


@pytest.mark.parametrize("rec", GOLD["stats"], ids=lambda r: f"N{r['N']}-{r['BM']}x{r['BN']}-b{r['base']:g}")
def test_schedule_stats_match_reference(rec):
    d, base, k, N, BM, BN = rec["head_dim"], rec["base"], rec["k_ret"], rec["N"], rec["BM"], rec["BN"]
    w = WT.wavelengths_sorted(d, base, k)
    wo = OWT.wavelengths_sorted(d, base, k)
    for phase, mm in (("prefill", N), ("decode", 1)):
        got = WT.mma_slice_stats(phase, mm, N, BM if phase == "prefill" else 1, BN, w, d)
        exp = rec[phase]
        assert got["qk_mma_slices_windowed"] == exp["qk_mma_slices_windowed"]
        assert got["qk_mma_slices_full"] == exp["qk_mma_slices_full"]
        assert got["qk_slice_ratio"] == exp["qk_slice_ratio"]
        assert got["kload_dim_ratio"] == exp["kload_dim_ratio"]
        assert OWT.mma_slice_stats(phase, mm, N, BM if phase == "prefill" else 1, BN, wo, d) == exp
    for q0, segs in rec["segments"].items():
        q0 = int(q0)
        exp = [tuple(s) for s in segs]
        assert WT.deff_segments("prefill", q0, min(q0 + BM, N), BM, BN, N, w, d) == exp
        assert OWT.deff_segments("prefill", q0, min(q0 + BM, N), BM, BN, N, wo, d) == exp


def test_c1_recorded_tables():
    """window_tables/c1_window_tables.txt: Qwen2.5-7B-1M, base 1e7, cap 1.1M."""
    c1 = GOLD["c1_recorded"]
    for kstr, t in c1["tables"].items():
        k = float(kstr)
        assert list(WT.window_zhi_from_kret(128, 1e7, k, c1["cap"])) == t["fa4_16snap"]
        assert list(OWT.window_zhi_from_kret(128, 1e7, k, c1["cap"])) == t["fa4_16snap"]
        assert WT.zhi_slice_vec8(128, 1e7, k, device="cpu").tolist() == t["fi_8snap"]


def test_zhi_boundaries_exhaustive_small():
    """Every level boundary of the closed-form table is where D_eff drops
    (tools/cpu_checks.py:76-93), across bases, k and head dims."""
    for d in (64, 128):
        for base in (1e4, 5e5, 1e6, 5e6, 1e7):
            for k in (0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 64.0):
                w = OWT.wavelengths_sorted(d, base, k)
                for cap in (8192, 131072, 1_100_000):
                    zhi = WT.zhi_table(w, d, cap)
                    for i, z in enumerate(zhi):
                        e = 16 * (i + 1)
                        assert OWT.deff_of_zmin(z, w, d) >= e
                        if z < cap:
                            assert OWT.deff_of_zmin(z + 1, w, d) < e


def test_baseline_slice_ratios():
    """s for the BASELINE prefill configs at the kernel's 128x128 tiles."""
    r = WT.prefill_work(28, 131072, 131072, WT.window_zhi_from_kret(128, 1e7, 2.0, 2 ** 31 - 1))
    assert abs(r["s"] - 0.5624) < 5e-4
    r = WT.prefill_work(28, 131072, 131072, WT.window_zhi_from_kret(128, 1e7, 64.0, 2 ** 31 - 1))
    assert abs(r["s"] - 0.7865) < 5e-4
    N = 131072
    r = WT.prefill_work(28, N, N, None)
    assert r["flops"] == r["flops_dense"] == 2.0 * 28 * 128 * N * (N + 1)
    assert abs(r["flops"] - 1.2315e14) / 1.2315e14 < 1e-3
    r2 = WT.prefill_work(28, N, N, WT.window_zhi_from_kret(128, 1e7, 2.0, 2 ** 31 - 1))
    assert abs(r2["flops"] - 9.63e13) / 9.63e13 < 2e-3


def _lib_or_skip():
    from atflash import _ffi
    try:
        return _ffi.load()
    except (ImportError, OSError) as e:
        pytest.skip(f"library not built: {e}")


def test_c_abi_tables_match_reference():
    lib = _lib_or_skip()
    for rec in GOLD["tables"]:
        d, base, k = rec["head_dim"], rec["base"], _k(rec)
        P = d // 2
        buf = (ctypes.c_float * P)()
        assert lib.atf_window_widths(d, base, k, buf) == 0
        assert [_bits(x) for x in buf] == rec["wvec_bits"]
        for cap, zhi in rec["zhi16"].items():
            out = (ctypes.c_int32 * (d // 16))()
            assert lib.atf_window_zhi16(buf, d, int(cap), out) == 0
            assert list(out) == zhi
            for z, deff in rec["deff"]:
                if z <= int(cap):
                    assert lib.atf_window_deff(out, d // 16, z) == deff
        z8 = (ctypes.c_int32 * (d // 8))()
        assert lib.atf_window_zhi8(buf, d, z8) == 0
        assert list(z8) == rec["zhi8"]


# ------------------------------------------------------- RoPE-scaled (entity) tables
def _wmeta():
    import json
    return json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                                       "w_meta_tables.json")))["tables"]


def test_widths_from_inv_freq_match_reference_entity_tables():
    """k * 2*pi / inv_freq in fp64, rounded to fp32 and sorted, bit for bit as the
    reference's recorded tables (base model and YaRN s=2 included)."""
    import struct
    from atflash import window_table as WT
    tabs = _wmeta()
    assert len(tabs) == 3 and any(t["rope_scaling"] for t in tabs)
    for t in tabs:
        w = WT.wavelengths_from_inv_freq(t["inv_freq"], t["k"])
        bits = [struct.unpack("<I", struct.pack("<f", x))[0] for x in w.tolist()]
        assert bits == t["w_sorted_fp32_bits"], t["source"]


def test_window_table_from_inv_freq_levels_match_reference():
    from atflash import window_table as WT
    for t in _wmeta():
        wt = WT.WindowTable.from_inv_freq(t["inv_freq"], t["k"])
        assert wt.head_dim == t["head_dim"]
        for cap, zhi in t["zhi16"].items():
            assert list(wt.zhi(int(cap))) == zhi, (t["source"], cap)
        # the kernel table covers every distance and agrees with D_eff of the widths
        for z in (0, 1, 100, 10_000, 1_000_000):
            assert wt.deff(z) == WT.deff_of_zmin(z, wt.wvec, wt.head_dim)


def test_pair_order_gate():
    """The reference's harness stops unless the model's wavelengths grow with the
    pair index (e2e_pipeline/atflash_e2e_fafi.py:143-157); so does from_inv_freq."""
    from atflash import window_table as WT
    for t in _wmeta():
        order, canonical = WT.pair_order_from_inv_freq(t["inv_freq"])
        assert canonical and order[0] == len(t["inv_freq"]) - 1
    inv = list(_wmeta()[0]["inv_freq"])
    inv[3], inv[7] = inv[7], inv[3]
    assert not WT.pair_order_from_inv_freq(inv)[1]
    with pytest.raises(ValueError):
        WT.WindowTable.from_inv_freq(inv, 2.0)


@pytest.mark.parametrize("base,k_ret", [(1e4, 2.0), (5e5, 2.0), (1e7, 64.0), (1e7, 2.0), (5e5, float("inf"))])
def test_bisected_segments_equal_the_tile_walk(base, k_ret):
    """deff_segments_bisect (used by the oracle for long decode contexts) gives
    exactly the runs of the reference's tile-by-tile walk (deff_segments)."""
    w = OWT.wavelengths_sorted(128, base, k_ret)
    for (phase, q0, n_hi, bm, bn, n_ctx) in [("decode", 0, 20000, 1, 1, 20000), ("decode", 0, 4099, 1, 16, 4099),
                                             ("prefill", 8192, 8192 + 128, 128, 128, 9000),
                                             ("prefill", 3000, 3064, 64, 32, 3064), ("prefill", 0, 100, 128, 128, 100),
                                             ("decode", 0, 1, 1, 1, 1)]:
        assert OWT.deff_segments_bisect(phase, q0, n_hi, bm, bn, n_ctx, w, 128) == \
            OWT.deff_segments(phase, q0, n_hi, bm, bn, n_ctx, w, 128)
