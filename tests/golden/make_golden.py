#!/usr/bin/env python
"""Generate the golden fixtures in this directory from the reference itself.

Run where the reference tree is available (its path is given by --reference or
the ATFLASH_REFERENCE environment variable); the fixtures are committed so that
the tests never need the reference at run time:

    python tests/golden/make_golden.py --reference <path of the reference tree>

What is recorded, all produced by the reference's own code:
  w_meta_tables.json  the reference's recorded RoPE-scaled window inputs
                      (window_tables/w_meta_*.json: a model's own inv_freq and
                      the widths k * 2*pi / inv_freq) with the zhi levels the
                      reference's zhi_table gives for them.
  window_tables.json  atflash/window_table.py (torch) and the torch-free twin
                      window_tables/atflash_window.py: fp32 widths (bit patterns),
                      D_eff at many distances, zhi levels (16-snap) at three caps,
                      vec8 slice tables and their s-bar (fiwin_common.py:35-60),
                      mma_slice_stats and deff_segments for small prefill / decode
                      tilings; plus the recorded C1 tables of
                      window_tables/c1_window_tables.txt (the reference's own golden
                      vector, checked by tools/cpu_checks.py:108-117).
  attn_*.npz          atflash.reference.ref_window_attn outputs (fp32 and the bf16
                      anchor) and gates/g2_correctness.ref_decode_sliced outputs on
                      seeded inputs built with the reference's RoPE front-end
                      (gates/g2_correctness.py:79-98). Inputs are not stored; the
                      tests rebuild them from the seed and check their sha256.
"""
import argparse
import hashlib
import json
import math
import os
import re
import struct
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

BASES = (1e4, 5e5, 1e6, 5e6, 1e7)
K_RETS = (1.0, 1.5, 2.0, 3.0, 4.0, 64.0, float("inf"))
HEAD_DIMS = (64, 128)
CAPS = (8192, 131072, 1_100_000)

INF = float("inf")
# (name, hq, hkv, N, base, k_ret list, seed, tiles) -- prefill cases at the kernel
# tile (block 128 x 128). tiles = None records every output row; otherwise only
# the rows of the listed 128-row query tiles are stored (the reference still
# computes the whole output), which keeps the fixtures of the longer cases small.
PREFILL_CASES = [
    ("prefill_g3", 3, 1, 448, 1e4, (2.0, INF), 777, None),
    ("prefill_g7", 7, 1, 320, 1e4, (1.0,), 778, None),
    # BASELINE config 1 / 3 RoPE base (5e5), GQA group 3
    ("prefill_t5e5_g3", 3, 1, 2048, 5e5, (2.0, INF), 781, (5, 15)),
    # BASELINE config 2 / 4 RoPE base (1e7), GQA group 7; k=64 cuts a level from z > 2341 on
    ("prefill_t1e7_g7", 7, 1, 4096, 1e7, (2.0, 64.0, INF), 782, (31,)),
]
# decode cases: (name, hq, hkv, N, base, k_ret, seed)
DECODE_CASES = [
    ("decode_g3", 6, 2, 1000, 1e4, (2.0, INF), 1234 + 1000 + 128),
    ("decode_t5e5_g3_8k", 6, 2, 8192, 5e5, (2.0, INF), 1234 + 8192 + 128),
    ("decode_t1e7_g7_32k", 7, 1, 32768, 1e7, (2.0, 64.0, INF), 1234 + 32768 + 128),
]


def f32_bits(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def sha_bf16(t):
    return hashlib.sha256(t.contiguous().view(torch.int16).numpy().tobytes()).hexdigest()


def _same_npz(path, arrays):
    """True when `path` already holds exactly these arrays (so a re-run leaves
    the committed file untouched)."""
    if not os.path.exists(path):
        return False
    old = np.load(path)
    return sorted(old.files) == sorted(arrays) and all(
        np.array_equal(old[n], np.asarray(arrays[n])) for n in arrays)


def build_inputs(G2, hq, hkv, N, d, base, seed, phase):
    """Seeded pre-RoPE N(0,1) bf16 q/k/v, rotated by the reference's _rope_hf at
    positions 0..N-1 (decode: q at N-1), permuted to sorted pairs, cast to bf16."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    M = N if phase == "prefill" else 1
    q = torch.randn((1, hq, M, d), generator=g, dtype=torch.float32).to(torch.bfloat16)
    k = torch.randn((1, hkv, N, d), generator=g, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn((1, hkv, N, d), generator=g, dtype=torch.float32).to(torch.bfloat16)
    inv = 1.0 / (base ** (torch.arange(0, d, 2).float() / d))
    pos_k = torch.arange(N)
    pos_q = pos_k if phase == "prefill" else torch.tensor([N - 1])
    perm = G2.hf_to_sorted_pair_perm(d)
    qs = G2._rope_hf(q, pos_q, inv)[..., perm].to(torch.bfloat16)
    ks = G2._rope_hf(k, pos_k, inv)[..., perm].to(torch.bfloat16)
    return qs, ks, v


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ATFLASH_REFERENCE"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference tree with --reference or ATFLASH_REFERENCE")
    ref = args.reference
    sys.path[:0] = [os.path.join(ref, "window_tables"),
                    os.path.join(ref, "kernels", "flashinfer_port"), ref,
                    os.path.join(ref, "gates")]
    import atflash_window as AW
    from atflash import window_table as WT
    from atflash.reference import ref_window_attn
    import fiwin_common as FC
    import g2_correctness as G2

    torch.backends.cuda.matmul.allow_tf32 = False
    tables = []
    for d in HEAD_DIMS:
        for base in BASES:
            for kr in K_RETS:
                w_t = WT.wavelengths_sorted(d, base, kr)
                w_a = AW.wavelengths_sorted(d, base, kr)
                assert w_t.tolist() == list(w_a)
                zs = sorted({0, 1, 7, 8, 9, 15, 16, 17, 100, 1000, 65535, 65536, 131071}
                            | {int(x) + e for x in w_a[-16:] if not math.isinf(x) for e in (-1, 0, 1)
                               if 0 <= int(x) + e < 2 ** 24})
                rec = {
                    "head_dim": d, "base": base, "k_ret": kr if not math.isinf(kr) else "inf",
                    "wvec_bits": [f32_bits(x) for x in w_a],
                    "deff": [[z, WT.deff_of_zmin(z, w_t, d)] for z in zs],
                    "n_active": [[z, WT.n_active(z, w_t)] for z in zs],
                    "zhi16": {str(c): list(AW.window_zhi_from_kret(d, base, kr, c)) for c in CAPS},
                    "zhi8": FC.zhi_slice_vec8(d, base, kr, device="cpu").tolist(),
                    "s_vec8": {str(n): list(FC.theory_s_vec8(d, base, kr, n)) for n in (8192, 131072)},
                }
                tables.append(rec)
    stats = []
    for (d, base, kr, N, BM, BN) in [(128, 5e5, 2.0, 2048, 128, 128), (128, 5e5, 2.0, 2048, 128, 64),
                                     (128, 1e4, 2.0, 1000, 128, 128), (64, 1e6, 2.0, 2048, 128, 128),
                                     (128, 1e7, 64.0, 4096, 128, 128), (128, 1e4, 1.0, 777, 64, 32)]:
        w = WT.wavelengths_sorted(d, base, kr)
        rec = {"head_dim": d, "base": base, "k_ret": kr, "N": N, "BM": BM, "BN": BN,
               "prefill": WT.mma_slice_stats("prefill", N, N, BM, BN, w, d),
               "decode": WT.mma_slice_stats("decode", 1, N, 1, BN, w, d),
               "segments": {str(q0): WT.deff_segments("prefill", q0, min(q0 + BM, N), BM, BN, N, w, d)
                            for q0 in range(0, N, BM)}}
        stats.append(rec)
    with open(os.path.join(ref, "window_tables", "c1_window_tables.txt"), encoding="utf-8") as f:
        txt = f.read()
    c1 = {}
    for m in re.finditer(r"k=(\d\.\d): FA4 16snap len=8 sha=(\w+) \[([^\]]*)\]\s+FI  8snap  len=16 sha=(\w+) \[([^\]]*)\]", txt):
        c1[m.group(1)] = {"fa4_16snap": [int(x) for x in m.group(3).split(",")], "sha16": m.group(2),
                          "fi_8snap": [int(x) for x in m.group(5).split(",")], "sha8": m.group(4)}
    assert len(c1) == 3, c1.keys()
    with open(os.path.join(HERE, "window_tables.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "tables": tables, "stats": stats,
                   "c1_recorded": {"model": "Qwen2.5-7B-Instruct-1M", "base": 1e7, "head_dim": 128,
                                   "cap": 1_100_000, "tables": c1}}, f, indent=0)

    # RoPE-scaled ("entity") window tables: the reference's recorded inv_freq and
    # widths (window_tables/w_meta_*.json, made by w_meta_from_hf.py and
    # w_meta_7b1m_yarn_s2.py) and the reference's zhi levels of those widths
    wmeta = []
    for fn in sorted(os.listdir(os.path.join(ref, "window_tables"))):
        if not (fn.startswith("w_meta_") and fn.endswith(".json")):
            continue
        m = json.load(open(os.path.join(ref, "window_tables", fn)))
        d = 2 * len(m["inv_freq"])
        w_sorted32 = sorted((struct.unpack("<f", struct.pack("<f", x))[0] for x in m["w"]), reverse=True)
        wmeta.append({"source": fn, "model": m["model"], "k": m["k_convex"],
                      "rope_scaling": m.get("rope_scaling"), "head_dim": d,
                      "inv_freq": m["inv_freq"], "w_fp64": m["w"],
                      "w_sorted_fp32_bits": [f32_bits(x) for x in w_sorted32],
                      "zhi16": {str(c): list(AW.zhi_table(w_sorted32, d, c)) for c in CAPS}})
    with open(os.path.join(HERE, "w_meta_tables.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "tables": wmeta}, f, indent=0)

    meta = {"prefill": [], "decode": []}
    d = 128
    for (name, hq, hkv, N, base, krs, seed, tiles) in PREFILL_CASES:
        q, k, v = build_inputs(G2, hq, hkv, N, d, base, seed, "prefill")
        rows = (np.concatenate([np.arange(t * 128, min((t + 1) * 128, N)) for t in tiles])
                if tiles is not None else np.arange(N))
        arrays = {}
        for kr in krs:
            w = WT.wavelengths_sorted(d, base, kr)
            tag = "inf" if math.isinf(kr) else f"{kr:g}"
            o32 = ref_window_attn(q, k, v, w, phase="prefill", block_m=128, block_n=128, mode="fp32")
            o16 = ref_window_attn(q, k, v, w, phase="prefill", block_m=128, block_n=128, mode="bf16")
            arrays[f"out32_k{tag}"] = o32[:, :, rows].numpy()
            arrays[f"anchor_k{tag}"] = np.float32((o16.float() - o32)[:, :, rows].abs().max().item())
        path = os.path.join(HERE, f"attn_{name}.npz")
        if not _same_npz(path, arrays):
            np.savez_compressed(path, **arrays)
        rec = {"name": name, "hq": hq, "hkv": hkv, "N": N, "d": d, "base": base,
               "k_rets": [("inf" if math.isinf(x) else x) for x in krs], "seed": seed,
               "block_m": 128, "block_n": 128,
               "sha_q": sha_bf16(q), "sha_k": sha_bf16(k), "sha_v": sha_bf16(v)}
        if tiles is not None:
            rec["tiles"] = list(tiles)
        meta["prefill"].append(rec)
    for (name, hq, hkv, N, base, krs, seed) in DECODE_CASES:
        q, k, v = build_inputs(G2, hq, hkv, N, d, base, seed, "decode")
        arrays = {}
        for kr in krs:
            w = WT.wavelengths_sorted(d, base, kr)
            tag = "inf" if math.isinf(kr) else f"{kr:g}"
            o32 = ref_window_attn(q, k, v, w, phase="decode", block_m=1, block_n=1, mode="fp32")
            arrays[f"out32_k{tag}"] = o32.numpy()
            zs = FC.zhi_slice_vec8(d, base, kr, device="cpu")
            q2 = q[0, :, 0, :]
            k2 = k[0].permute(1, 0, 2).contiguous()
            v2 = v[0].permute(1, 0, 2).contiguous()
            ov8, _ = G2.ref_decode_sliced(q2, k2, v2, zs, 8, "fp32")
            arrays[f"vec8_k{tag}"] = ov8.numpy()
        path = os.path.join(HERE, f"attn_{name}.npz")
        if not _same_npz(path, arrays):
            np.savez_compressed(path, **arrays)
        meta["decode"].append({"name": name, "hq": hq, "hkv": hkv, "N": N, "d": d, "base": base,
                               "k_rets": [("inf" if math.isinf(x) else x) for x in krs], "seed": seed,
                               "sha_q": sha_bf16(q), "sha_k": sha_bf16(k), "sha_v": sha_bf16(v)})
    with open(os.path.join(HERE, "attn_cases.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
