"""Prefill kernel parity on a B200: the tcgen05 kernel through the public API
(C ABI underneath) against the numpy oracle (a restatement of
atflash/reference.py pinned to the reference by test_oracle_golden.py).

Pass bar (absolute, fp32 oracle): max |err| <= 2e-2 and mean |err| <= 2e-3, window
on and off; the reference's own relative rule (max <= 2*anchor + 2e-3,
microbench/b1_correctness.py:89-91) is checked next to it. Bit-identity gates
adapted from gates/g1_bitexact.py (window None == k=inf) and
gates/c0_chunk_neutrality.py (chunked / sharded == single shot)."""
import json
import math
import os

import numpy as np
import pytest
import torch

from _inputs import MAX_ABS_TOL, MEAN_ABS_TOL, err_stats, inv_sorted_perm, make_bhsd, to_np
from oracle import attention as OA
from oracle import window_table as OWT

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
BM, BN = 128, 128  # the kernel's tile; the window is quantised per (query tile, key tile)


def _atf():
    import atflash
    return atflash


def _bshd(t, dev):
    return t.transpose(1, 2).contiguous().to(dev)


def _run(q, k, v, dev, base, k_ret, layout="sorted_pair", **kw):
    atflash = _atf()
    wt = None if (k_ret is None or math.isinf(k_ret)) else atflash.WindowTable(128, base, k_ret)
    if layout == "rotate_half":
        inv = inv_sorted_perm(128)
        q, k = q[..., inv], k[..., inv]
    out = atflash.flash_attn_func(_bshd(q, dev), _bshd(k, dev), _bshd(v, dev), causal=True,
                                  window_table=wt, qk_layout=layout, **kw)
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    return out


def _oracle(q, k, v, base, k_ret, mode="fp32", **kw):
    w = OWT.wavelengths_sorted(128, base, float("inf") if k_ret is None else k_ret)
    return OA.ref_window_attn(to_np(q), to_np(k), to_np(v), w, phase="prefill", block_m=BM,
                              block_n=BN, mode=mode, **kw)


CASES = [
    # (hq, hkv, N, base, k_ret, seed)
    (3, 1, 128, 1e4, 2.0, 1),
    (6, 2, 256, 1e4, 2.0, 2),
    (3, 1, 448, 1e4, 2.0, 777),
    (7, 1, 320, 1e4, 1.0, 778),
    (4, 4, 700, 1e4, 2.0, 3),
    (24, 8, 2048, 5e5, 2.0, 777),
    (28, 4, 1536, 1e7, 2.0, 11),
    (14, 2, 1000, 1e4, 3.0, 12),
    (4, 2, 384, 1e4, 2.0, 13),     # GQA group 2
    (8, 2, 640, 1e4, 2.0, 14),     # GQA group 4
    (8, 1, 512, 5e5, 2.0, 15),     # GQA group 8
]


@pytest.mark.parametrize("window", ["on", "off"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"h{c[0]}x{c[1]}-N{c[2]}-b{c[3]:g}-k{c[4]:g}")
def test_prefill_parity(cuda_device, case, window):
    hq, hkv, N, base, k_ret, seed = case
    kr = k_ret if window == "on" else None
    q, k, v, _ = make_bhsd(hq, hkv, N, 128, base, seed)
    out = _run(q, k, v, cuda_device, base, kr).transpose(1, 2).float().cpu().numpy()
    ref32 = _oracle(q, k, v, base, kr)
    mx, mean = err_stats(out, ref32)
    ref16 = _oracle(q, k, v, base, kr, mode="bf16")
    anchor = float(np.abs(ref16 - ref32).max())
    assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (mx, mean)
    assert mx <= 2 * anchor + 2e-3, (mx, anchor)


def test_prefill_rejects_a_wrong_out_buffer(cuda_device):
    """A caller-supplied out of the wrong shape, dtype or layout is refused before
    any launch (its strides would otherwise steer the kernel's stores)."""
    atflash = _atf()
    q = torch.zeros((1, 256, 4, 128), dtype=torch.bfloat16, device=cuda_device)
    k = torch.zeros((1, 256, 2, 128), dtype=torch.bfloat16, device=cuda_device)
    for bad in (torch.empty((1, 128, 4, 128), dtype=torch.bfloat16, device=cuda_device),
                torch.empty((1, 256, 4, 128), dtype=torch.float32, device=cuda_device),
                torch.empty((1, 256, 128, 4), dtype=torch.bfloat16, device=cuda_device).transpose(2, 3)):
        with pytest.raises(ValueError):
            atflash.prefill_fwd(q, k, k, out=bad)
    good = torch.empty((1, 256, 4, 128), dtype=torch.bfloat16, device=cuda_device)
    assert atflash.prefill_fwd(q, k, k, out=good) is good


def test_prefill_batch_of_two(cuda_device):
    """Two sequences in one call (B = 2, GQA group 4): each batch row matches the
    oracle run on its own."""
    hq, hkv, N, base, k_ret = 8, 2, 384, 1e4, 2.0
    parts = [make_bhsd(hq, hkv, N, 128, base, seed) for seed in (21, 22)]
    q, k, v = (torch.cat([p[i] for p in parts], dim=0) for i in range(3))
    out = _run(q, k, v, cuda_device, base, k_ret).transpose(1, 2).float().cpu().numpy()
    for b, (qb, kb, vb, _) in enumerate(parts):
        ref32 = _oracle(qb, kb, vb, base, k_ret)
        mx, mean = err_stats(out[b:b + 1], ref32)
        assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (b, mx, mean)


GOLDEN = json.load(open(os.path.join(HERE, "golden", "attn_cases.json")))


@pytest.mark.parametrize("case", GOLDEN["prefill"], ids=lambda c: c["name"])
def test_prefill_against_golden(cuda_device, case):
    """Kernel vs the reference's own recorded fp32 outputs (tests/golden), window
    on (every recorded k) and off, at RoPE bases 1e4, 5e5 and 1e7."""
    gold = np.load(os.path.join(HERE, "golden", f"attn_{case['name']}.npz"))
    q, k, v, _ = make_bhsd(case["hq"], case["hkv"], case["N"], 128, case["base"], case["seed"])
    rows = (np.concatenate([np.arange(t * 128, min((t + 1) * 128, case["N"])) for t in case["tiles"]])
            if "tiles" in case else np.arange(case["N"]))
    for kr in case["k_rets"]:
        tag = "inf" if kr == "inf" else f"{kr:g}"
        k_ret = float("inf") if kr == "inf" else float(kr)
        out = _run(q, k, v, cuda_device, case["base"], k_ret).transpose(1, 2).float().cpu().numpy()[:, :, rows]
        mx, mean = err_stats(out, gold[f"out32_k{tag}"])
        assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (tag, mx, mean)
        assert mx <= 2 * float(gold[f"anchor_k{tag}"]) + 2e-3, (tag, mx)


def test_prefill_pv_path_uniform_scores(cuda_device):
    """q = 0: every score is 0, so row i is the mean of V[0..i]. Checks the P.V
    tcgen05 path (P from TMEM, V MN-major 128B-swizzled) independent of QK."""
    N, hq, hkv = 256, 2, 1
    g = torch.Generator().manual_seed(5)
    q = torch.zeros((1, hq, N, 128), dtype=torch.bfloat16)
    k = torch.randn((1, hkv, N, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((1, hkv, N, 128), generator=g).to(torch.bfloat16)
    out = _run(q, k, v, cuda_device, 1e4, None).transpose(1, 2).float().cpu()
    ref = torch.cumsum(v[0, 0].float(), 0) / torch.arange(1, N + 1)[:, None]
    err = (out[0, 0] - ref).abs().max().item()
    assert err < 1e-2, err


def test_prefill_qk_path_identity_values(cuda_device):
    """Non-causal, 128 keys, V = identity: out = softmax(scale q k^T) row by row.
    Checks the QK tcgen05 path (no-swizzle K-major descriptors, all 8 levels)."""
    atflash = _atf()
    N, hq = 128, 1
    g = torch.Generator().manual_seed(6)
    q = (0.5 * torch.randn((1, N, hq, 128), generator=g)).to(torch.bfloat16)
    k = (0.5 * torch.randn((1, N, 1, 128), generator=g)).to(torch.bfloat16)
    v = torch.eye(128, dtype=torch.bfloat16).reshape(1, N, 1, 128)
    out = atflash.flash_attn_func(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), causal=False)
    torch.cuda.synchronize()
    s = (q[0, :, 0].float() @ k[0, :, 0].float().T) / math.sqrt(128)
    ref = torch.softmax(s, -1)
    err = (out[0, :, 0].float().cpu() - ref).abs().max().item()
    assert err < 5e-3, err


def test_prefill_row_ranges_one_launch(cuda_device):
    """Two row ranges in one launch (a zig-zag rank's blocks): their rows equal the
    same rows of the full run bit for bit, and no other row of out is written."""
    atflash = _atf()
    q, k, v, _ = make_bhsd(6, 2, 1280, 128, 1e4, 31)
    q, k, v = (_bshd(t, cuda_device) for t in (q, k, v))
    wt = atflash.WindowTable(128, 1e4, 2.0)
    full = atflash.prefill_fwd(q, k, v, causal=True, window_table=wt)
    out = torch.full_like(q, 7.0)
    ranges = [(128, 384), (896, 1200)]
    atflash.prefill_fwd(q, k, v, causal=True, window_table=wt, q_offset=0, out=out, row_ranges=ranges)
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    keep = torch.zeros(1280, dtype=torch.bool)
    for (b, e) in ranges:
        keep[b:e] = True
        assert torch.equal(out[:, b:e].view(torch.int16), full[:, b:e].view(torch.int16)), (b, e)
    assert bool((out[:, ~keep.to(cuda_device)] == 7.0).all())


@pytest.mark.parametrize("sq,sk", [(384, 640), (200, 333), (640, 640)])
def test_prefill_noncausal_multi_tile(cuda_device, sq, sk):
    """Non-causal, window off, both query tiles of a CTA over several key tiles
    (equal key-tile counts, so every step's P goes to the other tile's S
    columns), ragged tails: against a plain torch fp32 attention."""
    atflash = _atf()
    hq, hkv = 4, 2
    g = torch.Generator().manual_seed(sq * 1000 + sk)
    q = torch.randn((1, sq, hq, 128), generator=g).to(torch.bfloat16)
    k = torch.randn((1, sk, hkv, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((1, sk, hkv, 128), generator=g).to(torch.bfloat16)
    out = atflash.flash_attn_func(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), causal=False)
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    kk = k.float().repeat_interleave(hq // hkv, dim=2)
    vv = v.float().repeat_interleave(hq // hkv, dim=2)
    s = torch.einsum("bqhd,bkhd->bhqk", q.float(), kk) / math.sqrt(128)
    ref = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, -1), vv)
    mx, mean = err_stats(out.float().cpu().numpy(), ref.numpy())
    assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (mx, mean)


@pytest.mark.parametrize("layout", ["rotate_half"])
def test_prefill_rotate_half_layout(cuda_device, layout):
    """HF rotate_half q/k read in place (level halves are dims [56-8i,64-8i) and
    [120-8i,128-8i)) give the same result as the sorted-pair layout."""
    q, k, v, _ = make_bhsd(6, 2, 640, 128, 1e4, 21)
    a = _run(q, k, v, cuda_device, 1e4, 2.0, layout="sorted_pair")
    b = _run(q, k, v, cuda_device, 1e4, 2.0, layout=layout)
    # the dot products run over the same 16-dim levels in a different order
    assert (a.float() - b.float()).abs().max().item() < 2e-3
    ref = _oracle(q, k, v, 1e4, 2.0)
    mx, mean = err_stats(b.transpose(1, 2).float().cpu().numpy(), ref)
    assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL


def test_window_none_equals_kinf_bitwise(cuda_device):
    """gates/g1_bitexact.py:42-49 analogue: no table == k=inf table, byte for byte."""
    atflash = _atf()
    q, k, v, _ = make_bhsd(7, 1, 900, 128, 1e7, 31)
    q4, k4, v4 = _bshd(q, cuda_device), _bshd(k, cuda_device), _bshd(v, cuda_device)
    a = atflash.flash_attn_func(q4, k4, v4, causal=True)
    b = atflash.flash_attn_func(q4, k4, v4, causal=True, window_table=atflash.WindowTable(128, 1e7, float("inf")))
    c = atflash.flash_attn_func(q4, k4, v4, causal=True, window_table=(2 ** 31 - 1,) * 8)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    assert torch.equal(a.view(torch.int16), c.view(torch.int16))


def test_chunked_prefill_is_neutral(cuda_device):
    """gates/c0_chunk_neutrality.py analogue: a bottom-right chunk (q_offset =
    start, on the tile grid) reproduces the single-shot rows bit for bit, window
    on and off, since windows use global positions."""
    atflash = _atf()
    q, k, v, _ = make_bhsd(4, 2, 1280, 128, 1e4, 41)
    q4, k4, v4 = _bshd(q, cuda_device), _bshd(k, cuda_device), _bshd(v, cuda_device)
    for wt in (None, atflash.WindowTable(128, 1e4, 2.0)):
        full = atflash.flash_attn_func(q4, k4, v4, causal=True, window_table=wt)
        for s in (256, 640, 1152):
            part = atflash.flash_attn_func(q4[:, s:], k4, v4, causal=True, window_table=wt)
            assert torch.equal(part.view(torch.int16), full[:, s:].view(torch.int16)), s
        # a middle chunk with keys up to its end
        part = atflash.flash_attn_func(q4[:, 384:768], k4[:, :768], v4[:, :768], causal=True, window_table=wt)
        assert torch.equal(part.view(torch.int16), full[:, 384:768].view(torch.int16))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_zigzag_shards_equal_single_run(cuda_device, world):
    """Every rank's zig-zag blocks equal the same rows of the 1-GPU output."""
    atflash = _atf()
    q, k, v, _ = make_bhsd(7, 1, 4096, 128, 1e7, 51)
    q4, k4, v4 = _bshd(q, cuda_device), _bshd(k, cuda_device), _bshd(v, cuda_device)
    wt = atflash.WindowTable(128, 1e7, 2.0)
    full = atflash.flash_attn_func(q4, k4, v4, causal=True, window_table=wt)
    covered = 0
    for r in range(world):
        for (s, e, o) in atflash.dist.sharded_prefill(q4, k4, v4, rank=r, world=world, window_table=wt):
            covered += e - s
            assert torch.equal(o.view(torch.int16), full[:, s:e].view(torch.int16)), (r, s, e)
    assert covered == 4096


def test_prefill_lse(cuda_device):
    atflash = _atf()
    q, k, v, _ = make_bhsd(6, 2, 500, 128, 1e4, 61)
    w = OWT.wavelengths_sorted(128, 1e4, 2.0)
    ref, lse_ref = OA.ref_window_attn(to_np(q), to_np(k), to_np(v), w, phase="prefill", block_m=128,
                                      block_n=BN, return_lse=True)
    out, lse = atflash.prefill_fwd(_bshd(q, cuda_device), _bshd(k, cuda_device), _bshd(v, cuda_device),
                                   window_table=atflash.WindowTable(128, 1e4, 2.0), return_lse=True)
    torch.cuda.synchronize()
    assert np.abs(lse.cpu().numpy() - lse_ref).max() < 2e-3


def test_fa4_compat_entry(cuda_device):
    """_flash_attn_fwd(..., atflash_window_zhi=tuple) as the reference calls it."""
    atflash = _atf()
    q, k, v, _ = make_bhsd(6, 2, 384, 128, 5e5, 71)
    zhi = atflash.window_table.window_zhi_from_kret(128, 5e5, 2.0, 262144)
    out, lse = atflash._flash_attn_fwd(_bshd(q, cuda_device), _bshd(k, cuda_device), _bshd(v, cuda_device),
                                       causal=True, pack_gqa=True, atflash_window_zhi=zhi)
    ref = _oracle(q, k, v, 5e5, 2.0)
    mx, mean = err_stats(out.transpose(1, 2).float().cpu().numpy(), ref)
    assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL


def test_prefill_full_size_sampled_tiles(cuda_device):
    """BASELINE config 2 shape (28/4/128, theta 1e7, k=2) at N = 131072: every
    output row of three sampled query tiles (first, middle, last) against the
    oracle. Inputs are N(0,1) bf16 drawn on the device (the reference's
    microbench convention), treated as post-RoPE sorted-pair tensors."""
    atflash = _atf()
    N, hq, hkv = 131072, 28, 4
    g = torch.Generator(device=cuda_device).manual_seed(2026)
    q = torch.randn((1, N, hq, 128), generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn((1, N, hkv, 128), generator=g, device=cuda_device).to(torch.bfloat16)
    v = torch.randn((1, N, hkv, 128), generator=g, device=cuda_device).to(torch.bfloat16)
    wt = atflash.WindowTable(128, 1e7, 2.0)
    out = atflash.flash_attn_func(q, k, v, causal=True, window_table=wt)
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    tiles = [0, 511, 1023]
    heads = [0, 13, 27]
    w = OWT.wavelengths_sorted(128, 1e7, 2.0)
    for t in tiles:
        hi = (t + 1) * 128
        for h in heads:
            hk = h // 7
            qn = q[:, t * 128:hi, h:h + 1].transpose(1, 2).float().cpu().numpy()
            kn = k[:, :hi, hk:hk + 1].transpose(1, 2).float().cpu().numpy()
            vn = v[:, :hi, hk:hk + 1].transpose(1, 2).float().cpu().numpy()
            ref = OA.ref_window_attn(qn, kn, vn, w, phase="prefill", block_m=BM, block_n=BN,
                                     q_offset=t * 128)
            got = out[:, t * 128:hi, h:h + 1].transpose(1, 2).float().cpu().numpy()
            mx, mean = err_stats(got, ref)
            assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (t, h, mx, mean)


def test_prefill_512k_sampled_tiles(cuda_device):
    """BASELINE config 4 shape (N = 524288, 28/4/128, theta 1e7, k=2): every
    output row of two sampled query tiles (middle, last) of two heads against
    the oracle, as the reference checks large N on a subset (head-subset parity)."""
    atflash = _atf()
    N, hq, hkv = 524288, 28, 4
    g = torch.Generator(device=cuda_device).manual_seed(2027)
    q = torch.randn((1, N, hq, 128), generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn((1, N, hkv, 128), generator=g, device=cuda_device).to(torch.bfloat16)
    v = torch.randn((1, N, hkv, 128), generator=g, device=cuda_device).to(torch.bfloat16)
    wt = atflash.WindowTable(128, 1e7, 2.0)
    out = atflash.flash_attn_func(q, k, v, causal=True, window_table=wt)
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    w = OWT.wavelengths_sorted(128, 1e7, 2.0)
    for t in (2047, 4095):
        hi = (t + 1) * 128
        for h in (5, 26):
            hk = h // 7
            qn = q[:, t * 128:hi, h:h + 1].transpose(1, 2).float().cpu().numpy()
            kn = k[:, :hi, hk:hk + 1].transpose(1, 2).float().cpu().numpy()
            vn = v[:, :hi, hk:hk + 1].transpose(1, 2).float().cpu().numpy()
            ref = OA.ref_window_attn(qn, kn, vn, w, phase="prefill", block_m=BM, block_n=BN,
                                     q_offset=t * 128)
            got = out[:, t * 128:hi, h:h + 1].transpose(1, 2).float().cpu().numpy()
            mx, mean = err_stats(got, ref)
            assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (t, h, mx, mean)
