"""Paged decode parity on a B200 against the numpy oracle:
ref_window_attn(phase="decode", block_m=1, block_n=1) for the 16-snap window
(per-key levels) and ref_decode_sliced (gates/g2_correctness.py:43-70) for the
vec8 window; window off == k=inf bitwise (gates/g1_bitexact.py analogue); split
and KV-sharded runs merged by LSE equal the single run."""
import json
import math
import os

import numpy as np
import pytest
import torch

from _inputs import MAX_ABS_TOL, MEAN_ABS_TOL, err_stats, inv_sorted_perm, rope_tables, rope_hf_torch, sorted_perm
from oracle import attention as OA
from oracle import window_table as OWT

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def make_paged(kv_lens, hq, hkv, page_size, seed, layout="NHD", extra_pages=3):
    """Random post-RoPE (sorted-pair) q and a paged KV cache with a seeded
    permuted page table. Returns device tensors and per-request contiguous K/V."""
    g = torch.Generator().manual_seed(seed)
    npages = [(n + page_size - 1) // page_size for n in kv_lens]
    total = sum(npages) + extra_pages
    perm = torch.randperm(total, generator=g)
    if layout == "NHD":
        kc = torch.randn((total, page_size, hkv, 128), generator=g).to(torch.bfloat16)
        vc = torch.randn((total, page_size, hkv, 128), generator=g).to(torch.bfloat16)
    else:
        kc = torch.randn((total, hkv, page_size, 128), generator=g).to(torch.bfloat16)
        vc = torch.randn((total, hkv, page_size, 128), generator=g).to(torch.bfloat16)
    q = torch.randn((len(kv_lens), hq, 128), generator=g).to(torch.bfloat16)
    indptr = [0]
    indices = []
    c = 0
    for n in npages:
        indices += perm[c:c + n].tolist()
        c += n
        indptr.append(indptr[-1] + n)
    lpl = [((n - 1) % page_size) + 1 for n in kv_lens]
    ks, vs = [], []
    for b, n in enumerate(kv_lens):
        pages = indices[indptr[b]:indptr[b + 1]]
        if layout == "NHD":
            kb = kc[pages].reshape(-1, hkv, 128)[:n]
            vb = vc[pages].reshape(-1, hkv, 128)[:n]
        else:
            kb = kc[pages].permute(0, 2, 1, 3).reshape(-1, hkv, 128)[:n]
            vb = vc[pages].permute(0, 2, 1, 3).reshape(-1, hkv, 128)[:n]
        ks.append(kb.permute(1, 0, 2).contiguous())  # (hkv, n, d)
        vs.append(vb.permute(1, 0, 2).contiguous())
    return (q, kc, vc, torch.tensor(indptr, dtype=torch.int32), torch.tensor(indices, dtype=torch.int32),
            torch.tensor(lpl, dtype=torch.int32), ks, vs)


def oracle_decode(q, ks, vs, base, k_ret):
    w = OWT.wavelengths_sorted(128, base, float("inf") if k_ret is None else k_ret)
    outs = []
    for b in range(q.shape[0]):
        o = OA.ref_window_attn(q[b][None, :, None, :].float().numpy(), ks[b][None].float().numpy(),
                               vs[b][None].float().numpy(), w, phase="decode", block_m=1, block_n=1)
        outs.append(o[0, :, 0, :])
    return np.stack(outs)


def run_decode(dev, q, kc, vc, indptr, indices, lpl, hq, hkv, page, layout="NHD", window_table=None,
               window_mode="snap16", qk_layout="sorted_pair", max_chunk_keys=0, **runkw):
    import atflash
    ws = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, kv_layout=layout)
    w.plan(indptr, indices, lpl, hq, hkv, 128, page, window_table=window_table,
           window_mode=window_mode, qk_layout=qk_layout, max_chunk_keys=max_chunk_keys)
    res = w.run(q.to(dev), (kc.to(dev), vc.to(dev)), **runkw)
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    return res


CASES = [
    # (kv_lens, hq, hkv, page, layout, base, k_ret)
    ([1000, 37, 513], 6, 2, 16, "NHD", 1e4, 2.0),
    ([2048, 777], 24, 8, 16, "NHD", 5e5, 2.0),
    ([3000], 28, 4, 64, "NHD", 1e7, 2.0),
    ([1500, 64, 1], 28, 4, 64, "HND", 1e4, 1.0),
    ([4096, 100], 8, 8, 16, "HND", 1e4, 3.0),
    ([5000], 16, 1, 16, "NHD", 1e4, 2.0),
    ([700, 1200], 4, 2, 16, "NHD", 1e4, 2.0),       # GQA group 2
    ([2500], 16, 4, 64, "NHD", 5e5, 2.0),           # GQA group 4
    ([1800, 33], 32, 4, 16, "HND", 1e4, 2.0),       # GQA group 8
    ([3000, 129], 8, 2, 32, "NHD", 1e4, 2.0),       # page 32
    ([2200, 64], 28, 4, 128, "HND", 1e7, 2.0),      # page 128
    ([4000], 24, 8, 256, "NHD", 5e5, 2.0),          # page 256
    ([300 + 97 * i for i in range(16)], 12, 4, 16, "NHD", 1e4, 2.0),  # 16 ragged requests
]


@pytest.mark.parametrize("window", ["on", "off"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"L{'-'.join(map(str, c[0]))}-h{c[1]}x{c[2]}-p{c[3]}-{c[4]}")
def test_decode_parity(cuda_device, case, window):
    import atflash
    kv_lens, hq, hkv, page, layout, base, k_ret = case
    kr = k_ret if window == "on" else None
    q, kc, vc, indptr, indices, lpl, ks, vs = make_paged(kv_lens, hq, hkv, page, seed=sum(kv_lens) + hq,
                                                        layout=layout)
    wt = atflash.WindowTable(128, base, kr) if kr is not None else None
    out = run_decode(cuda_device, q, kc, vc, indptr, indices, lpl, hq, hkv, page, layout, wt)
    ref = oracle_decode(q, ks, vs, base, kr)
    mx, mean = err_stats(out.float().cpu().numpy(), ref)
    assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (mx, mean)


def test_decode_with_an_empty_request(cuda_device):
    """A batch holding an empty request (no keys, no split items): its output
    is zeros and its LSE -inf; the other requests match the oracle."""
    import atflash
    kv_lens, hq, hkv, page = [700, 0, 300], 6, 2, 16
    q, kc, vc, indptr, indices, lpl, ks, vs = make_paged(kv_lens, hq, hkv, page, seed=77)
    lpl[1] = 1
    wt = atflash.WindowTable(128, 1e4, 2.0)
    out, lse = run_decode(cuda_device, q, kc, vc, indptr, indices, lpl, hq, hkv, page, "NHD", wt,
                          return_lse=True)
    for b in (0, 2):
        ref = oracle_decode(q[b:b + 1], ks[b:b + 1], vs[b:b + 1], 1e4, 2.0)
        mx, mean = err_stats(out[b:b + 1].float().cpu().numpy(), ref)
        assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (b, mx, mean)
    assert torch.all(out[1] == 0) and torch.all(torch.isinf(lse[1]))


def test_decode_many_splits_and_lse(cuda_device):
    """Force 64-key items so a request spans dozens of splits; the merged output
    and LSE match the oracle."""
    import atflash
    kv_lens, hq, hkv, page = [3000, 450], 6, 2, 16
    q, kc, vc, indptr, indices, lpl, ks, vs = make_paged(kv_lens, hq, hkv, page, seed=7)
    wt = atflash.WindowTable(128, 1e4, 2.0)
    out, lse = run_decode(cuda_device, q, kc, vc, indptr, indices, lpl, hq, hkv, page, "NHD", wt,
                          max_chunk_keys=64, return_lse=True)
    ref = oracle_decode(q, ks, vs, 1e4, 2.0)
    mx, mean = err_stats(out.float().cpu().numpy(), ref)
    assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL
    # LSE of the windowed scores (natural log)
    w = OWT.wavelengths_sorted(128, 1e4, 2.0)
    for b in range(2):
        _, lse_ref = OA.ref_window_attn(q[b][None, :, None, :].float().numpy(), ks[b][None].float().numpy(),
                                        vs[b][None].float().numpy(), w, phase="decode", block_m=1,
                                        block_n=1, return_lse=True)
        assert np.abs(lse[b].cpu().numpy() - lse_ref[0, :, 0]).max() < 2e-3


def test_decode_window_off_equals_kinf_bitwise(cuda_device):
    import atflash
    q, kc, vc, indptr, indices, lpl, ks, vs = make_paged([2000, 300], 24, 8, 16, seed=9)
    a = run_decode(cuda_device, q, kc, vc, indptr, indices, lpl, 24, 8, 16, "NHD", None)
    b = run_decode(cuda_device, q, kc, vc, indptr, indices, lpl, 24, 8, 16, "NHD",
                   atflash.WindowTable(128, 5e5, float("inf")))
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("page,level_major,hq,hkv,kv_lens,base", [
    (16, False, 6, 2, [1000, 2500], 1e4),   # TMA kernel
    (8, False, 6, 2, [1000, 2500], 1e4),    # cp.async kernel (page 8)
    (64, True, 28, 4, [20000], 5e5),        # TMA kernel, level-major K, groups of 7
    (16, False, 48, 4, [3000], 1e4),        # groups of 12: cp.async kernel
], ids=["tma-p16", "cpasync-p8", "tma-p64-lm-g7", "cpasync-g12"])
def test_decode_vec8_matches_g2_oracle(cuda_device, page, level_major, hq, hkv, kv_lens, base):
    """vec8 window (the FlashInfer port's 8-dim slices) vs ref_decode_sliced, on
    both decode kernels: the TMA kernel splits a level whose second slice only
    some keys read into two 8-dim MMAs."""
    import atflash
    q, kc, vc, indptr, indices, lpl, ks, vs = make_paged(kv_lens, hq, hkv, page, seed=13)
    wt = atflash.WindowTable(128, base, 2.0)
    if level_major:
        kc = _level_major(kc)
    out = run_decode(cuda_device, q, kc, vc, indptr, indices, lpl, hq, hkv, page, "NHD", wt, window_mode="vec8")
    zs = OWT.zhi_slice_vec8(128, base, 2.0)
    for b in range(len(kv_lens)):
        ref = OA.ref_decode_sliced(q[b].float().numpy(), ks[b].permute(1, 0, 2).float().numpy(),
                                   vs[b].permute(1, 0, 2).float().numpy(), zs, 8)
        mx, mean = err_stats(out[b].float().cpu().numpy(), ref)
        assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL


GOLDEN = json.load(open(os.path.join(HERE, "golden", "attn_cases.json")))


@pytest.mark.parametrize("page", [1, 16])
@pytest.mark.parametrize("case", GOLDEN["decode"], ids=lambda c: c["name"])
def test_decode_against_golden(cuda_device, case, page):
    """Kernel vs the reference's recorded decode outputs, window on (every
    recorded k, 16-snap and vec8) and off. The contiguous KV is cut into pages
    of 1 token (the cp.async kernel) or 16 tokens (the TMA kernel)."""
    from _inputs import make_bhsd
    import atflash
    gold = np.load(os.path.join(HERE, "golden", f"attn_{case['name']}.npz"))
    q, k, v, _ = make_bhsd(case["hq"], case["hkv"], case["N"], 128, case["base"], case["seed"], phase="decode")
    N, hkv = case["N"], case["hkv"]
    npg = (N + page - 1) // page
    pad = npg * page - N
    kt = torch.cat([k[0].permute(1, 0, 2), torch.zeros((pad, hkv, 128), dtype=k.dtype)])
    vt = torch.cat([v[0].permute(1, 0, 2), torch.zeros((pad, hkv, 128), dtype=v.dtype)])
    kc = kt.reshape(npg, page, hkv, 128).contiguous()  # NHD pages in order
    vc = vt.reshape(npg, page, hkv, 128).contiguous()
    indptr = torch.tensor([0, npg], dtype=torch.int32)
    indices = torch.arange(npg, dtype=torch.int32)
    lpl = torch.tensor([N - (npg - 1) * page], dtype=torch.int32)
    for kr in case["k_rets"]:
        tag = "inf" if kr == "inf" else f"{kr:g}"
        wt = None if kr == "inf" else atflash.WindowTable(128, case["base"], float(kr))
        out = run_decode(cuda_device, q[0, :, 0][None], kc, vc, indptr, indices, lpl, case["hq"], hkv, page,
                         "NHD", wt)
        mx, mean = err_stats(out[0].float().cpu().numpy(), gold[f"out32_k{tag}"][0, :, 0])
        assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (tag, mx, mean)
        if wt is not None:
            out8 = run_decode(cuda_device, q[0, :, 0][None], kc, vc, indptr, indices, lpl, case["hq"], hkv, page,
                              "NHD", wt, window_mode="vec8")
            mx, mean = err_stats(out8[0].float().cpu().numpy(), gold[f"vec8_k{tag}"])
            assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (tag, mx, mean)


def test_decode_rotate_half_cache(cuda_device):
    """A cache holding K in HF rotate_half order (and q likewise) gives the
    sorted-layout result."""
    import atflash
    kv_lens, hq, hkv = [1200, 90], 6, 2
    q, kc, vc, indptr, indices, lpl, ks, vs = make_paged(kv_lens, hq, hkv, 16, seed=17)
    inv = inv_sorted_perm(128)
    wt = atflash.WindowTable(128, 1e4, 2.0)
    a = run_decode(cuda_device, q, kc, vc, indptr, indices, lpl, hq, hkv, 16, "NHD", wt)
    b = run_decode(cuda_device, q[..., inv].contiguous(), kc[..., inv].contiguous(), vc, indptr, indices, lpl,
                   hq, hkv, 16, "NHD", wt, qk_layout="rotate_half")
    assert (a.float() - b.float()).abs().max().item() < 2e-3


def test_kv_sharded_decode_merge(cuda_device):
    """Two KV shards with global positions (kv_pos0) merged by LSE equal the full
    decode: the single-GPU emulation of atflash.dist.sharded_decode."""
    import atflash
    N, hq, hkv, page = 4096, 28, 4, 64
    q, kc, vc, indptr, indices, lpl, ks, vs = make_paged([N], hq, hkv, page, seed=23)
    wt = atflash.WindowTable(128, 1e7, 64.0)
    full = run_decode(cuda_device, q, kc, vc, indptr, indices, lpl, hq, hkv, page, "NHD", wt)
    pages = indices.tolist()
    parts_o, parts_l = [], []
    for r, (p0, p1) in enumerate([(0, 24), (24, 64)]):
        sub_idx = torch.tensor(pages[p0:p1], dtype=torch.int32)
        o, l = run_decode(cuda_device, q, kc, vc, torch.tensor([0, p1 - p0], dtype=torch.int32), sub_idx,
                          torch.tensor([page], dtype=torch.int32), hq, hkv, page, "NHD", wt,
                          q_pos=torch.tensor([N - 1]), kv_pos0=torch.tensor([p0 * page]),
                          return_lse=True, out_dtype=torch.float32)
        parts_o.append(o)
        parts_l.append(l)
    merged = atflash.lse_merge(torch.stack(parts_o), torch.stack(parts_l))
    torch.cuda.synchronize()
    assert (merged.float() - full.float()).abs().max().item() < 4e-3
    ref = oracle_decode(q, ks, vs, 1e7, 64.0)
    mx, mean = err_stats(merged.float().cpu().numpy(), ref)
    assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL


def test_decode_rejects_wrong_out_and_lse_buffers(cuda_device):
    """Caller-supplied out / lse of the wrong shape or dtype are refused before any
    launch."""
    kv_lens, hq, hkv, page = [300, 40], 6, 2, 16
    q, kc, vc, indptr, indices, lpl, ks, vs = make_paged(kv_lens, hq, hkv, page, seed=41)
    bad_outs = [torch.empty((2, hq, 64), dtype=torch.bfloat16, device=cuda_device),
                torch.empty((2, hq, 128), dtype=torch.float16, device=cuda_device)]
    for bad in bad_outs:
        with pytest.raises((ValueError, TypeError)):
            run_decode(cuda_device, q, kc, vc, indptr, indices, lpl, hq, hkv, page, "NHD", None, out=bad)
    with pytest.raises(ValueError):
        run_decode(cuda_device, q, kc, vc, indptr, indices, lpl, hq, hkv, page, "NHD", None, return_lse=True,
                   lse=torch.empty((2, hq + 1), dtype=torch.float32, device=cuda_device))


def test_lse_merge_strided_parts_equal_packed(cuda_device):
    """Parts laid out as one flat buffer per rank (O block, then the LSE block
    padded to 4 floats), as atflash.dist all-gathers them, merge in place to the
    same bits as the packed (P, B, H, 128) / (P, B, H) layout."""
    import atflash
    P, B, H, D = 3, 2, 7, 128
    g = torch.Generator(device="cpu").manual_seed(31)
    po = torch.randn((P, B, H, D), generator=g).to(cuda_device)
    pl = (3 * torch.randn((P, B, H), generator=g)).to(cuda_device)
    pl[1, 0, 2] = -float("inf")  # an empty part
    n_o, n_l = B * H * D, (B * H + 3) // 4 * 4
    flat = torch.full((P * (n_o + n_l),), float("nan"), device=cuda_device)
    for r in range(P):
        flat[r * (n_o + n_l): r * (n_o + n_l) + n_o] = po[r].reshape(-1)
        flat[r * (n_o + n_l) + n_o: r * (n_o + n_l) + n_o + B * H] = pl[r].reshape(-1)
    vo = flat.as_strided((P, B, H, D), (n_o + n_l, H * D, D, 1))
    vl = flat.as_strided((P, B, H), (n_o + n_l, H, 1), n_o)
    for dt in (torch.float32, torch.bfloat16):
        o1, l1 = atflash.lse_merge(po, pl, out_dtype=dt, return_lse=True)
        o2, l2 = atflash.lse_merge(vo, vl, out_dtype=dt, return_lse=True)
        torch.cuda.synchronize()
        assert torch.equal(o1, o2) and torch.equal(l1, l2)
        assert not torch.isnan(o2.float()).any()


def test_rope_pack_bit_exact(cuda_device):
    """Fused RoPE + pack equals the reference front-end (fp32 rotate_half RoPE,
    permutation, bf16) bit for bit given the same cos/sin tables."""
    import atflash
    g = torch.Generator().manual_seed(3)
    B, S, H = 2, 333, 5
    x = torch.randn((B, S, H, 128), generator=g).to(torch.bfloat16)
    cos, sin = rope_tables(S + 50, 128, 5e5)
    for off in (0, 50):
        c, s_ = cos[off:off + S][None, :, None, :], sin[off:off + S][None, :, None, :]
        ref_rh = rope_hf_torch(x, c, s_).to(torch.bfloat16)
        ref_sp = rope_hf_torch(x, c, s_)[..., sorted_perm(128)].to(torch.bfloat16)
        got_rh = atflash.rope_pack(x.to(cuda_device), cos.to(cuda_device), sin.to(cuda_device), pos_offset=off,
                                   out_layout="rotate_half")
        got_sp = atflash.rope_pack(x.to(cuda_device), cos.to(cuda_device), sin.to(cuda_device), pos_offset=off,
                                   out_layout="sorted_pair")
        torch.cuda.synchronize()
        assert torch.equal(got_rh.cpu().view(torch.int16), ref_rh.view(torch.int16))
        assert torch.equal(got_sp.cpu().view(torch.int16), ref_sp.view(torch.int16))


def test_prefill_with_rope_end_to_end(cuda_device):
    """flash_attn_func(rope=(cos, sin)) on pre-RoPE HF tensors equals the oracle on
    the reference front-end's post-RoPE sorted tensors."""
    import atflash
    from _inputs import make_bhsd
    q, k, v, (q0, k0, cos, sin) = make_bhsd(6, 2, 640, 128, 5e5, 29)
    dev = cuda_device
    out = atflash.flash_attn_func(q0.transpose(1, 2).contiguous().to(dev), k0.transpose(1, 2).contiguous().to(dev),
                                  v.transpose(1, 2).contiguous().to(dev), causal=True,
                                  window_table=atflash.WindowTable(128, 5e5, 2.0),
                                  rope=(cos.to(dev), sin.to(dev)))
    torch.cuda.synchronize()
    w = OWT.wavelengths_sorted(128, 5e5, 2.0)
    ref = OA.ref_window_attn(q.float().numpy(), k.float().numpy(), v.float().numpy(), w, phase="prefill",
                             block_m=128, block_n=128)
    mx, mean = err_stats(out.transpose(1, 2).float().cpu().numpy(), ref)
    assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL
    # q is rotated inside the prefill as it is loaded: bit-identical to running
    # the kernel on the front-end's post-RoPE sorted-pair tensors
    pre = atflash.flash_attn_func(q.transpose(1, 2).contiguous().to(dev), k.transpose(1, 2).contiguous().to(dev),
                                  v.transpose(1, 2).contiguous().to(dev), causal=True,
                                  window_table=atflash.WindowTable(128, 5e5, 2.0))
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), pre.view(torch.int16))
    # a chunk of the queries (rows 384..639 at positions 384..639) against all keys
    part = atflash.flash_attn_func(q0.transpose(1, 2)[:, 384:].contiguous().to(dev),
                                   k0.transpose(1, 2).contiguous().to(dev), v.transpose(1, 2).contiguous().to(dev),
                                   causal=True, window_table=atflash.WindowTable(128, 5e5, 2.0),
                                   rope=(cos.to(dev), sin.to(dev)), q_offset=384)
    torch.cuda.synchronize()
    assert torch.equal(part.view(torch.int16), out[:, 384:].view(torch.int16))


def _level_major(kc):
    """(P, page, Hkv, 128) NHD sorted-pair K pages -> level-major (P, Hkv, 8, page, 16)."""
    P, page, hkv, _ = kc.shape
    return kc.view(P, page, hkv, 8, 16).permute(0, 2, 3, 1, 4).contiguous()


@pytest.mark.parametrize("page,k_ret", [(16, 2.0), (64, 2.0), (16, None), (128, 1.0)])
def test_decode_level_major_k_pages_equal_nhd(cuda_device, page, k_ret):
    """Level-major K pages (a page's in-window levels contiguous) give the same
    decode as the NHD pages they were laid out from, bit for bit."""
    import atflash
    lens, hq, hkv = [3000, 517, 64], 24, 8
    q, kc, vc, indptr, indices, lpl, _, _ = make_paged(lens, hq, hkv, page, 40 + page)
    wt = atflash.WindowTable(128, 1e4, k_ret) if k_ret is not None else None
    ref = run_decode(cuda_device, q, kc, vc, indptr, indices, lpl, hq, hkv, page, window_table=wt)
    got = run_decode(cuda_device, q, _level_major(kc), vc, indptr, indices, lpl, hq, hkv, page, window_table=wt)
    assert torch.equal(ref, got)


@pytest.mark.parametrize("qk_layout", ["sorted_pair", "rotate_half"])
def test_decode_pdl_bit_identical(cuda_device, qk_layout):
    """enable_pdl=True (the decode launched as a programmatic dependent of the
    previous kernel) gives the plain launch's bits, on the TMA kernel (sorted
    pairs) and on the general kernel (rotate_half), also when the kernel just
    before the decode rewrites the query and a KV page: those are read after
    the decode's wait for the previous grid."""
    import atflash
    kv_lens, hq, hkv, page = [3000, 700, 64], 24, 8, 16
    q, kc, vc, indptr, indices, lpl, _, _ = make_paged(kv_lens, hq, hkv, page, seed=23)
    q, kc, vc = q.to(cuda_device), kc.to(cuda_device), vc.to(cuda_device)
    w = atflash.BatchDecodeWithPagedKVCacheWrapper(torch.empty(64 << 20, dtype=torch.uint8, device=cuda_device),
                                                   "NHD")
    w.plan(indptr, indices, lpl, hq, hkv, 128, page, window_table=atflash.WindowTable(128, 5e5, 2.0),
           qk_layout=qk_layout)
    g = torch.Generator(device=cuda_device).manual_seed(3)
    out_p = torch.empty((len(kv_lens), hq, 128), dtype=torch.bfloat16, device=cuda_device)
    pg = int(indices[5])
    for step in range(3):
        # kernels that write the decode's inputs, directly before each decode
        q.copy_(torch.randn(q.shape, generator=g, device=cuda_device).to(torch.bfloat16))
        kc[pg].mul_(-1.0)
        w.run(q, (kc, vc), out=out_p, enable_pdl=True)
        ref = w.run(q, (kc, vc))
        torch.cuda.synchronize()
        assert torch.equal(out_p.view(torch.int16), ref.view(torch.int16)), step
    # back to back, the next decode launched while the previous merge runs
    outs = [w.run(q, (kc, vc), enable_pdl=True) for _ in range(4)]
    torch.cuda.synchronize()
    assert all(torch.equal(o.view(torch.int16), ref.view(torch.int16)) for o in outs)
    assert atflash.check_device_errors() == 0
