"""Parity at the BASELINE target configurations, on a B200, against the numpy
oracle (ref_window_attn of atflash/reference.py:27-80, pinned to the reference
by test_oracle_golden.py).

The full-size inputs are N(0,1) bf16 drawn on the device (the reference's
microbench convention) and taken as post-RoPE sorted-pair tensors. The oracle is
run on a subset that keeps its cost to seconds: for decode, a few (request, kv
head) pairs, each with its whole GQA group of query heads and every key; for
prefill, every row of sampled 128-row query tiles for sampled heads.

  config 3  paged decode, batch 8, 24/8 heads, page 16, theta 5e5, seeded
            permuted page table, 8K / 32K / 128K keys, window k=2 and off
  config 5  one 1M-key request, 28/4 heads, page 64, theta 1e7, window k=64 and
            off; also the KV sequence cut into 4 shards with global positions
            and merged by LSE (the single-GPU emulation of the 4-GPU step)
  (decode)  the same cache with level-major K pages gives bit-identical output
  config 2  128K prefill, 28/4 heads, theta 1e7, window k=2, k=64 and off

Pass bar: max |err| <= 2e-2 and mean |err| <= 2e-3 against the fp32 oracle."""
import numpy as np
import pytest
import torch

from _inputs import MAX_ABS_TOL, MEAN_ABS_TOL, err_stats
from oracle import attention as OA
from oracle import window_table as OWT

pytestmark = pytest.mark.gpu
D = 128


def _paged_device_cache(dev, B, N, hq, hkv, page, seed):
    """Device q and NHD KV pages of B requests of N keys each, with a seeded
    permuted page table (torch.randperm on the CPU, as the bench builds it)."""
    npg = (N + page - 1) // page
    total = B * npg
    g = torch.Generator(device="cpu").manual_seed(seed)
    perm = torch.randperm(total, generator=g).to(torch.int32)
    gd = torch.Generator(device=dev).manual_seed(seed + 1)
    kc = torch.randn((total, page, hkv, D), generator=gd, device=dev).to(torch.bfloat16)
    vc = torch.randn((total, page, hkv, D), generator=gd, device=dev).to(torch.bfloat16)
    q = torch.randn((B, hq, D), generator=gd, device=dev).to(torch.bfloat16)
    indptr = torch.arange(0, total + 1, npg, dtype=torch.int32)
    lpl = torch.full((B,), N - (npg - 1) * page, dtype=torch.int32)
    return q, kc, vc, indptr, perm, lpl


def _request_head(kc, vc, perm, indptr, b, hk, N):
    """(N, d) fp32 numpy K and V of request b, kv head hk, in key order."""
    pages = perm[indptr[b]:indptr[b + 1]].to(kc.device).long()
    k = kc[pages, :, hk].reshape(-1, D)[:N]
    v = vc[pages, :, hk].reshape(-1, D)[:N]
    return k.float().cpu().numpy(), v.float().cpu().numpy()


def _level_major(kc):
    """The same K pages level-major, (P, Hkv, 8, page, 16): the cache layout
    atf_paged_kv_append writes with k_level_major."""
    P, page, hkv, _ = kc.shape
    return kc.view(P, page, hkv, 8, 16).permute(0, 2, 3, 1, 4).contiguous()


def _oracle_decode_group(q_group, k, v, w):
    """ref_window_attn(phase="decode", block_m=1, block_n=1) for the G query
    heads of one kv head: q_group (G, d), k/v (N, d) -> (G, d)."""
    o = OA.ref_window_attn(q_group[None, :, None, :], k[None, None], v[None, None], w, phase="decode",
                           block_m=1, block_n=1)
    return o[0, :, 0, :]


def _run_decode(dev, q, kc, vc, indptr, perm, lpl, hq, hkv, page, wt, **kw):
    import atflash
    ws = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
    w.plan(indptr, perm, lpl, hq, hkv, D, page, window_table=wt)
    res = w.run(q, (kc, vc), **kw)
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    return res


@pytest.mark.parametrize("N", [8192, 32768, 131072], ids=lambda n: f"{n // 1024}K")
def test_decode_config3(cuda_device, N):
    """BASELINE config 3 at 8K / 32K / 128K keys, window k=2 and off: requests 0
    and 7, kv heads 0, 3 and 7 (q heads 0-2, 9-11, 21-23), every key."""
    import atflash
    B, hq, hkv, page, base = 8, 24, 8, 16, 5e5
    G = hq // hkv
    q, kc, vc, indptr, perm, lpl = _paged_device_cache(cuda_device, B, N, hq, hkv, page, 1234 + N + D)
    for k_ret in (2.0, None):
        wt = atflash.WindowTable(D, base, k_ret) if k_ret is not None else None
        out_t = _run_decode(cuda_device, q, kc, vc, indptr, perm, lpl, hq, hkv, page, wt)
        # level-major K pages hold the same values: the same bits out
        out_lm = _run_decode(cuda_device, q, _level_major(kc), vc, indptr, perm, lpl, hq, hkv, page, wt)
        assert torch.equal(out_lm.view(torch.int16), out_t.view(torch.int16)), k_ret
        out = out_t.float().cpu().numpy()
        w = OWT.wavelengths_sorted(D, base, float("inf") if k_ret is None else k_ret)
        for b in (0, B - 1):
            for hk in (0, 3, hkv - 1):
                k, v = _request_head(kc, vc, perm, indptr, b, hk, N)
                ref = _oracle_decode_group(q[b, hk * G:(hk + 1) * G].float().cpu().numpy(), k, v, w)
                mx, mean = err_stats(out[b, hk * G:(hk + 1) * G], ref)
                assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (k_ret, b, hk, mx, mean)


def test_decode_config5_1m(cuda_device):
    """one 1,048,576-key request, page 64, 28/4 heads, theta
    1e7, window k=64 and off, kv heads 0 and 3 against the oracle; and the same
    request cut into 4 contiguous KV shards (global key positions through
    kv_pos0 / q_pos), each decoded on its own and merged by LSE, against the
    single run (the 4-GPU sharded step emulated on one GPU)."""
    import atflash
    N, hq, hkv, page, base = 1 << 20, 28, 4, 64, 1e7
    G = hq // hkv
    q, kc, vc, indptr, perm, lpl = _paged_device_cache(cuda_device, 1, N, hq, hkv, page, 4242)
    npg = N // page
    for k_ret in (64.0, None):
        wt = atflash.WindowTable(D, base, k_ret) if k_ret is not None else None
        out = _run_decode(cuda_device, q, kc, vc, indptr, perm, lpl, hq, hkv, page, wt)
        out_lm = _run_decode(cuda_device, q, _level_major(kc), vc, indptr, perm, lpl, hq, hkv, page, wt)
        assert torch.equal(out_lm.view(torch.int16), out.view(torch.int16)), k_ret
        del out_lm
        w = OWT.wavelengths_sorted(D, base, float("inf") if k_ret is None else k_ret)
        outn = out.float().cpu().numpy()
        for hk in (0, hkv - 1):
            k, v = _request_head(kc, vc, perm, indptr, 0, hk, N)
            ref = _oracle_decode_group(q[0, hk * G:(hk + 1) * G].float().cpu().numpy(), k, v, w)
            mx, mean = err_stats(outn[0, hk * G:(hk + 1) * G], ref)
            assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (k_ret, hk, mx, mean)
        shards = 4
        parts_o, parts_l = [], []
        for r in range(shards):
            p0, p1 = r * npg // shards, (r + 1) * npg // shards
            o, l = _run_decode(cuda_device, q, kc, vc, torch.tensor([0, p1 - p0], dtype=torch.int32),
                               perm[p0:p1].contiguous(), torch.tensor([page], dtype=torch.int32), hq, hkv, page,
                               wt, q_pos=torch.tensor([N - 1]), kv_pos0=torch.tensor([p0 * page]),
                               return_lse=True, out_dtype=torch.float32)
            parts_o.append(o)
            parts_l.append(l)
        merged = atflash.lse_merge(torch.stack(parts_o), torch.stack(parts_l))
        torch.cuda.synchronize()
        assert (merged.float() - out.float()).abs().max().item() < 4e-3, k_ret


@pytest.mark.parametrize("k_ret", [2.0, 64.0, None], ids=["k2", "k64", "off"])
def test_prefill_config2_sampled_tiles(cuda_device, k_ret):
    """BASELINE config 2 (N = 131072, 28/4 heads, theta 1e7) with the window at
    k=2, k=64 and off: every row of query tiles 0, 300, 700 and 1023 for q heads
    0, 13 and 27 against the oracle (all keys of each tile's causal range)."""
    import atflash
    N, hq, hkv, base = 131072, 28, 4, 1e7
    G = hq // hkv
    g = torch.Generator(device=cuda_device).manual_seed(2026)
    q = torch.randn((1, N, hq, D), generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn((1, N, hkv, D), generator=g, device=cuda_device).to(torch.bfloat16)
    v = torch.randn((1, N, hkv, D), generator=g, device=cuda_device).to(torch.bfloat16)
    wt = atflash.WindowTable(D, base, k_ret) if k_ret is not None else None
    out = atflash.flash_attn_func(q, k, v, causal=True, window_table=wt)
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    w = OWT.wavelengths_sorted(D, base, float("inf") if k_ret is None else k_ret)
    for t in (0, 300, 700, 1023):
        hi = (t + 1) * 128
        for h in (0, 13, 27):
            hk = h // G
            qn = q[:, t * 128:hi, h:h + 1].transpose(1, 2).float().cpu().numpy()
            kn = k[:, :hi, hk:hk + 1].transpose(1, 2).float().cpu().numpy()
            vn = v[:, :hi, hk:hk + 1].transpose(1, 2).float().cpu().numpy()
            ref = OA.ref_window_attn(qn, kn, vn, w, phase="prefill", block_m=128, block_n=128, q_offset=t * 128)
            got = out[:, t * 128:hi, h:h + 1].transpose(1, 2).float().cpu().numpy()
            mx, mean = err_stats(got, ref)
            assert mx <= MAX_ABS_TOL and mean <= MEAN_ABS_TOL, (k_ret, t, h, mx, mean)
