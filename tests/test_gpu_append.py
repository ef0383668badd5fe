"""Paged-KV append on a B200: tokens land in the right (page, slot, head) for
both cache layouts, bit for bit with a torch scatter; with RoPE at write, K
equals the fused RoPE pack of the same tokens; out-of-range page indices are
skipped and flagged; a decode over an appended cache equals the decode over
the same cache written directly."""
import pytest
import torch

from _inputs import rope_tables

pytestmark = pytest.mark.gpu


def _setup(layout, seed, page=16, hkv=4, lens=(37, 80, 5), extra_pages=4):
    g = torch.Generator().manual_seed(seed)
    npg = [(n + page - 1) // page for n in lens]
    total = sum(npg) + extra_pages
    perm = torch.randperm(total, generator=g).to(torch.int32)
    indptr = [0]
    for n in npg:
        indptr.append(indptr[-1] + n)
    shape = (total, page, hkv, 128) if layout == "NHD" else (total, hkv, page, 128)
    kc = torch.randn(shape, generator=g).to(torch.bfloat16)
    vc = torch.randn(shape, generator=g).to(torch.bfloat16)
    return g, kc, vc, torch.tensor(indptr, dtype=torch.int32), perm[: indptr[-1]].contiguous(), list(lens)


def _ref_scatter(kc, vc, k, v, bidx, pos, indptr, indices, layout, page):
    kc, vc = kc.clone(), vc.clone()
    for i in range(k.shape[0]):
        b, p = int(bidx[i]), int(pos[i])
        pg = int(indices[int(indptr[b]) + p // page])
        if layout == "NHD":
            kc[pg, p % page] = k[i]
            vc[pg, p % page] = v[i]
        else:
            kc[pg, :, p % page] = k[i]
            vc[pg, :, p % page] = v[i]
    return kc, vc


@pytest.mark.parametrize("layout", ["NHD", "HND"])
def test_append_matches_torch_scatter(layout):
    import atflash
    dev = torch.device("cuda:0")
    g, kc, vc, indptr, indices, lens = _setup(layout, 11)
    # append the last 20 / 33 / 5 tokens of each request
    app = [20, 33, 5]
    append_indptr = torch.tensor([0, 20, 53, 58])
    bidx, pos = atflash.get_batch_indices_positions(append_indptr, torch.tensor(lens), 58)
    k = torch.randn((58, 4, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((58, 4, 128), generator=g).to(torch.bfloat16)
    ref_k, ref_v = _ref_scatter(kc, vc, k, v, bidx, pos, indptr, indices, layout, 16)
    kd, vd = kc.to(dev), vc.to(dev)
    atflash.append_paged_kv_cache(k.to(dev), v.to(dev), bidx.to(dev), pos.to(dev), (kd, vd),
                                  indices.to(dev), indptr.to(dev), kv_layout=layout)
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    assert torch.equal(kd.cpu(), ref_k) and torch.equal(vd.cpu(), ref_v)
    assert sum(app) == 58


@pytest.mark.parametrize("out_layout", ["sorted_pair", "rotate_half"])
def test_append_with_rope_equals_rope_pack(out_layout):
    import atflash
    dev = torch.device("cuda:0")
    g, kc, vc, indptr, indices, lens = _setup("NHD", 12)
    nnz = sum(lens)
    bidx, pos = atflash.get_batch_indices_positions(torch.tensor([0, 37, 117, 122]), torch.tensor(lens), nnz)
    k = torch.randn((nnz, 4, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((nnz, 4, 128), generator=g).to(torch.bfloat16)
    cos, sin = rope_tables(200, 128, 1e4)
    kd, vd = kc.to(dev), vc.to(dev)
    atflash.append_paged_kv_cache(k.to(dev), v.to(dev), bidx.to(dev), pos.to(dev), (kd, vd), indices.to(dev),
                                  indptr.to(dev), rope=(cos.to(dev), sin.to(dev)), out_layout=out_layout)
    # expected K: the fused RoPE pack of each token at its own position
    kr = atflash.rope_pack(k.to(dev)[None], cos.to(dev), sin.to(dev), positions=pos.to(dev).long(),
                           out_layout=out_layout)[0].cpu()
    ref_k, ref_v = _ref_scatter(kc, vc, kr, v, bidx, pos, indptr, indices, "NHD", 16)
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    assert torch.equal(kd.cpu(), ref_k) and torch.equal(vd.cpu(), ref_v)


def test_append_out_of_range_pages_are_flagged_and_skipped():
    import atflash
    dev = torch.device("cuda:0")
    g, kc, vc, indptr, indices, lens = _setup("NHD", 13)
    k = torch.randn((2, 4, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((2, 4, 128), generator=g).to(torch.bfloat16)
    bidx = torch.tensor([0, 1], dtype=torch.int32)
    pos = torch.tensor([48, 5], dtype=torch.int32)  # request 0 owns 3 pages (48 slots): position 48 is past them
    ref_k, ref_v = _ref_scatter(kc, vc, k[1:], v[1:], bidx[1:], pos[1:], indptr, indices, "NHD", 16)
    kd, vd = kc.to(dev), vc.to(dev)
    atflash.append_paged_kv_cache(k.to(dev), v.to(dev), bidx.to(dev), pos.to(dev), (kd, vd), indices.to(dev),
                                  indptr.to(dev))
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 2
    assert torch.equal(kd.cpu(), ref_k) and torch.equal(vd.cpu(), ref_v)


def test_decode_over_appended_cache():
    """Prefill-to-decode handoff: K appended with RoPE at write (sorted pairs)
    gives the same windowed decode as the cache written by the RoPE pack."""
    import atflash
    dev = torch.device("cuda:0")
    g, kc, vc, indptr, indices, lens = _setup("NHD", 14, lens=(300, 129))
    nnz = sum(lens)
    bidx, pos = atflash.get_batch_indices_positions(torch.tensor([0, 300, 429]), torch.tensor(lens), nnz)
    k = torch.randn((nnz, 4, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((nnz, 4, 128), generator=g).to(torch.bfloat16)
    q = torch.randn((2, 12, 128), generator=g).to(torch.bfloat16)
    cos, sin = rope_tables(400, 128, 1e4)
    cosd, sind = cos.to(dev), sin.to(dev)
    ka, va = kc.to(dev), vc.to(dev)
    atflash.append_paged_kv_cache(k.to(dev), v.to(dev), bidx.to(dev), pos.to(dev), (ka, va), indices.to(dev),
                                  indptr.to(dev), rope=(cosd, sind), out_layout="sorted_pair")
    kr = atflash.rope_pack(k.to(dev)[None], cosd, sind, positions=pos.to(dev).long(), out_layout="sorted_pair")[0]
    rk, rv = _ref_scatter(kc, vc, kr.cpu(), v, bidx, pos, indptr, indices, "NHD", 16)
    # the two queries as one 2-token sequence: query b at position lens[b]-1
    qr = atflash.rope_pack(q.to(dev)[None], cosd, sind, positions=torch.tensor([299, 128], device=dev),
                           out_layout="sorted_pair")[0]
    lpl = torch.tensor([(n - 1) % 16 + 1 for n in lens], dtype=torch.int32)
    outs = []
    for (kk, vv) in ((ka, va), (rk.to(dev), rv.to(dev))):
        ws = torch.empty(32 << 20, dtype=torch.uint8, device=dev)
        w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD")
        w.plan(indptr, indices, lpl, 12, 4, 128, 16, window_table=atflash.WindowTable(128, 1e4, 2.0))
        outs.append(w.run(qr.contiguous(), (kk, vv)))
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("rope", [False, True])
def test_append_into_level_major_k_pages(rope):
    """Appending into level-major K pages writes the same values as appending
    into NHD pages and laying them out level-major."""
    import atflash
    dev = torch.device("cuda:0")
    g, kc, vc, indptr, indices, lens = _setup("NHD", 15)
    nnz = sum(lens)
    bidx, pos = atflash.get_batch_indices_positions(torch.tensor([0, 37, 117, 122]), torch.tensor(lens), nnz)
    k = torch.randn((nnz, 4, 128), generator=g).to(torch.bfloat16)
    v = torch.randn((nnz, 4, 128), generator=g).to(torch.bfloat16)
    kw = {}
    if rope:
        cos, sin = rope_tables(200, 128, 1e4)
        kw = dict(rope=(cos.to(dev), sin.to(dev)), out_layout="sorted_pair")
    P, page, hkv, _ = kc.shape
    k_nhd, v_nhd = kc.to(dev), vc.to(dev)
    k_lm = kc.view(P, page, hkv, 8, 16).permute(0, 2, 3, 1, 4).contiguous().to(dev)
    v_lm = vc.to(dev)
    args = (k.to(dev), v.to(dev), bidx.to(dev), pos.to(dev))
    atflash.append_paged_kv_cache(*args, (k_nhd, v_nhd), indices.to(dev), indptr.to(dev), **kw)
    atflash.append_paged_kv_cache(*args, (k_lm, v_lm), indices.to(dev), indptr.to(dev), **kw)
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    expect = k_nhd.view(P, page, hkv, 8, 16).permute(0, 2, 3, 1, 4)
    assert torch.equal(k_lm, expect) and torch.equal(v_lm, v_nhd)
