"""CPU checks of the C ABI library: it loads, exports every function
include/atflash_b200.h declares, rejects bad arguments before touching a GPU,
and its host-side split-KV planner covers every key exactly once."""
import ctypes
import os
import re

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
HEADER = os.path.join(ROOT, "include", "atflash_b200.h")


def _lib():
    from atflash import _ffi
    try:
        return _ffi.load()
    except (ImportError, OSError) as e:
        pytest.skip(f"library not built: {e}")


def declared_functions():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:int64_t|int|const char\*)\s+(atf_\w+)\(", txt, flags=re.M)))


def test_header_declares_the_abi():
    names = declared_functions()
    for n in ("atf_prefill_fwd", "atf_decode_plan", "atf_decode_run", "atf_lse_merge",
              "atf_status_string", "atf_rope_pack", "atf_window_zhi16"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib()
    for name in declared_functions():
        assert hasattr(lib, name), name
    from atflash import _ffi
    assert set(_ffi.EXPORTED) >= set(declared_functions())


def test_params_struct_sizes_match_the_mirrors():
    """Every params struct of the header has the size of its ctypes mirror, so a
    field appended on one side only is caught on the CPU."""
    from atflash import _ffi
    lib = _lib()
    names = re.findall(r"^\}\s+(Atf\w+);", open(HEADER).read(), flags=re.M)
    assert "AtfMergeParams" in names and "AtfDecodeParams" in names
    for n in names:
        assert lib.atf_params_size(n.encode()) == ctypes.sizeof(getattr(_ffi, n)), n
    assert lib.atf_params_size(b"NoSuchStruct") == -1


def test_status_strings():
    from atflash import _ffi
    _lib()
    assert _ffi.status_string(0) == "ok"
    assert "argument" in _ffi.status_string(-1)
    assert _ffi.status_string(-99) == "unknown status"


def test_invalid_arguments_rejected_without_gpu():
    from atflash import _ffi
    lib = _lib()
    assert lib.atf_prefill_fwd(None, None) == -1
    p = _ffi.AtfPrefillParams()
    assert lib.atf_prefill_fwd(ctypes.byref(p), None) == -1  # null tensors
    p.q = p.k = p.v = p.out = 16
    p.head_dim = 64
    assert lib.atf_prefill_fwd(ctypes.byref(p), None) == -2  # head_dim 64 unsupported
    p.head_dim = 128
    p.batch = p.seqlen_q = p.seqlen_k = 1
    p.num_heads_q, p.num_heads_kv = 6, 4
    assert lib.atf_prefill_fwd(ctypes.byref(p), None) == -1  # heads not a multiple
    p.num_heads_kv = 2
    p.softmax_scale = 0.1
    p.q = 17
    assert lib.atf_prefill_fwd(ctypes.byref(p), None) == -3  # misaligned
    p.q = 16
    p.window = _ffi.ATF_WINDOW_SNAP16
    for i, z in enumerate((100, 50, 60, 10, 0, 0, 0, 0)):
        p.zhi[i] = z
    assert lib.atf_prefill_fwd(ctypes.byref(p), None) == -1  # levels must not widen
    p.window = _ffi.ATF_WINDOW_OFF
    p.seqlen_q = p.seqlen_k = 1024
    for ranges in (((64, 256),), ((0, 256), (128, 512)), ((256, 128),), ((0, 1100),), ((0, 128),) * 3):
        p.num_row_ranges = len(ranges)
        for i, (b, e) in enumerate(ranges[:2]):
            p.row_begin[i], p.row_end[i] = b, e
        # unaligned begin, overlapping, empty, past the rows, more than two ranges
        assert lib.atf_prefill_fwd(ctypes.byref(p), None) == -1, ranges
    p.num_row_ranges = 0
    d = _ffi.AtfDecodeParams()
    d.q = d.k_cache = d.v_cache = d.indptr = d.indices = d.last_page_len = 16
    d.items = d.item_indptr = d.partial_o = d.partial_lse = d.out = 16
    d.head_dim, d.batch_size, d.num_qo_heads, d.num_kv_heads, d.page_size = 128, 1, 8, 8, 16
    d.window = _ffi.ATF_WINDOW_SNAP16
    for i, z in enumerate((100, 50, 60, 10, 0, 0, 0, 0)):
        d.zhi16[i] = z
    assert lib.atf_decode_run(ctypes.byref(d), None) == -1
    assert lib.atf_decode_run(None, None) == -1
    assert lib.atf_lse_merge(None, None) == -1
    assert lib.atf_rope_pack(None, None) == -1
    r = _ffi.AtfRopeParams()
    r.x, r.out, r.cos, r.sin = 16, 16, 32, 48
    r.head_dim, r.n_pos, r.cs_stride_pos = 128, 1, 64
    assert lib.atf_rope_pack(ctypes.byref(r), None) == -1  # in place
    assert lib.atf_state_push(None, None) == -1
    assert lib.atf_state_merge(None, None) == -1
    assert lib.atf_decode_run_exchange(None, None, None) == -1
    x = _ffi.AtfExchangeParams()
    x.o = x.lse = x.peer_base = x.base = 256
    x.batch, x.num_heads, x.world, x.rank = 1, 28, 2, 2  # rank outside the group
    assert lib.atf_state_push(ctypes.byref(x), None) == -1
    x.rank = 1
    x.base = 272  # the region must be 256-byte aligned
    assert lib.atf_state_push(ctypes.byref(x), None) == -3
    # region: 2 parities x world x (B*H*128 + round4(B*H)) floats, flags, step, tickets
    S = 28 * 128 + 28
    assert lib.atf_exchange_region_bytes(1, 28, 8) == ((2 * 8 * S * 4 + 8 * 8 + 8 + 8) + 255) // 256 * 256
    assert lib.atf_exchange_region_bytes(0, 28, 8) == -1
    # the fused decode step: the exchange must match the decode's batch and heads
    d = _ffi.AtfDecodeParams()
    d.q = d.k_cache = d.v_cache = d.indptr = d.indices = d.last_page_len = 256
    d.items = d.item_indptr = d.partial_o = d.partial_lse = d.out = 256
    d.head_dim, d.batch_size, d.num_qo_heads, d.num_kv_heads, d.page_size = 128, 1, 28, 4, 16
    x.base = 256
    x.num_heads = 24
    assert lib.atf_decode_run_exchange(ctypes.byref(d), ctypes.byref(x), None) == -1
    x.num_heads = 28
    x.base = 272
    assert lib.atf_decode_run_exchange(ctypes.byref(d), ctypes.byref(x), None) == -3


def test_decode_run_rejects_misaligned_workspace_and_output():
    """The split kernel stores float4 rows into partial_o and the merge stores
    4 values per lane into out; misaligned buffers or output strides are
    refused before any launch."""
    from atflash import _ffi
    lib = _lib()

    def params():
        d = _ffi.AtfDecodeParams()
        d.q = d.k_cache = d.v_cache = d.indptr = d.indices = d.last_page_len = 256
        d.items = d.item_indptr = d.partial_o = d.partial_lse = d.out = 256
        d.head_dim, d.batch_size, d.num_qo_heads, d.num_kv_heads, d.page_size = 128, 1, 8, 8, 16
        d.kv_stride_page, d.kv_stride_token, d.kv_stride_head = 16 * 8 * 128, 8 * 128, 128
        d.q_stride_b, d.q_stride_h = 8 * 128, 128
        d.o_stride_b, d.o_stride_h = 8 * 128, 128
        d.num_pages = 1
        return d

    for field, value in (("partial_o", 264), ("partial_lse", 258), ("out", 260), ("o_stride_b", 1026),
                         ("o_stride_h", 130)):
        d = params()
        setattr(d, field, value)
        assert lib.atf_decode_run(ctypes.byref(d), None) == -3, field
    d = params()
    d.out_dtype = _ffi.ATF_DTYPE_F32
    d.out = 264  # 8-byte aligned is enough for bf16, not for fp32
    assert lib.atf_decode_run(ctypes.byref(d), None) == -3


def _plan(lib, lens, page, hq=24, hkv=8, **kw):
    from atflash import _ffi
    npages = [(n + page - 1) // page for n in lens]
    indptr = np.concatenate([[0], np.cumsum(npages)]).astype(np.int32)
    lpl = np.array([((n - 1) % page) + 1 for n in lens], dtype=np.int32)
    pp = _ffi.AtfDecodePlanParams()
    pp.batch_size, pp.num_qo_heads, pp.num_kv_heads, pp.head_dim, pp.page_size = len(lens), hq, hkv, 128, page
    pp.indptr_host, pp.last_page_len_host = indptr.ctypes.data, lpl.ctypes.data
    pp.num_sms = kw.get("sms", 148)
    pp.max_chunk_keys = kw.get("max_chunk", 0)
    zhi = kw.get("zhi")
    if zhi is not None:
        pp.window = _ffi.ATF_WINDOW_SNAP16
        for i in range(8):
            pp.zhi16[i] = zhi[i]
    plan = _ffi.AtfDecodePlan()
    assert lib.atf_decode_plan(ctypes.byref(pp), None, 0, None, ctypes.byref(plan)) == 0
    items = np.zeros((max(1, plan.num_items), 4), dtype=np.int32)
    iptr = np.zeros(len(lens) + 1, dtype=np.int32)
    P32 = ctypes.POINTER(ctypes.c_int32)
    assert lib.atf_decode_plan(ctypes.byref(pp), items.ctypes.data_as(P32), items.shape[0],
                               iptr.ctypes.data_as(P32), ctypes.byref(plan)) == 0
    return plan, items[:plan.num_items], iptr


_ZHI_K2 = (2147483647, 992572, 192482, 37326, 7238, 1403, 272, 52)  # theta 5e5, k = 2


@pytest.mark.parametrize("zhi", [None, _ZHI_K2])
@pytest.mark.parametrize("lens,page", [([131072] * 8, 16), ([8192, 1, 70000], 16), ([1048576], 64), ([5], 1),
                                       ([0, 300, 0], 16)])
def test_decode_plan_covers_every_key_once(lens, page, zhi):
    lib = _lib()
    plan, items, iptr = _plan(lib, lens, page, zhi=zhi)
    assert plan.chunk_keys == max([int(k1 - k0) for (_, k0, k1, _) in items] + [0])
    for b, n in enumerate(lens):
        its = items[iptr[b]:iptr[b + 1]]
        assert its[:, 0].tolist() == [b] * len(its)
        cover = np.zeros(n, dtype=np.int32)
        for (_, k0, k1, _) in its:
            assert k0 % 64 == 0 and 0 < k1 - k0 <= 16384
            cover[k0:k1] += 1
        assert (cover == 1).all()
    assert plan.partial_o_floats == plan.num_items * 24 * 128


def _item_bytes(items, lens, zhi):
    """Bytes one kv head's CTA reads for each item: V rows plus the in-window
    K levels of every key (a key at distance z reads max(1, #{zhi[i] >= z}))."""
    out = []
    for (b, k0, k1, _) in items:
        z = lens[b] - 1 - np.arange(k0, k1)
        levels = np.maximum(1, (np.asarray(zhi)[None, :] >= z[:, None]).sum(1))
        out.append(int((256 + 32 * levels).sum()))
    return np.array(out)


@pytest.mark.parametrize("lens,page,hkv", [([131072] * 8, 16, 8), ([1048576], 64, 4), ([200000, 9000], 16, 8)])
def test_decode_plan_balances_window_bytes(lens, page, hkv):
    """Under a snap16 window the items of a request carry equal bytes (to a
    64-key stage), not equal key counts: far keys read fewer K levels, so the
    items far from the query are longer."""
    lib = _lib()
    _, items, iptr = _plan(lib, lens, page, hkv=hkv, zhi=_ZHI_K2)
    for b in range(len(lens)):
        its = items[iptr[b]:iptr[b + 1]]
        if len(its) < 2:
            continue
        c = _item_bytes(its, lens, _ZHI_K2)
        # each cut falls on a stage boundary: within two stages of the densest keys
        assert c.max() - c.min() <= 2 * 64 * 512
        keys = its[:, 2] - its[:, 1]
        assert keys[0] >= keys[-1]  # the oldest keys are the cheapest
    _, even, _ = _plan(lib, lens, page, hkv=hkv)
    # the same number of CTAs as the unwindowed plan
    assert len(items) == len(even)


def test_decode_plan_rejects_bad_tables():
    from atflash import _ffi
    lib = _lib()
    indptr = np.array([0, 2], dtype=np.int32)
    lpl = np.array([17], dtype=np.int32)  # > page size
    pp = _ffi.AtfDecodePlanParams()
    pp.batch_size, pp.num_qo_heads, pp.num_kv_heads, pp.head_dim, pp.page_size = 1, 8, 8, 128, 16
    pp.indptr_host, pp.last_page_len_host = indptr.ctypes.data, lpl.ctypes.data
    plan = _ffi.AtfDecodePlan()
    assert lib.atf_decode_plan(ctypes.byref(pp), None, 0, None, ctypes.byref(plan)) == -1
    pp.num_qo_heads = 8 * 17  # group of 17 > 16
    lpl[0] = 3
    assert lib.atf_decode_plan(ctypes.byref(pp), None, 0, None, ctypes.byref(plan)) == -2


def test_append_rejects_bad_arguments_without_gpu():
    from atflash import _ffi
    lib = _lib()
    assert lib.atf_paged_kv_append(None, None) == -1
    p = _ffi.AtfAppendParams()
    assert lib.atf_paged_kv_append(ctypes.byref(p), None) == -1  # null tensors
    p.append_k = p.append_v = p.batch_indices = p.positions = 256
    p.k_cache = p.v_cache = p.kv_indptr = p.kv_indices = 256
    p.head_dim, p.num_kv_heads, p.page_size, p.batch_size, p.num_pages = 64, 1, 16, 1, 1
    assert lib.atf_paged_kv_append(ctypes.byref(p), None) == -2  # head_dim 64
    p.head_dim = 128
    p.cos = 256  # cos without sin
    assert lib.atf_paged_kv_append(ctypes.byref(p), None) == -1
    p.cos = None
    p.a_stride_n = 3  # misaligned token stride
    assert lib.atf_paged_kv_append(ctypes.byref(p), None) == -3


def test_fa4_entry_rejects_unsupported_options_before_any_launch():
    """The FA4-shaped entry accepts the reference's own arguments and FA4's tuning
    hints, but refuses options it cannot honour instead of dropping them."""
    import torch
    import atflash
    q = torch.zeros((1, 4, 2, 128), dtype=torch.bfloat16)
    for name, value in (("softcap", 30.0), ("window_size_left", 128), ("cu_seqlens_q", q),
                        ("page_table", q)):
        with pytest.raises(NotImplementedError, match=name):
            atflash._flash_attn_fwd(q, q, q, causal=True, **{name: value})
    # defaults and tuning hints pass the check and reach the device check (no GPU here)
    if not torch.cuda.is_available():
        with pytest.raises(Exception) as e:
            atflash._flash_attn_fwd(q, q, q, causal=True, pack_gqa=True, softcap=None,
                                    m_block_size=128, num_threads=384)
        assert not isinstance(e.value, NotImplementedError)
