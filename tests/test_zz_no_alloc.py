"""atf_decode_run_noalloc: the paged decode with its split workspace in the
library's fixed scratch array instead of caller memory.

Named to be collected last, so that it runs both on its own in a fresh process
and after every other test has used the allocating entry point. On the GPU, two
calls in a row, on different inputs, must each equal atf_decode_run on the same
inputs bit for bit (both take the same kernels; only the workspace address
differs). On the CPU, the size and argument checks answer before any device
call."""
import ctypes

import pytest
import torch

from atflash import _ffi


def _lib():
    try:
        return _ffi.load()
    except (ImportError, OSError) as e:
        pytest.skip(f"library not built: {e}")


def test_rejects_plans_beyond_the_scratch_without_a_device():
    lib = _lib()
    p = _ffi.AtfDecodeParams()
    p.num_qo_heads = 32
    p.num_items = _ffi.ATF_NOALLOC_MAX_PARTIAL_ROWS // 32 + 1
    rc = lib.atf_decode_run_noalloc(ctypes.byref(p), None)
    assert rc == -5, _ffi.status_string(rc)
    assert "workspace" in _ffi.status_string(rc)


def test_rejects_a_caller_workspace():
    lib = _lib()
    p = _ffi.AtfDecodeParams()
    p.num_qo_heads, p.num_items = 8, 1
    p.partial_o = 256
    assert lib.atf_decode_run_noalloc(ctypes.byref(p), None) == -1
    p.partial_o = None
    p.partial_lse = 256
    assert lib.atf_decode_run_noalloc(ctypes.byref(p), None) == -1
    assert lib.atf_decode_run_noalloc(None, None) == -1


def _decode_with_params(dev, case, seed, window_table):
    """Runs the allocating wrapper and returns (out, lse, params it passed)."""
    import atflash
    from test_gpu_decode import make_paged
    kv_lens, hq, hkv, page, layout = case
    q, kc, vc, indptr, indices, lpl, _, _ = make_paged(kv_lens, hq, hkv, page, seed, layout)
    ws = torch.empty(64 * 1024 * 1024, dtype=torch.uint8, device=dev)
    w = atflash.BatchDecodeWithPagedKVCacheWrapper(ws, kv_layout=layout)
    w.plan(indptr, indices, lpl, hq, hkv, 128, page, window_table=window_table)
    lib = _ffi.load()
    real = lib.atf_decode_run
    seen = {}

    def spy(pp, stream):
        seen["p"] = _ffi.AtfDecodeParams.from_buffer_copy(pp._obj)
        return real(pp, stream)

    lib.atf_decode_run = spy
    try:
        tensors = (q.to(dev), kc.to(dev), vc.to(dev))
        out, lse = w.run(tensors[0], tensors[1:], return_lse=True)
    finally:
        lib.atf_decode_run = real
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    # keep the plan's device tables and the inputs alive with the params
    return out, lse, seen["p"], (w, tensors, ws)


@pytest.mark.gpu
def test_noalloc_equals_allocating_decode_on_two_calls_in_a_row():
    import atflash
    from atflash import _runtime
    dev = torch.device("cuda:0")
    wt = atflash.WindowTable(128, 1e4, 2.0)
    cases = [([3000, 517, 64], 32, 8, 16, "NHD"), ([2049, 4100], 28, 4, 64, "HND")]
    runs = [_decode_with_params(dev, c, 100 + i, wt) for i, c in enumerate(cases)]
    lib = _ffi.load()
    results = []
    for out_ref, lse_ref, p, _keep in runs:  # two calls back to back, nothing in between
        out = torch.full_like(out_ref, float("nan"))
        lse = torch.full_like(lse_ref, float("nan"))
        p.partial_o = None
        p.partial_lse = None
        p.out = out.data_ptr()
        p.lse_out = lse.data_ptr()
        with torch.cuda.device(dev):
            rc = lib.atf_decode_run_noalloc(ctypes.byref(p), _runtime.stream_handle(dev))
        _ffi.check("atf_decode_run_noalloc", rc)
        results.append((out, lse))
    torch.cuda.synchronize()
    assert atflash.check_device_errors() == 0
    for (out_ref, lse_ref, _, _), (out, lse) in zip(runs, results):
        assert torch.equal(out, out_ref)
        assert torch.equal(lse, lse_ref)


@pytest.mark.gpu
def test_noalloc_fills_the_whole_scratch():
    """A plan that uses every one of the ATF_NOALLOC_MAX_PARTIAL_ROWS rows (512
    one-item requests x 32 heads): the last row lands at the end of the scratch
    and the output still equals atf_decode_run bit for bit, on two calls."""
    import atflash
    from atflash import _runtime
    dev = torch.device("cuda:0")
    case = ([64 + (i % 7) for i in range(512)], 32, 8, 16, "NHD")
    out_ref, lse_ref, p, _keep = _decode_with_params(dev, case, 11, atflash.WindowTable(128, 1e4, 2.0))
    assert p.num_items * p.num_qo_heads == _ffi.ATF_NOALLOC_MAX_PARTIAL_ROWS
    lib = _ffi.load()
    p.partial_o = None
    p.partial_lse = None
    for _ in range(2):
        out = torch.full_like(out_ref, float("nan"))
        lse = torch.full_like(lse_ref, float("nan"))
        p.out = out.data_ptr()
        p.lse_out = lse.data_ptr()
        with torch.cuda.device(dev):
            rc = lib.atf_decode_run_noalloc(ctypes.byref(p), _runtime.stream_handle(dev))
        _ffi.check("atf_decode_run_noalloc", rc)
        torch.cuda.synchronize()
        assert atflash.check_device_errors() == 0
        assert torch.equal(out, out_ref)
        assert torch.equal(lse, lse_ref)


@pytest.mark.gpu
def test_noalloc_rejects_an_oversized_plan_on_the_device():
    import atflash
    dev = torch.device("cuda:0")
    case = ([64] * 600, 32, 8, 16, "NHD")  # 600 items x 32 heads > 16384 rows
    out_ref, lse_ref, p, _keep = _decode_with_params(dev, case, 7, atflash.WindowTable(128, 1e4, 2.0))
    assert p.num_items * p.num_qo_heads > _ffi.ATF_NOALLOC_MAX_PARTIAL_ROWS
    p.partial_o = None
    p.partial_lse = None
    assert _ffi.load().atf_decode_run_noalloc(ctypes.byref(p), None) == -5
