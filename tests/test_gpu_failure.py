"""Failure detection on a B200 without a GPU fault.

Every device-side wait of the library is bounded: a kernel waits on an mbarrier
that nothing arrives on, gives up after the limit (2 s), reports through the
error flag and returns, and the context stays usable for the next launch. A
prefill that finds the error flag already set returns at once without
computing; the host reads the flag."""
import math
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    import atflash
    from atflash import _runtime
    dev = torch.device("cuda:0")
    assert atflash.check_device_errors(dev) == 0
    t0 = time.time()
    flag = _runtime.selftest_wait_timeout(dev)
    dt = time.time() - t0
    assert flag == 1, flag
    assert 1.5 < dt < 30, dt
    # the context is still usable and the flag was cleared
    x = torch.randn((1, 256, 2, 128), device=dev).to(torch.bfloat16)
    cos, sin = atflash.cos_sin_table(256, 128, 1e4, device=dev)
    y = atflash.rope_pack(x, cos, sin)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    assert atflash.check_device_errors(dev) == 0


def test_prefill_returns_early_when_the_error_flag_is_set():
    import atflash
    from atflash import _runtime
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(3)
    q = torch.randn((1, 512, 4, 128), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((1, 512, 2, 128), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((1, 512, 2, 128), generator=g, device=dev).to(torch.bfloat16)
    out = torch.full_like(q, float("nan"))
    _runtime.error_flag(dev).fill_(7)  # as if an earlier launch had failed
    atflash.prefill_fwd(q, k, v, out=out)
    assert atflash.check_device_errors(dev) == 7
    assert torch.isnan(out.float()).all()  # nothing was computed
    atflash.prefill_fwd(q, k, v, out=out)  # flag cleared: runs normally
    assert atflash.check_device_errors(dev) == 0
    assert torch.isfinite(out.float()).all()
