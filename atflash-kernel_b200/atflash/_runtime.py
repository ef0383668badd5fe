"""Per-device runtime state of the Python layer: the device error flag that the
kernels' bounded waits report into, and the current stream handle."""
import ctypes
import threading

import torch

from . import _ffi

_flags = {}
_lock = threading.Lock()


def error_flag(device: torch.device) -> torch.Tensor:
    """int32[1] on `device`, zero-initialised once per device."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _lock:
        t = _flags.get(idx)
        if t is None:
            t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            _flags[idx] = t
    return t


def check_device_errors(device=None) -> int:
    """Synchronise `device`, return (and clear) its kernel error flag.

    Non-zero means a bounded device wait expired and a kernel returned early;
    its outputs are not valid."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    flag = error_flag(dev)
    out = ctypes.c_int(0)
    with torch.cuda.device(dev):
        _ffi.check("atf_read_error_flag", _ffi.load().atf_read_error_flag(flag.data_ptr(), ctypes.byref(out)))
    return out.value


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("atflash kernels take CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


def selftest_wait_timeout(device=None) -> int:
    """Run the bounded-wait self-test on `device` (about 2 s): a kernel waits on
    a barrier nothing arrives on, gives up after the wait limit and reports
    through the error flag. Returns the flag value (1 = wait timed out)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    flag = error_flag(dev)
    with torch.cuda.device(dev):
        _ffi.check("atf_selftest_wait_timeout",
                   _ffi.load().atf_selftest_wait_timeout(flag.data_ptr(), stream_handle(dev)))
    return check_device_errors(dev)
