"""RoPE tables and the fused RoPE + pair-order pack kernel.

Table construction follows the reference's RoPE front-end
(microbench/b1_correctness.py:113-123): inv_freq = 1 / base^(arange(0, d, 2)/d)
in fp32, angle t = float(pos) * inv_freq in fp32, cos/sin in fp32.
"""
import ctypes
from typing import Optional

import torch

from . import _ffi, _runtime

_LAYOUTS = {"sorted_pair": _ffi.ATF_LAYOUT_SORTED_PAIR, "rotate_half": _ffi.ATF_LAYOUT_ROTATE_HALF}


def inv_freq(head_dim: int, rope_base: float, device="cpu") -> torch.Tensor:
    return 1.0 / (rope_base ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))


def cos_sin_table(n_pos: int, head_dim: int, rope_base: float, device="cpu", positions=None):
    """fp32 (cos, sin) of shape (n_pos, head_dim/2) at positions 0..n_pos-1."""
    invf = inv_freq(head_dim, rope_base, device)
    pos = torch.arange(n_pos, device=device) if positions is None else positions.to(device)
    t = pos.float()[:, None] * invf[None, :]
    return torch.cos(t), torch.sin(t)


def rope_pack(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *, pos_offset: int = 0,
              positions: Optional[torch.Tensor] = None, out_layout: str = "rotate_half",
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rotate pre-RoPE x (B, S, H, 128) bf16 in rotate_half order; write bf16 in
    `out_layout` order ("rotate_half" or "sorted_pair"). Token s sits at
    position positions[s] (or pos_offset + s)."""
    dev = _runtime.require_cuda(x, cos, sin)
    if x.dim() != 4 or x.shape[-1] != 128 or x.dtype != torch.bfloat16 or x.stride(-1) != 1:
        raise ValueError("x must be (B, S, H, 128) bf16 with a contiguous last axis")
    if cos.dtype != torch.float32 or sin.dtype != torch.float32 or cos.shape != sin.shape:
        raise ValueError("cos/sin must be matching fp32 tables (n_pos, 64)")
    if cos.dim() != 2 or cos.shape[1] < 64 or cos.stride(1) != 1 or cos.stride() != sin.stride():
        raise ValueError("cos/sin must be (n_pos, >=64) with a contiguous last axis")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=dev)
    p = _ffi.AtfRopeParams()
    p.x, p.out = x.data_ptr(), out.data_ptr()
    p.batch, p.seqlen, p.num_heads, p.head_dim = x.shape
    p.x_stride_b, p.x_stride_s, p.x_stride_h = x.stride(0), x.stride(1), x.stride(2)
    p.o_stride_b, p.o_stride_s, p.o_stride_h = out.stride(0), out.stride(1), out.stride(2)
    p.cos, p.sin = cos.data_ptr(), sin.data_ptr()
    p.cs_stride_pos = cos.stride(0)
    p.n_pos = cos.shape[0]
    if positions is not None:
        positions = positions.to(device=dev, dtype=torch.int64).contiguous()
        p.positions = positions.data_ptr()
    p.pos_offset = int(pos_offset)
    p.out_layout = _LAYOUTS[out_layout]
    with torch.cuda.device(dev):
        rc = _ffi.load().atf_rope_pack(ctypes.byref(p), _runtime.stream_handle(dev))
    _ffi.check("atf_rope_pack", rc)
    return out
