"""Windowed prefill shaped like ``flash_attn_func``.

The reference calls its windowed FA4 forward as
``_flash_attn_fwd(q, k, v, causal=True, pack_gqa=..., atflash_window_zhi=zhi)``
with BSHD tensors (e2e_pipeline/atflash_e2e_fafi.py:113-119,
microbench/b1_correctness.py:84-85); both that spelling and the public
``flash_attn_func`` signature are provided here, plus ``window_table``.
"""
import ctypes
import math
from typing import Optional, Sequence, Tuple, Union

import torch

from . import _ffi, _runtime
from .rope import rope_pack
from .window_table import KERNEL_CAP, WindowTable

WindowSpec = Union[None, WindowTable, Sequence[int]]
_LAYOUTS = {"sorted_pair": _ffi.ATF_LAYOUT_SORTED_PAIR, "rotate_half": _ffi.ATF_LAYOUT_ROTATE_HALF}


def resolve_zhi(window_table: WindowSpec, head_dim: int, max_distance: int) -> Optional[Tuple[int, ...]]:
    """Window spec -> 16-snap zhi levels for the kernel, or None for dense."""
    if window_table is None:
        return None
    if isinstance(window_table, WindowTable):
        if window_table.head_dim != head_dim:
            raise ValueError("window table head_dim does not match the tensors")
        return tuple(window_table.zhi16)
    zhi = tuple(int(x) for x in window_table)
    if len(zhi) != head_dim // 16:
        raise ValueError(f"a zhi level table has head_dim/16 = {head_dim // 16} entries")
    if any(zhi[i] < zhi[i + 1] for i in range(len(zhi) - 1)):
        raise ValueError("zhi levels must be non-increasing")
    if zhi[0] < max_distance:
        # zhi[0] is the cap of the table; every distance must be covered by level 0
        zhi = (max(zhi[0], min(KERNEL_CAP, max_distance)),) + zhi[1:]
    return zhi


def _check_qkv(q, k, v):
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, v must be (batch, seqlen, heads, head_dim)")
    for t in (q, k, v):
        if t.dtype != torch.bfloat16:
            raise TypeError("q, k, v must be bfloat16")
        if t.stride(-1) != 1:
            raise ValueError("the head_dim axis must be contiguous")
    if q.shape[0] != k.shape[0] or k.shape != v.shape or q.shape[-1] != k.shape[-1]:
        raise ValueError("shape mismatch between q, k and v")
    if q.shape[2] % k.shape[2] != 0:
        raise ValueError("num_heads_q must be a multiple of num_heads_kv")


def prefill_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = True,
                softmax_scale: Optional[float] = None, window_table: WindowSpec = None,
                qk_layout: str = "sorted_pair", q_offset: Optional[int] = None,
                out: Optional[torch.Tensor] = None, return_lse: bool = False,
                q_rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                row_ranges: Optional[Sequence[Tuple[int, int]]] = None):
    """Run the tcgen05 windowed prefill kernel. q (B, Sq, Hq, 128), k/v (B, Sk, Hkv, 128).

    q_rope: optional fp32 (cos, sin) tables (n_pos, >= 64): q is then pre-RoPE in
    rotate_half order and the kernel rotates each query row at position
    q_offset + row as it loads it (k must be post-RoPE, sorted pairs).
    row_ranges: up to two sorted, disjoint [begin, end) ranges of query rows,
    begins on multiples of 128: only those rows of out are computed, in one
    launch (the rows are bit-identical to a run over all rows)."""
    _check_qkv(q, k, v)
    dev = _runtime.require_cuda(q, k, v)
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    if q_offset is None:
        q_offset = Sk - Sq
    if causal and q_offset < 0:
        raise ValueError("causal prefill needs seqlen_q <= seqlen_k (bottom-right alignment)")
    if qk_layout not in _LAYOUTS:
        raise ValueError(f"qk_layout must be one of {sorted(_LAYOUTS)}")
    zhi = resolve_zhi(window_table, D, q_offset + Sq)
    if out is None:
        out = torch.empty((B, Sq, Hq, D), dtype=torch.bfloat16, device=dev)
    elif (tuple(out.shape) != (B, Sq, Hq, D) or out.dtype != torch.bfloat16 or out.device != q.device
          or out.stride(-1) != 1):
        raise ValueError(f"out must be a bf16 ({B}, {Sq}, {Hq}, {D}) tensor on {q.device} "
                         "with a contiguous head_dim axis")
    lse = torch.empty((B, Hq, Sq), dtype=torch.float32, device=dev) if return_lse else None
    p = _ffi.AtfPrefillParams()
    p.q, p.k, p.v, p.out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.lse = lse.data_ptr() if lse is not None else None
    p.batch, p.seqlen_q, p.seqlen_k, p.num_heads_q, p.num_heads_kv, p.head_dim = B, Sq, Sk, Hq, Hkv, D
    p.q_stride_b, p.q_stride_s, p.q_stride_h = q.stride(0), q.stride(1), q.stride(2)
    p.k_stride_b, p.k_stride_s, p.k_stride_h = k.stride(0), k.stride(1), k.stride(2)
    p.v_stride_b, p.v_stride_s, p.v_stride_h = v.stride(0), v.stride(1), v.stride(2)
    p.o_stride_b, p.o_stride_s, p.o_stride_h = out.stride(0), out.stride(1), out.stride(2)
    p.q_offset = int(q_offset)
    p.softmax_scale = float(softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D))
    p.causal = 1 if causal else 0
    p.qk_layout = _LAYOUTS[qk_layout]
    p.window = _ffi.ATF_WINDOW_SNAP16 if zhi is not None else _ffi.ATF_WINDOW_OFF
    if zhi is not None:
        for i, z in enumerate(zhi):
            p.zhi[i] = z
    p.error_flag = _runtime.error_flag(dev).data_ptr()
    if row_ranges is not None:
        rr = [(int(b), int(e)) for (b, e) in row_ranges]
        if not 1 <= len(rr) <= 2:
            raise ValueError("row_ranges holds one or two ranges")
        for i, (b, e) in enumerate(rr):
            if b < 0 or e <= b or e > Sq or b % 128 or (i and b < rr[i - 1][1]):
                raise ValueError("row ranges must be sorted, disjoint, non-empty, inside the rows and "
                                 "begin on multiples of 128")
            p.row_begin[i], p.row_end[i] = b, e
        p.num_row_ranges = len(rr)
    if q_rope is not None:
        cos, sin = q_rope
        if qk_layout != "sorted_pair":
            raise ValueError("RoPE at load needs k in sorted-pair order")
        if (cos.dtype != torch.float32 or sin.dtype != torch.float32 or cos.shape != sin.shape or cos.dim() != 2
                or cos.shape[1] < 64 or cos.stride(1) != 1 or cos.stride() != sin.stride() or not cos.is_cuda
                or cos.device != dev or sin.device != dev):
            raise ValueError("q_rope must be matching fp32 (n_pos, >=64) tables on the tensors' device")
        if cos.shape[0] < q_offset + Sq:
            raise ValueError(f"the RoPE tables cover {cos.shape[0]} positions, the queries need {q_offset + Sq}")
        p.q_cos, p.q_sin = cos.data_ptr(), sin.data_ptr()
        p.q_cs_stride_pos, p.q_n_pos = cos.stride(0), cos.shape[0]
    with torch.cuda.device(dev):
        rc = _ffi.load().atf_prefill_fwd(ctypes.byref(p), _runtime.stream_handle(dev))
    _ffi.check("atf_prefill_fwd", rc)
    return (out, lse) if return_lse else out


def flash_attn_func(q, k, v, dropout_p=0.0, softmax_scale=None, causal=False, window_size=(-1, -1),
                    softcap=0.0, alibi_slopes=None, deterministic=False, return_attn_probs=False, *,
                    window_table: WindowSpec = None, qk_layout: str = "sorted_pair",
                    rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                    q_offset: Optional[int] = None, out: Optional[torch.Tensor] = None):
    """flash_attn_func(q, k, v, ...) with an optional ATFlash window table.

    q: (batch, seqlen_q, nheads, 128); k, v: (batch, seqlen_k, nheads_k, 128), bf16.
    window_table: None (dense), a WindowTable, or a zhi level tuple.
    qk_layout: pair order of q/k along head_dim: "sorted_pair" (the reference's
      kernel layout) or "rotate_half" (HF order; read in place, no permute copy).
    rope: optional (cos, sin) fp32 tables of shape (n_pos, 64); when given, q and k
      are pre-RoPE in rotate_half order (query i at position q_offset + i, key n at
      position n). k is rotated into sorted-pair order first (one pass); q is
      rotated by the prefill kernel itself as it loads each query tile.
    Returns out, or (out, softmax_lse, None) when return_attn_probs.
    """
    if dropout_p != 0.0:
        raise NotImplementedError("dropout is not supported")
    if tuple(window_size) != (-1, -1):
        raise NotImplementedError("sliding-window (window_size) is not supported; use window_table")
    if softcap != 0.0 or alibi_slopes is not None:
        raise NotImplementedError("softcap / alibi are not supported")
    q_rope = None
    if rope is not None:
        cos, sin = rope
        k = rope_pack(k, cos, sin, pos_offset=0, out_layout="sorted_pair")
        qk_layout = "sorted_pair"
        q_rope = (cos, sin)
    res = prefill_fwd(q, k, v, causal=causal, softmax_scale=softmax_scale, window_table=window_table,
                      qk_layout=qk_layout, q_offset=q_offset, out=out, return_lse=return_attn_probs,
                      q_rope=q_rope)
    if return_attn_probs:
        return res[0], res[1], None
    return res


_FA4_TUNING_SUFFIXES = ("_block_size", "num_threads", "num_stages", "_compute_capability")


def _flash_attn_fwd(q, k, v, softmax_scale=None, causal=False, pack_gqa=None,
                    atflash_window_zhi=None, **other):
    """Drop-in for the windowed FA4 entry point the reference calls
    (``flash_attn.cute.interface._flash_attn_fwd``): returns (out, lse).

    ``pack_gqa`` and FA4's tile-size / thread-count hints are accepted and
    ignored: this kernel always packs the G q heads of a kv head together.
    Any other FA4 option (varlen, paged K/V, softcap, sliding window, sinks)
    must be left at None; a value raises NotImplementedError instead of being
    dropped silently."""
    for name, value in other.items():
        if value is not None and not name.endswith(_FA4_TUNING_SUFFIXES):
            raise NotImplementedError(f"_flash_attn_fwd: {name}={value!r} is not supported by the windowed prefill")
    return prefill_fwd(q, k, v, causal=causal, softmax_scale=softmax_scale,
                       window_table=atflash_window_zhi, return_lse=True)
