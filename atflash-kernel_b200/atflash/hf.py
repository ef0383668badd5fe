"""Hugging Face transformers integration: an ``AttentionInterface`` function that
runs a model's attention on the windowed kernels.

This mirrors the reference's harness function ``atflash_attention``
(e2e_pipeline/atflash_e2e_fafi.py:81-120) and its model setup (:123-190):

  * L > 1 (prefill or a prefill chunk): the windowed prefill on BSHD views of
    HF's (b, h, L, d) tensors, bottom-right causal (the chunk sees the whole
    cache);
  * L == 1 (decode): the decode kernel over HF's own contiguous KV cache, read
    as one page of S tokens per request (HND pages).

HF applies RoPE in rotate_half order; both kernels read that order in place
(``qk_layout="rotate_half"``), so no permutation of q/k is needed (the
reference patched apply_rotary_pos_emb to permute). Window widths come from the
raw RoPE base (the reference's width/order separation), or from the model's own
inv_freq (``widths="inv_freq"``); the pair order must be canonical either way.

Usage::

    import atflash.hf
    name = atflash.hf.register(model, k_ret_prefill=2.0, k_ret_decode=2.0)
    model.set_attn_implementation(name)   # or load with attn_implementation=name
"""
import math
from typing import Optional

import torch

from . import window_table as WT
from .decode import BatchDecodeWithPagedKVCacheWrapper
from .prefill import prefill_fwd

# transformers routes any implementation whose name contains "flash" through its
# FlashAttention path, hence a name without it (as the reference notes).
DEFAULT_NAME = "atf_window"

_STATE = {"prefill": None, "decode": None, "ws": {}, "plans": {}}


def window_tables_for_model(model, k_ret_prefill: float, k_ret_decode: Optional[float] = None,
                            widths: str = "raw_base"):
    """(prefill, decode) WindowTables for an HF model. widths="raw_base" takes the
    config's rope_theta (the reference's tables); "inv_freq" takes the model's
    own, possibly scaled, frequencies. Raises if the pair order is not canonical
    (e2e_pipeline/atflash_e2e_fafi.py:143-157)."""
    k_ret_decode = k_ret_prefill if k_ret_decode is None else k_ret_decode
    inv = model.model.rotary_emb.inv_freq.detach().float().cpu()
    order, canonical = WT.pair_order_from_inv_freq(inv)
    if not canonical:
        raise ValueError(f"the model's inv_freq is not in canonical pair order: {order[:8]}")
    d = 2 * inv.numel()
    if widths == "inv_freq":
        return WT.WindowTable.from_inv_freq(inv, k_ret_prefill), WT.WindowTable.from_inv_freq(inv, k_ret_decode)
    if widths != "raw_base":
        raise ValueError('widths must be "raw_base" or "inv_freq"')
    cfg = model.config
    base = getattr(cfg, "rope_theta", None) or (getattr(cfg, "rope_scaling", None) or {}).get("rope_theta")
    if base is None:
        rp = getattr(cfg, "rope_parameters", None) or {}
        base = rp.get("rope_theta")
    if base is None:
        raise ValueError("the model config has no rope_theta")
    return WT.WindowTable(d, float(base), float(k_ret_prefill)), WT.WindowTable(d, float(base), float(k_ret_decode))


def configure(prefill: Optional[WT.WindowTable], decode: Optional[WT.WindowTable]) -> None:
    """Set the windows the attention function uses (None: dense)."""
    _STATE["prefill"] = prefill
    _STATE["decode"] = decode
    _STATE["plans"].clear()


def _workspace(dev) -> torch.Tensor:
    ws = _STATE["ws"].get(dev)
    if ws is None:
        ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)
        _STATE["ws"][dev] = ws
    return ws


def atflash_attention(module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                      attention_mask=None, scaling: Optional[float] = None, dropout: float = 0.0, **kwargs):
    """transformers AttentionInterface entry: query (b, hq, L, d), key/value
    (b, hkv, S, d) after RoPE; returns ((b, L, hq, d), None). Causal with the
    query block at the end of the keys; padding masks are not applied (as in
    the reference's harness)."""
    if dropout != 0.0:
        raise NotImplementedError("attention dropout is not supported")
    b, hq, L, d = query.shape
    S = key.shape[-2]
    if L > S:
        raise ValueError(f"query block longer than the keys: L={L} S={S}")
    if L == 1:
        return _decode(query, key, value, scaling), None
    q = query.transpose(1, 2)
    k = key.transpose(1, 2)
    v = value.transpose(1, 2)
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    out = prefill_fwd(q, k, v, causal=True, softmax_scale=scaling, window_table=_STATE["prefill"],
                      qk_layout="rotate_half", q_offset=S - L)
    return out, None


def _decode(query, key, value, scaling):
    b, hq, _, d = query.shape
    hkv, S = key.shape[1], key.shape[2]
    kc, vc = key, value
    if kc.stride(-1) != 1 or kc.stride(1) != S * d or kc.stride(0) != hkv * S * d:
        kc = kc.contiguous()
    if vc.stride() != kc.stride():
        vc = vc.contiguous()
        kc = kc.contiguous()
    dev = query.device
    # every layer of one decode step has the same shapes: plan once per step
    # (the last planned shape is kept; a new length replaces it)
    key = (dev, b, hq, hkv, d, S, scaling)
    w = _STATE["plans"].get(key)
    if w is None:
        w = BatchDecodeWithPagedKVCacheWrapper(_workspace(dev), kv_layout="HND")
        indptr = torch.arange(b + 1, dtype=torch.int32)
        w.plan(indptr, torch.arange(b, dtype=torch.int32), torch.full((b,), S, dtype=torch.int32), hq, hkv, d, S,
               window_table=_STATE["decode"], qk_layout="rotate_half",
               sm_scale=scaling if scaling is not None else 1.0 / math.sqrt(d))
        _STATE["plans"].clear()
        _STATE["plans"][key] = w
    out = w.run(query[:, :, 0, :], (kc, vc))           # (b, hq, d)
    return out.view(b, 1, hq, d)


def register(model=None, k_ret_prefill: Optional[float] = None, k_ret_decode: Optional[float] = None,
             widths: str = "raw_base", name: str = DEFAULT_NAME) -> str:
    """Register ``atflash_attention`` with transformers under `name` and set the
    windows: from `model` and the k values when given, dense otherwise."""
    from transformers import AttentionInterface
    if "flash" in name:
        raise ValueError("transformers treats names containing 'flash' as FlashAttention")
    AttentionInterface.register(name, atflash_attention)
    if model is not None and k_ret_prefill is not None:
        configure(*window_tables_for_model(model, k_ret_prefill, k_ret_decode, widths))
    else:
        configure(None, None)
    return name
