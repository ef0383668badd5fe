# -*- coding: utf-8 -*-
"""ATFlash windowed attention on B200 (sm_100a).

    window_table   the window rule (per-pair widths, D_eff, zhi levels), bit-exact
                   with the reference's atflash/window_table.py
    flash_attn_func / prefill_fwd / _flash_attn_fwd
                   windowed causal prefill on the tcgen05/TMEM kernel
    BatchDecodeWithPagedKVCacheWrapper
                   windowed paged-KV GQA decode (split-KV + LSE merge)
    rope_pack      fused RoPE + pair-order pack (pre-RoPE HF q/k -> kernel layout)
    append_paged_kv_cache
                   write new K/V tokens into a paged cache (RoPE + pack on K)
    dist           zig-zag sharded prefill and KV-sharded decode over torch.distributed
    hf             transformers AttentionInterface function (import atflash.hf)

All compute runs in libatflash_b200.so through its C ABI (include/atflash_b200.h);
there is no CPU path.
"""
from . import window_table
from ._ffi import AtfError, lib_path
from ._runtime import check_device_errors
from .append import append_paged_kv_cache, get_batch_indices_positions
from .decode import BatchDecodeWithPagedKVCacheWrapper, lse_merge
from .prefill import _flash_attn_fwd, flash_attn_func, prefill_fwd
from .rope import cos_sin_table, inv_freq, rope_pack
from .window_table import WindowTable
from . import dist


def _fail_loudly_without_library():
    import os

    import torch
    if torch.cuda.is_available() and not os.path.exists(lib_path()):
        raise ImportError(f"atflash: {lib_path()} is missing on a CUDA machine; build it with "
                          "`python atflash-kernel_b200/build.py`")


_fail_loudly_without_library()

__all__ = ["window_table", "WindowTable", "flash_attn_func", "prefill_fwd", "_flash_attn_fwd",
           "BatchDecodeWithPagedKVCacheWrapper", "lse_merge", "rope_pack", "cos_sin_table",
           "inv_freq", "check_device_errors", "dist", "AtfError", "append_paged_kv_cache",
           "get_batch_indices_positions"]
