"""Paged-KV append: write new K/V tokens into a paged cache (FlashInfer's
``append_paged_kv_cache`` call shape), optionally applying RoPE to K and packing
it into the kernels' pair order on the way.

The reference's decode reads the KV cache that FlashInfer's append fills
(e2e_pipeline/atflash_e2e_fafi.py:219-223); this is that write side on the
library's own kernel (``atf_paged_kv_append``)."""
import ctypes
from typing import Optional, Tuple

import torch

from . import _ffi, _runtime

_LAYOUTS = {"sorted_pair": _ffi.ATF_LAYOUT_SORTED_PAIR, "rotate_half": _ffi.ATF_LAYOUT_ROTATE_HALF}


def get_batch_indices_positions(append_indptr: torch.Tensor, seq_lens: torch.Tensor,
                                nnz: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Request index and KV position of each appended token. Request b appends
    append_indptr[b+1] - append_indptr[b] tokens that end its sequence of
    seq_lens[b] tokens (lengths after the append)."""
    dev = append_indptr.device
    indptr = append_indptr.to(torch.int64)
    counts = indptr[1:] - indptr[:-1]
    batch = torch.repeat_interleave(torch.arange(counts.numel(), device=dev), counts)
    offs = torch.arange(nnz, device=dev) - indptr[batch]
    pos = seq_lens.to(dev, torch.int64)[batch] - counts[batch] + offs
    return batch.to(torch.int32), pos.to(torch.int32)


def append_paged_kv_cache(append_key: torch.Tensor, append_value: torch.Tensor, batch_indices: torch.Tensor,
                          positions: torch.Tensor, paged_kv_cache, kv_indices: torch.Tensor,
                          kv_indptr: torch.Tensor, kv_last_page_len: Optional[torch.Tensor] = None,
                          kv_layout: str = "NHD", *, rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                          rope_positions: Optional[torch.Tensor] = None, out_layout: str = "sorted_pair") -> None:
    """append_key / append_value (nnz, Hkv, 128) bf16; token i goes to request
    batch_indices[i] at KV position positions[i]. paged_kv_cache = (k_pages,
    v_pages) or one tensor with a k/v axis at dim 1; kv_layout "NHD" or "HND".
    rope = (cos, sin) fp32 (n_pos, >=64): K is pre-RoPE in HF rotate_half order
    and is rotated at rope_positions[i] (default positions[i]) and written in
    out_layout order. Out-of-range page indices are skipped and reported by
    ``atflash.check_device_errors()`` (code 2). kv_last_page_len is accepted for
    call compatibility; positions fully determine the slots."""
    if isinstance(paged_kv_cache, (tuple, list)):
        kc, vc = paged_kv_cache
    else:
        kc, vc = paged_kv_cache[:, 0], paged_kv_cache[:, 1]
    dev = _runtime.require_cuda(append_key, append_value, kc, vc)
    k_level_major = kc.dim() == 5
    for t in (append_key, append_value, vc) + (() if k_level_major else (kc,)):
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1 or t.shape[-1] != 128:
            raise ValueError("keys, values and cache pages must be bf16 with a contiguous head_dim of 128")
    if append_key.shape != append_value.shape or append_key.stride() != append_value.stride():
        raise ValueError("append_key and append_value must have the same shape and strides")
    if k_level_major:
        # (P, Hkv, 8 levels, page, 16) sorted-pair K pages (see BatchDecodeWithPagedKVCacheWrapper.run)
        if (kc.dtype != torch.bfloat16 or kc.shape[2] != 8 or kc.shape[4] != 16 or kc.stride(4) != 1
                or kc.stride(3) != 16 or vc.dim() != 4 or kc.shape[0] != vc.shape[0]):
            raise ValueError("level-major k pages must be (P, Hkv, 8, page, 16) bf16 with 16-element rows")
        if rope is not None and out_layout != "sorted_pair":
            raise ValueError("level-major k pages hold sorted-pair K")
    elif kc.shape != vc.shape or kc.stride() != vc.stride() or kc.dim() != 4:
        raise ValueError("k and v pages must have the same 4-d shape and strides")
    nnz, hkv, _ = append_key.shape
    if kv_layout == "NHD":
        npages, page, hk2, _ = vc.shape
        s_page, s_tok, s_head = vc.stride(0), vc.stride(1), vc.stride(2)
    elif kv_layout == "HND":
        npages, hk2, page, _ = vc.shape
        s_page, s_head, s_tok = vc.stride(0), vc.stride(1), vc.stride(2)
    else:
        raise ValueError("kv_layout must be NHD or HND")
    if hk2 != hkv:
        raise ValueError("append_key heads do not match the cache")
    bi = batch_indices.to(device=dev, dtype=torch.int32).contiguous()
    ps = positions.to(device=dev, dtype=torch.int32).contiguous()
    ip = kv_indptr.to(device=dev, dtype=torch.int32).contiguous()
    ix = kv_indices.to(device=dev, dtype=torch.int32).contiguous()
    if bi.numel() != nnz or ps.numel() != nnz:
        raise ValueError("batch_indices and positions need one entry per appended token")
    p = _ffi.AtfAppendParams()
    p.append_k, p.append_v, p.nnz = append_key.data_ptr(), append_value.data_ptr(), nnz
    p.a_stride_n, p.a_stride_h = append_key.stride(0), append_key.stride(1)
    p.batch_indices, p.positions = bi.data_ptr(), ps.data_ptr()
    p.k_cache, p.v_cache, p.num_pages = kc.data_ptr(), vc.data_ptr(), npages
    p.kv_stride_page, p.kv_stride_token, p.kv_stride_head = s_page, s_tok, s_head
    p.num_kv_heads, p.head_dim, p.page_size, p.batch_size = hkv, 128, page, ip.numel() - 1
    p.kv_indptr, p.kv_indices = ip.data_ptr(), ix.data_ptr()
    keep = [bi, ps, ip, ix]
    if rope is not None:
        cos, sin = rope
        if cos.dtype != torch.float32 or cos.shape != sin.shape or cos.stride() != sin.stride() or cos.stride(1) != 1:
            raise ValueError("cos/sin must be matching fp32 (n_pos, >=64) tables")
        p.cos, p.sin, p.cs_stride_pos, p.n_pos = cos.data_ptr(), sin.data_ptr(), cos.stride(0), cos.shape[0]
        if rope_positions is not None:
            rp = rope_positions.to(device=dev, dtype=torch.int64).contiguous()
            keep.append(rp)
            p.rope_positions = rp.data_ptr()
    p.out_layout = _LAYOUTS[out_layout]
    p.error_flag = _runtime.error_flag(dev).data_ptr()
    if k_level_major:
        if kc.shape[1] != hkv or kc.shape[3] != page:
            raise ValueError("level-major k pages do not match the v pages")
        p.k_level_major = 1
        p.k_stride_page, p.k_stride_head, p.k_stride_level = kc.stride(0), kc.stride(1), kc.stride(2)
    with torch.cuda.device(dev):
        rc = _ffi.load().atf_paged_kv_append(ctypes.byref(p), _runtime.stream_handle(dev))
    _ffi.check("atf_paged_kv_append", rc)
