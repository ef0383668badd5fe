"""Paged-KV decode wrapper shaped like FlashInfer's BatchDecodeWithPagedKVCacheWrapper.

The reference decodes one request at a time through
``single_decode_with_kv_cache_with_jit_module(mod, q, k, v, None, zhi8, ...)``
(e2e_pipeline/atflash_e2e_fafi.py:106-110) with the window in the K-load
predicate (kernels/flashinfer_port/decode.cuh.diff:51-89). This wrapper keeps
FlashInfer's batch plan()/run() interface and adds ``window_table``.

Window modes: "snap16" (16-dim levels at per-key granularity, equal to
atflash/reference.py with phase="decode", block_m = block_n = 1) or "vec8"
(8-dim slices, the FlashInfer port's table; sorted-pair K layout only).
"""
import ctypes
import math
from typing import Optional, Sequence, Tuple, Union

import numpy as np
import torch

from . import _ffi, _runtime
from .window_table import KERNEL_CAP, WindowTable, zhi_slice_vec8

_LAYOUTS = {"sorted_pair": _ffi.ATF_LAYOUT_SORTED_PAIR, "rotate_half": _ffi.ATF_LAYOUT_ROTATE_HALF}


def _host_i32(t) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        return t.detach().to("cpu", torch.int32).numpy().astype(np.int32, copy=True)
    return np.asarray(t, dtype=np.int32).copy()


class BatchDecodeWithPagedKVCacheWrapper:
    def __init__(self, float_workspace_buffer: torch.Tensor, kv_layout: str = "NHD",
                 use_cuda_graph: bool = False, use_tensor_cores: bool = False,
                 paged_kv_indptr_buffer=None, paged_kv_indices_buffer=None,
                 paged_kv_last_page_len_buffer=None, backend: str = "auto", jit_args=None):
        if kv_layout not in ("NHD", "HND"):
            raise ValueError("kv_layout must be NHD or HND")
        if not float_workspace_buffer.is_cuda:
            raise ValueError("the workspace buffer must be a CUDA tensor")
        self._ws = float_workspace_buffer
        self._kv_layout = kv_layout
        self._plan = None
        self._use_cuda_graph = bool(use_cuda_graph)

    @property
    def is_cuda_graph_enabled(self) -> bool:
        """True when built with use_cuda_graph: run() may then be captured in a
        CUDA graph and replayed, with the plan and the q / cache / out buffers
        fixed (the tables live on the device and run() neither allocates nor
        synchronises when out is given)."""
        return self._use_cuda_graph

    def reset_workspace_buffer(self, float_workspace_buffer, int_workspace_buffer=None):
        self._ws = float_workspace_buffer
        if self._plan is not None:
            # the planned launch parameters point into the workspace
            P = self._plan
            need = 4 * (P["po_floats"] + P["pl_floats"]) + 256
            if self._ws.numel() * self._ws.element_size() < need:
                raise ValueError(f"workspace too small for the current plan: need {need} bytes")
            self._bind_workspace()

    def plan(self, indptr, indices, last_page_len, num_qo_heads: int, num_kv_heads: int,
             head_dim: int, page_size: int, pos_encoding_mode: str = "NONE", window_left: int = -1,
             logits_soft_cap=None, q_data_type="bfloat16", kv_data_type=None, data_type=None,
             sm_scale: Optional[float] = None, rope_scale=None, rope_theta=None,
             non_blocking: bool = True, *, window_table: Union[None, WindowTable, Sequence[int]] = None,
             window_mode: str = "snap16", qk_layout: str = "sorted_pair",
             max_chunk_keys: int = 0, min_chunk_keys: int = 0, q_pos=None, kv_pos0=None):
        """Build the split-KV schedule for a batch of paged requests.

        window_table: None (dense), a WindowTable, or a zhi level tuple (snap16).
        qk_layout: pair order of the cached K and of q ("sorted_pair" or "rotate_half").
        q_pos / kv_pos0: the positions run() will be given (per request; defaults
        kv_len - 1 and 0). Under a snap16 window the work items are cut to equal
        bytes read at these distances; they steer the balance only, never the result.
        """
        if pos_encoding_mode != "NONE":
            raise NotImplementedError("RoPE is applied before the cache (pos_encoding_mode NONE)")
        if window_left != -1 or logits_soft_cap not in (None, 0.0):
            raise NotImplementedError("window_left / logits_soft_cap are not supported")
        if head_dim != 128:
            raise NotImplementedError("head_dim must be 128")
        if window_mode not in ("snap16", "vec8"):
            raise ValueError("window_mode must be snap16 or vec8")
        if qk_layout not in _LAYOUTS:
            raise ValueError(f"qk_layout must be one of {sorted(_LAYOUTS)}")
        dev = self._ws.device
        indptr_h = _host_i32(indptr)
        lpl_h = _host_i32(last_page_len)
        B = len(indptr_h) - 1
        if B < 1 or len(lpl_h) != B:
            raise ValueError("indptr must have batch+1 entries and last_page_len batch entries")
        nnz = int(indptr_h[-1])
        idx_dev = indices if isinstance(indices, torch.Tensor) else torch.tensor(indices)
        if idx_dev.numel() < nnz:
            raise ValueError("indices is shorter than indptr[-1]")
        if np.any(np.diff(indptr_h) < 0) or indptr_h[0] != 0:
            raise ValueError("indptr must start at 0 and be non-decreasing")
        pp = _ffi.AtfDecodePlanParams()
        pp.batch_size, pp.num_qo_heads, pp.num_kv_heads = B, num_qo_heads, num_kv_heads
        pp.head_dim, pp.page_size = head_dim, page_size
        pp.indptr_host = indptr_h.ctypes.data
        pp.last_page_len_host = lpl_h.ctypes.data
        pp.num_sms = torch.cuda.get_device_properties(dev).multi_processor_count
        pp.min_chunk_keys, pp.max_chunk_keys = int(min_chunk_keys), int(max_chunk_keys)
        # window tables
        zhi16 = [KERNEL_CAP] * 8
        zhi8 = [2 ** 31 - 1] * 16
        mode = _ffi.ATF_WINDOW_OFF
        if window_table is not None:
            if window_mode == "vec8":
                if qk_layout != "sorted_pair":
                    raise ValueError("vec8 windows need the sorted-pair K layout")
                if not isinstance(window_table, WindowTable):
                    zhi8 = [int(x) for x in window_table]
                    if len(zhi8) != 16:
                        raise ValueError("a vec8 table has 16 entries")
                else:
                    zhi8 = window_table.zhi8
                mode = _ffi.ATF_WINDOW_VEC8
            else:
                zhi16 = list(window_table.zhi16 if isinstance(window_table, WindowTable)
                             else [int(x) for x in window_table])
                if len(zhi16) != 8:
                    raise ValueError("a zhi level table has 8 entries")
                if any(zhi16[i] < zhi16[i + 1] for i in range(7)) or min(zhi16) < 0:
                    raise ValueError("zhi levels must be non-negative and non-increasing")
                zhi16[0] = max(zhi16[0], KERNEL_CAP)
                mode = _ffi.ATF_WINDOW_SNAP16
        pp.window = mode
        for i in range(8):
            pp.zhi16[i] = zhi16[i]
        pos_h = []
        for name, v in (("q_pos", q_pos), ("kv_pos0", kv_pos0)):
            if v is None:
                pos_h.append(None)
                continue
            a = np.ascontiguousarray((v.detach().cpu().numpy() if isinstance(v, torch.Tensor) else np.asarray(v))
                                     .astype(np.int64).reshape(-1))
            if a.shape[0] != B:
                raise ValueError(f"{name} must have one entry per request")
            pos_h.append(a)
        pp.q_pos_host = pos_h[0].ctypes.data if pos_h[0] is not None else None
        pp.kv_pos0_host = pos_h[1].ctypes.data if pos_h[1] is not None else None
        plan = _ffi.AtfDecodePlan()
        lib = _ffi.load()
        _ffi.check("atf_decode_plan", lib.atf_decode_plan(ctypes.byref(pp), None, 0, None, ctypes.byref(plan)))
        items = np.zeros((max(1, plan.num_items), 4), dtype=np.int32)
        item_indptr = np.zeros(B + 1, dtype=np.int32)
        _ffi.check("atf_decode_plan", lib.atf_decode_plan(
            ctypes.byref(pp), items.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), items.shape[0],
            item_indptr.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ctypes.byref(plan)))
        need = 4 * (plan.partial_o_floats + plan.partial_lse_floats) + 256
        if self._ws.numel() * self._ws.element_size() < need:
            raise ValueError(f"workspace too small: need {need} bytes")
        kv_lens = [(int(indptr_h[b + 1] - indptr_h[b]) - 1) * page_size + int(lpl_h[b])
                   if indptr_h[b + 1] > indptr_h[b] else 0 for b in range(B)]
        self._plan = {
            "B": B, "Hq": num_qo_heads, "Hkv": num_kv_heads, "page_size": page_size,
            "num_items": plan.num_items, "chunk_keys": plan.chunk_keys,
            "items": torch.from_numpy(items).to(dev, non_blocking=False),
            "item_indptr": torch.from_numpy(item_indptr).to(dev),
            "indptr": torch.from_numpy(indptr_h).to(dev),
            "indices": idx_dev.to(device=dev, dtype=torch.int32).contiguous(),
            "last_page_len": torch.from_numpy(lpl_h).to(dev),
            "po_floats": plan.partial_o_floats, "pl_floats": plan.partial_lse_floats,
            "sm_scale": float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(head_dim),
            "window": mode, "zhi16": zhi16, "zhi8": zhi8, "layout": _LAYOUTS[qk_layout],
            "kv_lens": kv_lens,
        }
        # everything of the launch parameters that the plan fixes, filled once;
        # run() copies this template and sets the per-call pointers only
        P = self._plan
        t = _ffi.AtfDecodeParams()
        t.kv_layout = _ffi.ATF_KV_NHD if self._kv_layout == "NHD" else _ffi.ATF_KV_HND
        t.qk_layout = P["layout"]
        t.indptr, t.indices = P["indptr"].data_ptr(), P["indices"].data_ptr()
        t.last_page_len = P["last_page_len"].data_ptr()
        t.items, t.item_indptr, t.num_items = P["items"].data_ptr(), P["item_indptr"].data_ptr(), P["num_items"]
        t.batch_size, t.num_qo_heads, t.num_kv_heads, t.head_dim, t.page_size = B, num_qo_heads, num_kv_heads, 128, \
            page_size
        t.sm_scale = P["sm_scale"]
        t.window = P["window"]
        for i in range(8):
            t.zhi16[i] = zhi16[i]
        for i in range(16):
            t.zhi8[i] = zhi8[i]
        t.error_flag = _runtime.error_flag(dev).data_ptr()
        self._tmpl = t
        self._bind_workspace()

    def _bind_workspace(self):
        """Point the launch template at the workspace: partial outputs, then
        partial LSEs."""
        P, t = self._plan, self._tmpl
        ws = self._ws.view(torch.uint8) if self._ws.dtype != torch.uint8 else self._ws
        base = (ws.data_ptr() + 255) // 256 * 256
        t.partial_o, t.partial_lse = base, base + 4 * P["po_floats"]

    begin_forward = plan

    def run(self, q: torch.Tensor, paged_kv_cache, *args, q_scale=None, k_scale=None, v_scale=None,
            out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
            return_lse: bool = False, enable_pdl=None, window_left=None,
            q_pos: Optional[torch.Tensor] = None, kv_pos0: Optional[torch.Tensor] = None,
            out_dtype: Optional[torch.dtype] = None, exchange=None):
        """q (B, Hq, 128) bf16; paged_kv_cache = (k_pages, v_pages) or one tensor with
        a k/v axis at dim 1. Returns out (B, Hq, 128) [, lse (B, Hq), natural log].

        enable_pdl=True launches the decode as a programmatic dependent of the
        previous kernel on the stream: its prologue (the plan and the page table:
        items, indptr, indices, last_page_len) runs while that kernel finishes, and
        everything else (q, q_pos, kv_pos0, the KV pages, the outputs) waits for
        it. Leave it off when the kernel just before the decode writes the page
        table. The results are the same either way.

        With `exchange` (an atflash.dist.StateExchange whose ranks run on
        different GPUs) this is one KV-sharded step: the decode's split merge also
        exchanges the ranks' states (atf_decode_run_exchange), and out / lse are
        the merge over every rank of the exchange."""
        if self._plan is None:
            raise RuntimeError("plan() must be called before run()")
        if q_scale is not None or k_scale is not None or v_scale is not None:
            raise NotImplementedError("fp8 scales are not supported")
        P = self._plan
        if isinstance(paged_kv_cache, (tuple, list)):
            kc, vc = paged_kv_cache
        else:
            kc, vc = paged_kv_cache[:, 0], paged_kv_cache[:, 1]
        dev = _runtime.require_cuda(q, kc, vc)
        if kc.dtype != torch.bfloat16 or vc.dtype != torch.bfloat16 or q.dtype != torch.bfloat16:
            raise TypeError("q and the KV cache must be bfloat16")
        # K pages are either laid out like V (4-d, NHD / HND) or level-major:
        # (P, Hkv, 8 levels, page, 16) in sorted-pair order, so that a page's
        # in-window levels are one contiguous run
        k_level_major = kc.dim() == 5
        if k_level_major:
            if (kc.shape[2] != 8 or kc.shape[4] != 16 or kc.stride(4) != 1 or kc.stride(3) != 16
                    or vc.dim() != 4 or kc.shape[0] != vc.shape[0]):
                raise ValueError("level-major k pages must be (P, Hkv, 8, page, 16) with 16-element rows")
        elif kc.stride() != vc.stride() or kc.shape != vc.shape or kc.dim() != 4:
            raise ValueError("k and v pages must have the same 4-d shape and strides")
        if vc.stride(-1) != 1 or q.stride(-1) != 1:
            raise ValueError("the head_dim axis must be contiguous")
        if self._kv_layout == "NHD":
            _, page, hkv, d = vc.shape
            s_page, s_tok, s_head = vc.stride(0), vc.stride(1), vc.stride(2)
        else:
            _, hkv, page, d = vc.shape
            s_page, s_head, s_tok = vc.stride(0), vc.stride(1), vc.stride(2)
        if k_level_major and (kc.shape[1] != hkv or kc.shape[3] != page):
            raise ValueError("level-major k pages do not match the v pages")
        if page != P["page_size"] or hkv != P["Hkv"] or d != 128:
            raise ValueError("KV cache shape does not match the plan")
        B, Hq = P["B"], P["Hq"]
        if tuple(q.shape) != (B, Hq, 128):
            raise ValueError(f"q must be ({B}, {Hq}, 128)")
        odt = out_dtype or (out.dtype if out is not None else torch.bfloat16)
        if odt not in (torch.bfloat16, torch.float32):
            raise TypeError("out_dtype must be bfloat16 or float32")
        if out is None:
            out = torch.empty((B, Hq, 128), dtype=odt, device=dev)
        elif (tuple(out.shape) != (B, Hq, 128) or out.dtype != odt or out.device != q.device
              or out.stride(-1) != 1):
            raise ValueError(f"out must be a ({B}, {Hq}, 128) {odt} tensor on {q.device} with a "
                             "contiguous head_dim axis")
        if return_lse and lse is None:
            lse = torch.empty((B, Hq), dtype=torch.float32, device=dev)
        if lse is not None and (tuple(lse.shape) != (B, Hq) or lse.dtype != torch.float32
                                or lse.device != q.device or lse.stride() != (Hq, 1)):
            raise ValueError(f"lse must be a contiguous float32 ({B}, {Hq}) tensor on {q.device}")
        a = _ffi.AtfDecodeParams.from_buffer_copy(self._tmpl)
        a.q, a.q_stride_b, a.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
        a.k_cache, a.v_cache = kc.data_ptr(), vc.data_ptr()
        a.num_pages = kc.shape[0]
        a.kv_stride_page, a.kv_stride_token, a.kv_stride_head = s_page, s_tok, s_head
        keep = []
        if q_pos is not None:
            q_pos = q_pos.to(device=dev, dtype=torch.int64).contiguous()
            keep.append(q_pos)
            a.q_pos = q_pos.data_ptr()
        if kv_pos0 is not None:
            kv_pos0 = kv_pos0.to(device=dev, dtype=torch.int64).contiguous()
            keep.append(kv_pos0)
            a.kv_pos0 = kv_pos0.data_ptr()
        a.out, a.o_stride_b, a.o_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
        a.out_dtype = _ffi.ATF_DTYPE_F32 if out.dtype == torch.float32 else _ffi.ATF_DTYPE_BF16
        a.lse_out = lse.data_ptr() if lse is not None else None
        # programmatic dependent launch: the decode's prologue (plan and page
        # table reads) overlaps the previous kernel on the stream; opt-in, since a
        # kernel that writes the page table must not directly precede the decode
        a.enable_pdl = 1 if enable_pdl else 0
        if k_level_major:
            a.k_level_major = 1
            a.k_stride_page, a.k_stride_head, a.k_stride_level = kc.stride(0), kc.stride(1), kc.stride(2)
        if exchange is not None:
            x = exchange._fused_params(dev)
            with torch.cuda.device(dev):
                rc = _ffi.load().atf_decode_run_exchange(ctypes.byref(a), ctypes.byref(x),
                                                         _runtime.stream_handle(dev))
            _ffi.check("atf_decode_run_exchange", rc)
            return (out, lse) if return_lse else out
        with torch.cuda.device(dev):
            rc = _ffi.load().atf_decode_run(ctypes.byref(a), _runtime.stream_handle(dev))
        _ffi.check("atf_decode_run", rc)
        return (out, lse) if return_lse else out

    forward = run


def lse_merge(part_o: torch.Tensor, part_lse: torch.Tensor, *, lse_log2: bool = False,
              out_dtype: torch.dtype = torch.bfloat16, return_lse: bool = False):
    """Merge P partial states: part_o (P, B, H, 128) fp32, part_lse (P, B, H) fp32.
    The parts may be strided views (e.g. of one all-gathered flat buffer): each
    part's own block must be contiguous, the part stride of part_o a multiple of 4."""
    dev = _runtime.require_cuda(part_o, part_lse)
    Pn, B, H, D = part_o.shape
    if D != 128 or tuple(part_lse.shape) != (Pn, B, H):
        raise ValueError("part_o must be (P, B, H, 128) and part_lse (P, B, H)")
    part_o = part_o.float()
    part_lse = part_lse.float()

    def _parts_ok(t, align0):
        # each part's block contiguous; the part stride spans at least a block
        exp = 1
        for dim in range(t.dim() - 1, 0, -1):
            if t.shape[dim] != 1 and t.stride(dim) != exp:
                return False
            exp *= t.shape[dim]
        return t.shape[0] == 1 or (t.stride(0) >= exp and t.stride(0) % align0 == 0)

    if not _parts_ok(part_o, 4):
        part_o = part_o.contiguous()
    if not _parts_ok(part_lse, 1):
        part_lse = part_lse.contiguous()
    out = torch.empty((B, H, D), dtype=out_dtype, device=dev)
    lse = torch.empty((B, H), dtype=torch.float32, device=dev) if return_lse else None
    m = _ffi.AtfMergeParams()
    m.part_o, m.part_lse, m.part_indptr = part_o.data_ptr(), part_lse.data_ptr(), None
    m.num_parts, m.batch, m.num_heads, m.head_dim = Pn, B, H, D
    m.lse_log2 = 1 if lse_log2 else 0
    m.out, m.o_stride_b, m.o_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    m.out_dtype = _ffi.ATF_DTYPE_F32 if out_dtype == torch.float32 else _ffi.ATF_DTYPE_BF16
    m.lse_out = lse.data_ptr() if lse is not None else None
    m.part_stride_o = part_o.stride(0) if Pn > 1 else 0
    m.part_stride_lse = part_lse.stride(0) if Pn > 1 else 0
    with torch.cuda.device(dev):
        rc = _ffi.load().atf_lse_merge(ctypes.byref(m), _runtime.stream_handle(dev))
    _ffi.check("atf_lse_merge", rc)
    return (out, lse) if return_lse else out
