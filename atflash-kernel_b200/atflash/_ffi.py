"""ctypes binding of libatflash_b200.so (include/atflash_b200.h).

The structures below mirror the C header field by field. The library is
loaded from this package's ``_lib`` directory; importing a kernel entry point
without it raises immediately (there is no CPU fallback).
"""
import ctypes
import os
import threading

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libatflash_b200.so")
_lib = None
_lock = threading.Lock()

ATF_OK = 0
ATF_LAYOUT_SORTED_PAIR, ATF_LAYOUT_ROTATE_HALF = 0, 1
ATF_KV_NHD, ATF_KV_HND = 0, 1
ATF_WINDOW_OFF, ATF_WINDOW_SNAP16, ATF_WINDOW_VEC8 = 0, 1, 2
ATF_DTYPE_BF16, ATF_DTYPE_F32 = 0, 1
ATF_NOALLOC_MAX_PARTIAL_ROWS = 16384

EXPORTED = ("atf_window_widths", "atf_window_zhi16", "atf_window_zhi8", "atf_window_deff",
            "atf_prefill_fwd", "atf_decode_plan", "atf_decode_run", "atf_decode_run_noalloc", "atf_lse_merge",
            "atf_rope_pack", "atf_paged_kv_append", "atf_status_string", "atf_version",
            "atf_read_error_flag", "atf_selftest_wait_timeout", "atf_params_size",
            "atf_exchange_region_bytes", "atf_state_push", "atf_state_merge", "atf_decode_run_exchange",
            "atf_ipc_export", "atf_ipc_import", "atf_ipc_release")
ATF_IPC_HANDLE_BYTES = 64

_i64, _i32, _f32, _vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p


class AtfPrefillParams(ctypes.Structure):
    _fields_ = [("q", _vp), ("k", _vp), ("v", _vp), ("out", _vp), ("lse", _vp),
                ("batch", _i64), ("seqlen_q", _i64), ("seqlen_k", _i64), ("num_heads_q", _i64),
                ("num_heads_kv", _i64), ("head_dim", _i64),
                ("q_stride_b", _i64), ("q_stride_s", _i64), ("q_stride_h", _i64),
                ("k_stride_b", _i64), ("k_stride_s", _i64), ("k_stride_h", _i64),
                ("v_stride_b", _i64), ("v_stride_s", _i64), ("v_stride_h", _i64),
                ("o_stride_b", _i64), ("o_stride_s", _i64), ("o_stride_h", _i64),
                ("q_offset", _i64), ("softmax_scale", _f32), ("causal", ctypes.c_int),
                ("qk_layout", ctypes.c_int), ("window", ctypes.c_int), ("zhi", _i32 * 8),
                ("error_flag", _vp), ("q_cos", _vp), ("q_sin", _vp), ("q_cs_stride_pos", _i64),
                ("q_n_pos", _i64), ("num_row_ranges", _i32), ("row_begin", _i64 * 2), ("row_end", _i64 * 2)]


class AtfDecodePlanParams(ctypes.Structure):
    _fields_ = [("batch_size", _i32), ("num_qo_heads", _i32), ("num_kv_heads", _i32),
                ("head_dim", _i32), ("page_size", _i32), ("indptr_host", _vp),
                ("last_page_len_host", _vp), ("num_sms", _i32), ("min_chunk_keys", _i32),
                ("max_chunk_keys", _i32), ("window", ctypes.c_int), ("zhi16", _i32 * 8),
                ("q_pos_host", _vp), ("kv_pos0_host", _vp)]


class AtfDecodePlan(ctypes.Structure):
    _fields_ = [("num_items", _i32), ("chunk_keys", _i32), ("partial_o_floats", _i64),
                ("partial_lse_floats", _i64)]


class AtfDecodeParams(ctypes.Structure):
    _fields_ = [("q", _vp), ("q_stride_b", _i64), ("q_stride_h", _i64),
                ("k_cache", _vp), ("v_cache", _vp), ("num_pages", _i64),
                ("kv_stride_page", _i64), ("kv_stride_token", _i64), ("kv_stride_head", _i64),
                ("kv_layout", ctypes.c_int), ("qk_layout", ctypes.c_int),
                ("indptr", _vp), ("indices", _vp), ("last_page_len", _vp),
                ("items", _vp), ("item_indptr", _vp), ("num_items", _i32),
                ("batch_size", _i32), ("num_qo_heads", _i32), ("num_kv_heads", _i32),
                ("head_dim", _i32), ("page_size", _i32),
                ("q_pos", _vp), ("kv_pos0", _vp), ("sm_scale", _f32), ("window", ctypes.c_int),
                ("zhi16", _i32 * 8), ("zhi8", _i32 * 16),
                ("partial_o", _vp), ("partial_lse", _vp), ("out", _vp),
                ("o_stride_b", _i64), ("o_stride_h", _i64), ("out_dtype", ctypes.c_int),
                ("lse_out", _vp), ("error_flag", _vp),
                ("k_level_major", ctypes.c_int), ("k_stride_page", _i64), ("k_stride_head", _i64),
                ("k_stride_level", _i64), ("enable_pdl", ctypes.c_int)]


class AtfMergeParams(ctypes.Structure):
    _fields_ = [("part_o", _vp), ("part_lse", _vp), ("part_indptr", _vp), ("num_parts", _i32),
                ("batch", _i32), ("num_heads", _i32), ("head_dim", _i32), ("lse_log2", ctypes.c_int),
                ("out", _vp), ("o_stride_b", _i64), ("o_stride_h", _i64), ("out_dtype", ctypes.c_int),
                ("lse_out", _vp), ("part_stride_o", _i64), ("part_stride_lse", _i64)]


class AtfRopeParams(ctypes.Structure):
    _fields_ = [("x", _vp), ("out", _vp), ("batch", _i64), ("seqlen", _i64), ("num_heads", _i64),
                ("head_dim", _i64), ("x_stride_b", _i64), ("x_stride_s", _i64), ("x_stride_h", _i64),
                ("o_stride_b", _i64), ("o_stride_s", _i64), ("o_stride_h", _i64),
                ("cos", _vp), ("sin", _vp), ("cs_stride_pos", _i64), ("n_pos", _i64),
                ("positions", _vp), ("pos_offset", _i64), ("out_layout", ctypes.c_int)]


class AtfAppendParams(ctypes.Structure):
    _fields_ = [("append_k", _vp), ("append_v", _vp), ("nnz", _i64), ("a_stride_n", _i64), ("a_stride_h", _i64),
                ("batch_indices", _vp), ("positions", _vp), ("k_cache", _vp), ("v_cache", _vp),
                ("num_pages", _i64), ("kv_stride_page", _i64), ("kv_stride_token", _i64),
                ("kv_stride_head", _i64), ("num_kv_heads", _i32), ("head_dim", _i32), ("page_size", _i32),
                ("batch_size", _i32), ("kv_indptr", _vp), ("kv_indices", _vp), ("cos", _vp), ("sin", _vp),
                ("cs_stride_pos", _i64), ("n_pos", _i64), ("rope_positions", _vp), ("out_layout", ctypes.c_int),
                ("error_flag", _vp), ("k_level_major", ctypes.c_int), ("k_stride_page", _i64),
                ("k_stride_head", _i64), ("k_stride_level", _i64)]


class AtfExchangeParams(ctypes.Structure):
    _fields_ = [("o", _vp), ("lse", _vp), ("o_stride_b", _i64), ("o_stride_h", _i64), ("batch", _i32),
                ("num_heads", _i32), ("world", _i32), ("rank", _i32), ("peer_base", _vp), ("base", _vp),
                ("out", _vp), ("out_stride_b", _i64), ("out_stride_h", _i64), ("out_dtype", ctypes.c_int),
                ("lse_out", _vp), ("error_flag", _vp)]


class AtfError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, fn, status):
        self.status = status
        super().__init__(f"{fn} failed: {status_string(status)} ({status})")


def lib_path() -> str:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise ImportError(f"{_LIB_PATH} is missing: build it with "
                                  "`python atflash-kernel_b200/build.py` (no CPU fallback exists)")
            lib = ctypes.CDLL(_LIB_PATH)
            P = ctypes.POINTER
            lib.atf_window_widths.argtypes = [ctypes.c_int, ctypes.c_double, ctypes.c_double, P(_f32)]
            lib.atf_window_zhi16.argtypes = [P(_f32), ctypes.c_int, _i64, P(_i32)]
            lib.atf_window_zhi8.argtypes = [P(_f32), ctypes.c_int, P(_i32)]
            lib.atf_window_deff.argtypes = [P(_i32), ctypes.c_int, _i64]
            lib.atf_prefill_fwd.argtypes = [P(AtfPrefillParams), _vp]
            lib.atf_decode_plan.argtypes = [P(AtfDecodePlanParams), P(_i32), _i32, P(_i32), P(AtfDecodePlan)]
            lib.atf_decode_run.argtypes = [P(AtfDecodeParams), _vp]
            lib.atf_decode_run_noalloc.argtypes = [P(AtfDecodeParams), _vp]
            lib.atf_lse_merge.argtypes = [P(AtfMergeParams), _vp]
            lib.atf_rope_pack.argtypes = [P(AtfRopeParams), _vp]
            lib.atf_paged_kv_append.argtypes = [P(AtfAppendParams), _vp]
            lib.atf_status_string.argtypes = [ctypes.c_int]
            lib.atf_status_string.restype = ctypes.c_char_p
            lib.atf_read_error_flag.argtypes = [_vp, P(ctypes.c_int)]
            lib.atf_selftest_wait_timeout.argtypes = [_vp, _vp]
            lib.atf_params_size.argtypes = [ctypes.c_char_p]
            lib.atf_exchange_region_bytes.argtypes = [_i32, _i32, _i32]
            lib.atf_state_push.argtypes = [P(AtfExchangeParams), _vp]
            lib.atf_state_merge.argtypes = [P(AtfExchangeParams), _vp]
            lib.atf_decode_run_exchange.argtypes = [P(AtfDecodeParams), P(AtfExchangeParams), _vp]
            lib.atf_ipc_export.argtypes = [_vp, _vp, P(_i64)]
            lib.atf_ipc_import.argtypes = [_vp, _i64, P(_vp), P(_vp)]
            lib.atf_ipc_release.argtypes = [_vp]
            for name in EXPORTED:
                if name not in ("atf_status_string", "atf_params_size", "atf_exchange_region_bytes"):
                    getattr(lib, name).restype = ctypes.c_int
            lib.atf_params_size.restype = _i64
            lib.atf_exchange_region_bytes.restype = _i64
            _lib = lib
    return _lib


def status_string(status: int) -> str:
    return load().atf_status_string(int(status)).decode()


def check(fn: str, status: int) -> None:
    if status != ATF_OK:
        raise AtfError(fn, status)
