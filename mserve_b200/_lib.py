"""ctypes binding of libmserve_kv.so (C ABI declared in include/mserve_kv.h).

The library is loaded from the package directory; if it is missing this module raises
ImportError with the build command.  There is no fallback implementation: every public
operation of the package runs through these entry points.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmserve_kv.so"

MSKV_OK = 0
MSKV_ERR_ARG = 1
MSKV_ERR_NOT_MAPPED = 2
MSKV_ERR_DTYPE = 3
MSKV_ERR_CUDA = 4
MSKV_ERR_RANGE = 5

# size of the device array behind mskv_sparse_attention_noalloc (MSKV_NOALLOC_ATTN_SCRATCH_BYTES)
MSKV_NOALLOC_SCRATCH_BYTES = 8 << 20

STATUS_INDEX_OOB = 0x1
STATUS_BAD_PAGE = 0x2
STATUS_DST_OOB = 0x4
STATUS_TIMEOUT = 0x8

DT_F32 = 0
DT_F16 = 1
DT_BF16 = 2
DT_F64 = 3
DT_FP8_E4M3 = 4
DT_FP8_E5M2 = 5

_vp = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int32


class Rows(C.Structure):
    """mskv_rows: addressing of one side of a row move (see include/mserve_kv.h)."""
    _fields_ = [
        ("base_k", _vp), ("base_v", _vp),
        ("stride_b", _i64), ("stride_h", _i64), ("stride_t", _i64), ("stride_page", _i64),
        ("pt_stride_b", _i64), ("len_scalar", _i64), ("num_pages", _i64),
        ("page_table", _vp), ("ring_start", _vp), ("tok0", _vp), ("len", _vp),
        ("page_size", _i32), ("ring_cap", _i32),
    ]


class GatherDesc(C.Structure):
    _fields_ = [
        ("src", Rows), ("dst", Rows),
        ("indices", _vp), ("idx_stride_b", _i64), ("idx_stride_h", _i64),
        ("counts", _vp), ("cnt_stride_b", _i64), ("cnt_stride_h", _i64),
        ("row_bytes", _i64), ("status", _vp),
        ("index_bits", _i32), ("batch", _i32), ("heads", _i32), ("num_selected", _i32),
        ("max_ctas", _i32), ("pad_", _i32),
    ]


class CopyDesc(C.Structure):
    _fields_ = [
        ("src", Rows), ("dst", Rows),
        ("counts", _vp), ("row_bytes", _i64), ("status", _vp),
        ("batch", _i32), ("heads", _i32), ("num_tokens", _i32), ("max_ctas", _i32),
    ]


class ScoreDesc(C.Structure):
    _fields_ = [
        ("k", Rows), ("q", _vp), ("q_stride_b", _i64), ("q_stride_h", _i64),
        ("scores", _vp), ("scores_stride", _i64), ("max_tokens", _i64), ("status", _vp),
        ("dtype", _i32), ("method", _i32), ("batch", _i32), ("q_heads", _i32),
        ("kv_heads", _i32), ("head_dim", _i32),
    ]


class TopkDesc(C.Structure):
    _fields_ = [
        ("scores", _vp), ("scores_stride", _i64), ("out_idx", _vp), ("out_stride", _i64),
        ("counts", _vp), ("len", _vp), ("top_k", _vp), ("status", _vp),
        ("scale", C.c_float), ("len_scalar", _i32), ("top_k_scalar", _i32), ("recent", _i32),
        ("num_sel", _i32), ("rows_per_sel", _i32), ("sel_per_batch", _i32), ("out_bits", _i32),
        ("row_block", _i32), ("sel_stride", _i64), ("block_stride", _i64),
    ]


class AttnDesc(C.Structure):
    _fields_ = [
        ("q", _vp), ("q_stride_b", _i64), ("q_stride_h", _i64), ("q_stride_q", _i64),
        ("k", _vp), ("v", _vp), ("kv_stride_seg", _i64), ("kv_stride_s", _i64),
        ("counts", _vp), ("out", _vp), ("out_stride_b", _i64), ("out_stride_h", _i64),
        ("out_stride_q", _i64), ("workspace", _vp), ("workspace_bytes", C.c_uint64),
        ("status", _vp), ("scale", C.c_float), ("dtype", _i32), ("batch", _i32), ("q_heads", _i32),
        ("kv_heads", _i32), ("head_dim", _i32), ("q_len", _i32), ("num_selected", _i32),
    ]


class FilterDesc(C.Structure):
    _fields_ = [
        ("attn", _vp), ("stride_h", _i64), ("stride_q", _i64), ("stride_k", _i64),
        ("out_idx", _vp), ("out_count", _vp), ("workspace", _vp), ("workspace_bytes", C.c_uint64),
        ("global_thr", C.c_float), ("individual_thr", C.c_float), ("dtype", _i32), ("heads", _i32),
        ("img_start", _i32), ("img_seq", _i32), ("text_start", _i32), ("text_seq", _i32),
        ("round_f16", _i32), ("pad_", _i32),
    ]


# (name, restype, argtypes) of every exported function, in header order.
SIGNATURES = [
    ("mskv_abi_version", C.c_int, []),
    ("mskv_last_error", C.c_char_p, []),
    ("mskv_launch_count", C.c_uint64, []),
    ("mskv_host_alloc", C.c_int, [C.POINTER(_vp), C.c_uint64]),
    ("mskv_host_free", C.c_int, [_vp]),
    ("mskv_host_register", C.c_int, [_vp, C.c_uint64]),
    ("mskv_host_unregister", C.c_int, [_vp]),
    ("mskv_device_view", C.c_int, [_vp, C.POINTER(_vp)]),
    ("mskv_uva_gather", C.c_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32,
                                  _vp, _vp, _vp, _vp]),
    ("mskv_gather", C.c_int, [C.POINTER(GatherDesc), _vp]),
    ("mskv_copy_rows", C.c_int, [C.POINTER(CopyDesc), _vp]),
    ("mskv_score", C.c_int, [C.POINTER(ScoreDesc), _vp]),
    ("mskv_score_fanout", C.c_int, [C.POINTER(ScoreDesc), C.POINTER(_vp), _i32, _vp]),
    ("mskv_topk", C.c_int, [C.POINTER(TopkDesc), _vp]),
    ("mskv_attention_workspace_bytes", C.c_uint64, [C.POINTER(AttnDesc)]),
    ("mskv_sparse_attention", C.c_int, [C.POINTER(AttnDesc), _vp]),
    ("mskv_image_filter_workspace_bytes", C.c_uint64, [_i32, _i32]),
    ("mskv_image_filter", C.c_int, [C.POINTER(FilterDesc), _vp]),
    ("mskv_ipc_handle_bytes", C.c_uint64, []),
    ("mskv_ipc_alloc", C.c_int, [C.c_uint64, C.POINTER(_vp), _vp]),
    ("mskv_ipc_open", C.c_int, [_vp, C.POINTER(_vp)]),
    ("mskv_ipc_close", C.c_int, [_vp]),
    ("mskv_ipc_free", C.c_int, [_vp]),
    ("mskv_flag_signal", C.c_int, [C.POINTER(_vp), _i32, _i32, _i64, _vp]),
    ("mskv_flag_wait", C.c_int, [_vp, _i32, _i64, _i32, C.c_uint64, _vp, _vp]),
]

_lib = None


def lib() -> C.CDLL:
    """Loads libmserve_kv.so once (RuntimeError/ImportError with the build command if absent)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `python -m mserve_b200.build` "
                              "(nvcc with sm_100a support is required)")
        h = C.CDLL(str(LIB_PATH))
        for name, res, args in SIGNATURES:
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        if h.mskv_abi_version() != 2:
            raise ImportError(f"{LIB_PATH}: unexpected ABI version {h.mskv_abi_version()}")
        _lib = h
    return _lib


class MskvError(RuntimeError):
    """A libmserve_kv entry point returned an error code."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def check(rc: int) -> None:
    if rc != MSKV_OK:
        msg = lib().mskv_last_error().decode(errors="replace")
        raise MskvError(rc, msg)


def launch_count() -> int:
    return int(lib().mskv_launch_count())
