"""ctypes binding of libiak_b200.so (the C ABI in include/intent_attention_b200.h).

The library is loaded lazily; every product entry point calls ``lib()``, which
raises ``RuntimeError`` when the CUDA extension is missing.  There is no CPU
fallback anywhere on the decode path.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("IAK_LIB", os.path.join(_HERE, "libiak_b200.so"))

IAK_OK, IAK_ERR_INVALID_ARG, IAK_ERR_UNSUPPORTED, IAK_ERR_CUDA, IAK_ERR_WORKSPACE, IAK_ERR_TIMEOUT = range(6)
DT_F32, DT_F16, DT_BF16 = 0, 1, 2
FMT_SKIP, FMT_F16, FMT_FP8, FMT_INT8, FMT_INT4, FMT_INT4R, FMT_SPARSE = range(7)
SCALE_PAGE, SCALE_GROUP32, SCALE_CHANNEL = 0, 1, 2
SCALE_MODES = {"page": SCALE_PAGE, "group32": SCALE_GROUP32, "channel": SCALE_CHANNEL}
KERNEL_AUTO, KERNEL_GENERIC, KERNEL_TENSOR = 0, 1, 2
KERNELS = {"auto": KERNEL_AUTO, "generic": KERNEL_GENERIC, "tensor": KERNEL_TENSOR}

c_void_p = ctypes.c_void_p
c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64


class PagePools(ctypes.Structure):
    _fields_ = [
        ("k_f16", c_void_p), ("v_f16", c_void_p), ("k_fp8", c_void_p), ("v_fp8", c_void_p),
        ("k_i8", c_void_p), ("v_i8", c_void_p), ("k_i4", c_void_p), ("v_i4", c_void_p),
        ("k_i4r", c_void_p), ("v_i4r", c_void_p),
        ("k_scale", c_void_p), ("v_scale", c_void_p), ("k_res_scale", c_void_p), ("v_res_scale", c_void_p),
        ("num_pages", c_i64), ("page_size", c_i32), ("head_dim", c_i32), ("scale_mode", c_i32),
    ]


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("q_dtype", c_i32), ("q_stride_b", c_i64), ("q_stride_h", c_i64),
        ("out", c_void_p), ("out_dtype", c_i32), ("out_stride_b", c_i64), ("out_stride_h", c_i64),
        ("batch", c_i32), ("num_q_heads", c_i32), ("num_table_heads", c_i32),
        ("page_table", c_void_p), ("pt_stride_b", c_i64), ("pt_stride_h", c_i64), ("table_width", c_i32),
        ("page_counts", c_void_p), ("pc_stride_b", c_i64),
        ("page_tags", c_void_p), ("tag_bytes", c_i32), ("tag_map", ctypes.c_uint8 * 16), ("tag_default", ctypes.c_uint8),
        ("sm_scale", ctypes.c_float),
        ("partial_m", c_void_p), ("partial_l", c_void_p), ("partial_acc", c_void_p),
        ("num_splits", c_i32), ("kernel", c_i32),
        ("status", c_void_p), ("wait_budget_ns", ctypes.c_uint32),
    ]


STATUS_DECODE_TIMEOUT = 1


class PackArgs(ctypes.Structure):
    _fields_ = [
        ("logical_ids", c_void_p), ("num_ids", c_i32),
        ("logical_tags", c_void_p), ("num_logical_pages", c_i32),
        ("bases", c_void_p), ("batch", c_i32), ("num_table_heads", c_i32), ("table_width", c_i32),
        ("page_table", c_void_p), ("page_counts", c_void_p), ("page_tags", c_void_p),
        ("num_tag_pages", c_i64), ("pad_value", c_i32),
    ]


class QuantArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p), ("x_dtype", c_i32), ("num_src_pages", c_i64),
        ("dst_ids", c_void_p), ("formats", c_void_p),
        ("given_scale", c_void_p), ("given_res_scale", c_void_p),
        ("f16", c_void_p), ("fp8", c_void_p), ("i8", c_void_p), ("i4", c_void_p), ("i4r", c_void_p),
        ("scale", c_void_p), ("res_scale", c_void_p),
        ("num_pages", c_i64), ("page_size", c_i32), ("head_dim", c_i32), ("scale_mode", c_i32),
    ]


class MlaArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("q_dtype", c_i32), ("q_stride_b", c_i64), ("q_stride_h", c_i64),
        ("out", c_void_p), ("out_dtype", c_i32), ("out_stride_b", c_i64), ("out_stride_h", c_i64),
        ("batch", c_i32), ("num_heads", c_i32), ("d_qk", c_i32), ("d_v", c_i32),
        ("dense_pages", c_void_p), ("dense_dtype", c_i32),
        ("fp8_pages", c_void_p), ("fp8_scale", c_void_p),
        ("num_pages", c_i64), ("page_size", c_i32),
        ("page_table", c_void_p), ("pt_stride_b", c_i64), ("table_width", c_i32),
        ("page_counts", c_void_p),
        ("page_tags", c_void_p), ("tag_bytes", c_i32), ("tag_map", ctypes.c_uint8 * 16), ("tag_default", ctypes.c_uint8),
        ("sm_scale", ctypes.c_float),
        ("partial_m", c_void_p), ("partial_l", c_void_p), ("partial_acc", c_void_p),
        ("num_splits", c_i32), ("kernel", c_i32),
    ]


MLA_SKIP, MLA_DENSE, MLA_FP8 = 0, 1, 2

CONVERT_MAX_ELEMS = 16384


class PrefillArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("q_dtype", c_i32), ("q_stride_b", c_i64), ("q_stride_h", c_i64), ("q_stride_m", c_i64),
        ("out", c_void_p), ("out_dtype", c_i32), ("out_stride_b", c_i64), ("out_stride_h", c_i64),
        ("out_stride_m", c_i64),
        ("batch", c_i32), ("num_q_heads", c_i32), ("num_table_heads", c_i32), ("num_queries", c_i32),
        ("q_positions", c_void_p), ("qp_stride_b", c_i64), ("causal", c_i32),
        ("page_table", c_void_p), ("pt_stride_b", c_i64), ("pt_stride_h", c_i64), ("table_width", c_i32),
        ("page_counts", c_void_p), ("pc_stride_b", c_i64),
        ("bases", c_void_p), ("page_positions", c_void_p), ("pp_stride_b", c_i64), ("pp_stride_h", c_i64),
        ("row_masks", c_void_p), ("rm_stride_b", c_i64),
        ("page_tags", c_void_p), ("tag_bytes", c_i32), ("tag_map", ctypes.c_uint8 * 16), ("tag_default", ctypes.c_uint8),
        ("sm_scale", ctypes.c_float), ("kernel", c_i32),
    ]


class AppendArgs(ctypes.Structure):
    _fields_ = [
        ("k_new", c_void_p), ("v_new", c_void_p), ("new_dtype", c_i32),
        ("batch", c_i32), ("num_table_heads", c_i32), ("num_new", c_i32),
        ("positions", c_void_p), ("new_lengths", c_void_p), ("bases", c_void_p),
        ("page_tags", c_void_p), ("tag_bytes", c_i32), ("tag_map", ctypes.c_uint8 * 16),
        ("tag_default", ctypes.c_uint8),
        ("k_stage", c_void_p), ("v_stage", c_void_p), ("dropped", c_void_p),
    ]


class ConvertArgs(ctypes.Structure):
    _fields_ = [
        ("page_ids", c_void_p), ("num_ids", c_i32), ("new_formats", c_void_p),
        ("page_tags", c_void_p), ("tag_bytes", c_i32), ("tag_map", ctypes.c_uint8 * 16),
        ("tag_default", ctypes.c_uint8), ("fmt_to_tag", ctypes.c_uint8 * 8), ("rejected", c_void_p),
    ]

POLICY_ALWAYS, POLICY_ATTEND, POLICY_SKIP, POLICY_RECENT, POLICY_GLOBAL = range(5)
PREC_FP16, PREC_FP8, PREC_INT8, PREC_INT4, PREC_INT4_RESIDUAL, PREC_SKIP = range(6)
ROUTE_MAX_BLOCKS = 8192


class RouteArgs(ctypes.Structure):
    _fields_ = [
        ("num_blocks", c_i32), ("block_counts", c_void_p),
        ("block_start", c_void_p), ("block_end", c_void_p), ("block_policy", c_void_p),
        ("layout_stride", c_i64),
        ("scores", c_void_p), ("score_stride", c_i64),
        ("seq_lens", c_void_p),
        ("batch", c_i32), ("num_table_heads", c_i32), ("page_size", c_i32),
        ("top_k_blocks", c_i32), ("preserve_recent", c_i32), ("preserve_global", c_i32),
        ("score_threshold", ctypes.c_double), ("memory_pressure", ctypes.c_double),
        ("high_score_threshold", ctypes.c_double), ("medium_score_threshold", ctypes.c_double),
        ("bases", c_void_p), ("table_width", c_i32), ("pad_value", c_i32),
        ("page_table", c_void_p), ("page_counts", c_void_p), ("num_selected", c_void_p),
        ("page_prec", c_void_p),
        ("page_tags", c_void_p), ("num_tag_pages", c_i64), ("prec_to_tag", ctypes.c_uint8 * 6),
        ("row_masks", c_void_p),
    ]

MAX_PEERS = 8


class PeerExchange(ctypes.Structure):
    _fields_ = [("areas", c_void_p * MAX_PEERS), ("rank", c_i32), ("world", c_i32), ("rows", c_i64),
                ("head_dim", c_i32)]


# name -> (restype, argtypes); mirrors every declaration of the public header
SIGNATURES = {
    "iak_version": (ctypes.c_int, []),
    "iak_last_error": (ctypes.c_char_p, []),
    "iak_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32),
                                         ctypes.POINTER(ctypes.c_uint32), c_i32]),
    "iak_decode_workspace_size": (ctypes.c_int, [ctypes.POINTER(PagePools), ctypes.POINTER(DecodeArgs),
                                                 ctypes.POINTER(ctypes.c_size_t)]),
    "iak_decode": (ctypes.c_int, [ctypes.POINTER(PagePools), ctypes.POINTER(DecodeArgs), c_void_p,
                                  ctypes.c_size_t, c_void_p]),
    "iak_merge_partials": (ctypes.c_int, [c_void_p, c_void_p, c_void_p, c_i64, c_i32, c_i32, c_void_p, c_i32,
                                          c_i64, c_void_p]),
    "iak_pack_metadata": (ctypes.c_int, [ctypes.POINTER(PackArgs), c_void_p]),
    "iak_route_pages": (ctypes.c_int, [ctypes.POINTER(RouteArgs), c_void_p]),
    "iak_append_tokens": (ctypes.c_int, [ctypes.POINTER(PagePools), ctypes.POINTER(AppendArgs), c_void_p]),
    "iak_convert_pages": (ctypes.c_int, [ctypes.POINTER(PagePools), ctypes.POINTER(ConvertArgs), c_void_p]),
    "iak_prefill": (ctypes.c_int, [ctypes.POINTER(PagePools), ctypes.POINTER(PrefillArgs), c_void_p]),
    "iak_quantize_pages": (ctypes.c_int, [ctypes.POINTER(QuantArgs), c_void_p]),
    "iak_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(PagePools), ctypes.POINTER(DecodeArgs), c_void_p]),
    "iak_decode_exchange": (ctypes.c_int, [ctypes.POINTER(PagePools), ctypes.POINTER(DecodeArgs),
                                           ctypes.POINTER(PeerExchange), c_void_p, ctypes.c_size_t, c_void_p]),
    "iak_merge_partial_blocks": (ctypes.c_int, [c_void_p, c_i32, c_i64, c_i32, c_void_p, c_i32, c_i64, c_void_p]),
    "iak_mla_workspace_size": (ctypes.c_int, [ctypes.POINTER(MlaArgs), ctypes.POINTER(ctypes.c_size_t)]),
    "iak_mla_decode": (ctypes.c_int, [ctypes.POINTER(MlaArgs), c_void_p, ctypes.c_size_t, c_void_p]),
    "iak_exchange_area_bytes": (ctypes.c_int, [c_i32, c_i64, c_i32, ctypes.POINTER(ctypes.c_size_t)]),
    "iak_exchange_staging_ptr": (c_void_p, [c_void_p, c_i32, c_i64, c_i32]),
    "iak_exchange_push": (ctypes.c_int, [ctypes.POINTER(PeerExchange), c_void_p]),
    "iak_exchange_merge": (ctypes.c_int, [ctypes.POINTER(PeerExchange), c_void_p, c_i32, c_i64, c_void_p,
                                          ctypes.c_uint32, c_void_p]),
    "iak_ipc_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(c_void_p), c_void_p]),
    "iak_ipc_open": (ctypes.c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "iak_ipc_close": (ctypes.c_int, [c_void_p]),
    "iak_ipc_free": (ctypes.c_int, [c_void_p]),
    "iak_kernel_timer_enable": (ctypes.c_int, [c_i32]),
    "iak_kernel_timer_read": (ctypes.c_int, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(c_i32)]),
    "iak_kernel_timer_disable": (ctypes.c_int, []),
}
NOALLOC_SCRATCH_BYTES = 8 << 20

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None
_load_error: Optional[str] = None


def _load() -> Optional[ctypes.CDLL]:
    global _lib, _load_error
    with _lock:
        if _lib is not None or _load_error is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            _load_error = (f"the CUDA extension {LIB_PATH} is not built "
                           "(run: python intent-attention-kernel_b200/build.py)")
            return None
        try:
            lib = ctypes.CDLL(LIB_PATH)
        except OSError as e:  # pragma: no cover - depends on the machine
            _load_error = f"cannot load {LIB_PATH}: {e}"
            return None
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name, None)
            if fn is None:
                _load_error = f"{LIB_PATH} does not export {name}"
                return None
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return _lib


def available() -> bool:
    return _load() is not None


def lib() -> ctypes.CDLL:
    """The loaded library; raises RuntimeError if the extension is missing."""
    l = _load()
    if l is None:
        raise RuntimeError(_load_error)
    return l


def check(status: int, what: str) -> None:
    if status == IAK_OK:
        return
    msg = lib().iak_last_error().decode(errors="replace")
    if status == IAK_ERR_INVALID_ARG:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed (status {status}): {msg}")


def device_status(reset: bool = True) -> dict:
    """Timeout counters of the current device: warps whose bounded device-side
    wait gave up in the tensor-core decode, the tcgen05 MLA decode and the
    tcgen05 prefill since the last reset.  Waits for the device."""
    v = [ctypes.c_uint32(0) for _ in range(3)]
    st = lib().iak_device_status(ctypes.byref(v[0]), ctypes.byref(v[1]), ctypes.byref(v[2]), 1 if reset else 0)
    if st not in (IAK_OK, IAK_ERR_TIMEOUT):
        check(st, "iak_device_status")
    return {"decode": v[0].value, "mla": v[1].value, "prefill": v[2].value}


def raise_on_timeouts(reset: bool = True) -> None:
    """RuntimeError if any device-side wait gave up since the last reset."""
    st = device_status(reset)
    if any(st.values()):
        raise RuntimeError(f"device-side waits gave up (warps per kernel family): {st}")


class KernelTimer:
    """CUDA-event timing of the main decode kernel of each decode call
    (measurement only).  ``with KernelTimer(n) as t: ...`` then ``t.total_ms``,
    ``t.launches`` (read after the block, which waits for the events)."""

    def __init__(self, max_launches: int):
        self.max_launches = int(max_launches)
        self.total_ms = 0.0
        self.launches = 0

    def __enter__(self):
        check(lib().iak_kernel_timer_enable(self.max_launches), "iak_kernel_timer_enable")
        return self

    def __exit__(self, *exc):
        try:
            if exc[0] is None:
                ms, n = ctypes.c_double(0.0), c_i32(0)
                check(lib().iak_kernel_timer_read(ctypes.byref(ms), ctypes.byref(n)), "iak_kernel_timer_read")
                self.total_ms, self.launches = ms.value, n.value
        finally:
            lib().iak_kernel_timer_disable()
        return False
