"""ctypes binding of libwp_b200.so (the C ABI in include/wp_api.h).

The library is the only compute path: there is no CPU or stock-kernel
fallback. Importing this module does not need a GPU; loading the library
does not either (it links the CUDA runtime statically and calls nothing at
load time). Any call that needs a device fails loudly when there is none.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libwp_b200.so"

WP_OK = 0
WP_NOT_HANDLED = 1
WP_ERR_INVALID = -1
WP_ERR_CUDA = -2
WP_ERR_UNKNOWN_ADAPTER = -3
WP_ERR_CAPACITY = -4
WP_ERR_NCCL = -5
WP_ERR_DEVICE_TIMEOUT = -6

WP_DTYPE_F16 = 0
WP_DTYPE_BF16 = 1
WP_DTYPE_F32 = 2
WP_DTYPE_I32 = 3
WP_DTYPE_I64 = 4

WP_TABLE_LIVE = 0
WP_TABLE_REGISTRY = 1
WP_TABLE_TILES = 2
WP_TABLE_SHORT = 3

WP_SEG_DECODE = 0
WP_SEG_PREFILL = 1
WP_SEG_AUTO = 2


class WpConfig(ctypes.Structure):
    _fields_ = [
        ("device", ctypes.c_int32),
        ("max_tokens", ctypes.c_int32),
        ("num_staging_slots", ctypes.c_int32),
        ("slot_bytes", ctypes.c_int64),
        ("ctas_per_sm", ctypes.c_int32),
        ("use_pdl", ctypes.c_int32),
        ("prefetch_weights", ctypes.c_int32),
        ("kernel", ctypes.c_int32),
        ("prefill_tokens", ctypes.c_int32),
        ("peer_wait_ms", ctypes.c_int32),
        ("prefetch_inputs", ctypes.c_int32),
    ]


class WpBridge(ctypes.Structure):
    """wp_bridge (include/wp_api.h): one scheduler tick."""

    _fields_ = [
        ("whittle_scores", ctypes.c_float * 64),
        ("t_remaining_ms", ctypes.c_float * 64),
        ("gwar_pred_next3", ctypes.c_float * 64),
        ("lambda_hat", ctypes.c_float * 64),
        ("burst_active", ctypes.c_uint8 * 64),
        ("promo_eligible", ctypes.c_uint8 * 64),
        ("is_hot", ctypes.c_uint8 * 64),
        ("prefetch_ready", ctypes.c_uint8 * 64),
        ("tile_size_code", ctypes.c_uint8 * 64),
        ("step_id", ctypes.c_uint32),
        ("num_active_adapters", ctypes.c_uint32),
        ("num_segments", ctypes.c_uint32),
        ("global_load", ctypes.c_float),
    ]


class WpSegment(ctypes.Structure):
    _fields_ = [("adapter_id", ctypes.c_int32), ("token_start", ctypes.c_int32), ("token_count", ctypes.c_int32)]


_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_int = ctypes.c_int

# name -> (restype, argtypes); every function declared in include/wp_api.h.
SIGNATURES = {
    "wp_create": (_int, [ctypes.POINTER(WpConfig), ctypes.POINTER(_vp)]),
    "wp_destroy": (_int, [_vp]),
    "wp_last_error": (ctypes.c_char_p, [_vp]),
    "wp_rank_supported": (_int, [_i32]),
    "wp_kernel_launch_count": (_i64, [_vp]),
    "wp_last_apply_kernel": (ctypes.c_int32, [ctypes.c_void_p]),
    "wp_register_adapter": (_int, [_vp, _i32, _vp, _vp, _i32, _i32, _i32, _f32, _i32]),
    "wp_register_adapter_host": (_int, [_vp, _i32, _vp, _vp, _i32, _i32, _i32, _f32, _i32]),
    "wp_evict_adapter": (_int, [_vp, _i32]),
    "wp_build_segments": (_int, [_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32), _i32, _vp]),
    "wp_build_seg_bounds": (_int, [_vp, _vp, _i32, _i32, _vp]),
    "wp_build_seg_bounds_noalloc": (_int, [_vp, _i32, _i32, _vp, _vp, _vp]),
    "wp_seg_bounds_noalloc_max_tokens": (_int, []),
    "wp_read_seg_table": (_int, [_vp, _i32, ctypes.POINTER(WpSegment), _i32, ctypes.POINTER(_i32)]),
    "wp_shrink": (_int, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp]),
    "wp_expand": (_int, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp]),
    "wp_add_lora": (_int, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _i32, _f32, _i32, _i32, _i32, _i32, _i64, _i64,
                           _i32, _i32, _vp]),
    "wp_add_lora_slices": (_int, [_vp, _vp, _vp, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_i64),
                                  ctypes.POINTER(_vp), ctypes.POINTER(_i64), ctypes.POINTER(_i32), _i32, _f32,
                                  _i32, _i32, _i32, _i32, _i64, _i64, _i32, _vp]),
    "wp_add_lora_shrink": (_int, [_vp, _vp, _vp, _vp, _i64, _i32, _f32, _i32, _i32, _i32, _i64, _i32, _vp]),
    "wp_add_lora_expand": (_int, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i64, _i32, _i32, _vp]),
    "wp_prefetch_adapter": (_i32, [_vp, _i32]),
    "wp_prefetch_adapter_on": (_i32, [_vp, _i32, _vp]),
    "wp_is_prefetch_ready": (_i32, [_vp, _i32]),
    "wp_release_prefetch": (_int, [_vp, _i32]),
    "wp_slot_stats": (_int, [_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    "wp_device_error": (_int, [_vp, _i32, ctypes.POINTER(_i32)]),
    "wp_trace_enable": (_int, [_vp, _i32]),
    "wp_note_input_write": (_int, [_vp]),
    "wp_trace_read": (_int, [_vp, _i32, ctypes.POINTER(ctypes.c_uint64), _i32, ctypes.POINTER(_i32)]),
    "wp_apply_plan": (_int, [_vp, _i32, _i32, ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    "wp_tp_unique_id_bytes": (_i32, []),
    "wp_tp_get_unique_id": (_int, [_vp]),
    "wp_tp_init": (_int, [_vp, _vp, _i32, _i32]),
    "wp_tp_allreduce_f32": (_int, [_vp, _vp, _i64, _vp]),
    "wp_tp_destroy": (_int, [_vp]),
    "wp_tp_mailbox_handle_bytes": (_i32, []),
    "wp_tp_mailbox_create": (_int, [_vp, _i32, _i32, _i32, _vp]),
    "wp_tp_mailbox_open": (_int, [_vp, _vp]),
    "wp_tp_mailbox_close": (_int, [_vp]),
    "wp_add_lora_row_parallel": (_int, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _i32, _f32, _i32, _i32, _i32, _i32, _i64,
                                        _i64, _i32, _i32, _vp]),
    "wp_pool_create": (_int, [_vp, _i32, _i32, _i32, ctypes.POINTER(_i32), ctypes.POINTER(_i32), _i32, _i32,
                              ctypes.POINTER(_vp)]),
    "wp_pool_destroy": (_int, [_vp]),
    "wp_pool_layout": (_int, [_vp, _i32, ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "wp_pool_stack": (_int, [_vp, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_i64)]),
    "wp_pool_register_host": (_int, [_vp, _i32, _vp]),
    "wp_pool_evict": (_int, [_vp, _i32]),
    "wp_pool_prefetch": (_i32, [_vp, _i32]),
    "wp_pool_is_ready": (_i32, [_vp, _i32]),
    "wp_pool_release": (_int, [_vp, _i32]),
    "wp_pool_prepare": (_int, [_vp, ctypes.POINTER(_i32), _i32, _vp]),
    "wp_pool_stats": (_int, [_vp, ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(_i32)]),
    "wp_build_seg_bounds_pool": (_int, [_vp, _vp, _vp, _i32, _i32, _vp]),
    "wp_build_seg_bounds_ex": (_int, [_vp, _vp, _i32, _i32, _i32, _vp]),
    "wp_write_bridge": (_int, [_vp, ctypes.POINTER(WpBridge)]),
    "wp_read_bridge": (_int, [_vp, ctypes.POINTER(WpBridge)]),
    "wp_read_bridge_kernel": (_int, [_vp, ctypes.POINTER(ctypes.c_float), _i32, ctypes.POINTER(_i32)]),
}

_LIB = None


class WarpPipeError(RuntimeError):
    """An error status returned by libwp_b200.so."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[wp status {code}] {msg}")
        self.code = code


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load libwp_b200.so, building it in-tree first when it is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists() or os.environ.get("WP_REBUILD") == "1":
        if not build_if_missing:
            raise ImportError(f"{LIB_PATH} is not built; run python -m adapterslotsplusplus_b200.build")
        from .build import build

        build()
    lib = ctypes.CDLL(str(LIB_PATH), mode=ctypes.RTLD_LOCAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def check(rc: int, handle=None) -> int:
    """Raise WarpPipeError for negative statuses; return rc otherwise."""
    if rc < 0:
        lib = load()
        msg = lib.wp_last_error(handle).decode(errors="replace")
        raise WarpPipeError(rc, msg)
    return rc
