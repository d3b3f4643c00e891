"""ctypes binding of libpagegauge_b200.so (the C ABI in include/pagegauge_b200.h).

The shared library is built in-tree (``python -m pagegauge_b200.build``).
There is no fallback: if the library is missing, every operator raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_NAME = "libpagegauge_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_vp = ctypes.c_void_p
c_f32p = ctypes.POINTER(ctypes.c_float)
c_i32p = ctypes.POINTER(ctypes.c_int32)


class PgDecodeItem(ctypes.Structure):
    _fields_ = [("request", c_i32), ("head_seg", c_i32), ("idx_begin", c_i32), ("count", c_i32)]


class PgSegment(ctypes.Structure):
    _fields_ = [
        ("k_cache", c_vp), ("v_cache", c_vp), ("num_pages", c_i64),
        ("indices", c_vp), ("last_page_len", c_vp), ("k_scale", c_vp), ("v_scale", c_vp),
    ]


class PgPlanInfo(ctypes.Structure):
    _fields_ = [
        ("num_items", c_i64), ("max_items_per_head", c_i32), ("single_item_per_head", c_i32),
        ("split_pages", c_i32 * 2), ("warps_per_cta", c_i32),
    ]


class PgDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_vp), ("q_stride_b", c_i64), ("q_stride_h", c_i64),
        ("batch", c_i32), ("kv_heads", c_i32), ("group", c_i32), ("sm_scale", ctypes.c_float),
        ("seg", PgSegment * 2),
        ("items", c_vp), ("item_off", c_vp), ("num_items", c_i32), ("warps_per_cta", c_i32),
        ("part_o", c_vp), ("part_lse", c_vp), ("final_mode", c_i32),
        ("out", c_vp), ("out_stride_b", c_i64), ("out_stride_h", c_i64), ("lse_out", c_vp),
        ("extra_o", c_vp), ("extra_stride_b", c_i64), ("extra_stride_h", c_i64), ("extra_lse", c_vp),
        ("value_center", c_vp), ("vc_stride_b", c_i64), ("stage_mask", c_i32),
        ("merge_sem", c_vp), ("cluster", c_i32),
        ("representation", c_i32), ("k_bias", c_vp), ("v_bias", c_vp),
        ("int8_after_wait", c_i32),
    ]


class PgGemmArgs(ctypes.Structure):
    _fields_ = [
        ("w", c_vp), ("ldw", c_i64), ("x", c_vp), ("ldx", c_i64), ("y", c_vp), ("ldy", c_i64),
        ("residual", c_vp), ("ldr", c_i64),
        ("n", c_i32), ("k", c_i32), ("batch", c_i32), ("mode", c_i32), ("grid", c_i32),
        ("pdl", c_i32), ("partials", c_vp), ("partial_floats", c_i64), ("counters", c_vp),
        ("num_counters", c_i32), ("norm_weight", c_vp), ("norm_eps", ctypes.c_float),
        ("tp_world", c_i32), ("tp_rank", c_i32), ("tp_tiles_cap", c_i32), ("tp_peers", c_vp * 8),
    ]


# name -> (restype, argtypes); every entry point returns int32 status.
_SIGNATURES = {
    "pg_last_error": (ctypes.c_char_p, []),
    "pg_abi_version": (c_i32, []),
    "pg_read_device_error": (c_i32, [c_i32p]),
    "pg_struct_sizes": (c_i32, [ctypes.POINTER(c_i64), c_i32]),
    "pg_host_device_pointer": (c_i32, [c_vp, ctypes.POINTER(c_vp)]),
    "pg_tp_exchange_bytes": (c_i64, [c_i32]),
    "pg_tp_exchange_create": (c_i32, [c_i32, ctypes.POINTER(c_vp), c_vp]),
    "pg_tp_exchange_open": (c_i32, [c_vp, ctypes.POINTER(c_vp)]),
    "pg_tp_exchange_close": (c_i32, [c_vp]),
    "pg_tp_exchange_destroy": (c_i32, [c_vp]),
    "pg_tp_publish": (c_i32, [ctypes.POINTER(c_vp), c_i32, c_i32, c_i32, c_i32, c_i32, c_vp,
                              c_i64, c_vp]),
    "pg_tp_reduce": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_i64, c_vp, ctypes.c_float,
                             c_vp, c_i64, c_i32, c_vp]),
    "pg_rope_append_fp16": (c_i32, [c_vp] * 8 + [c_i64] * 3 + [c_i32] * 3 + [c_i64, c_i64, c_vp, c_i64, c_i64, c_vp]),
    "pg_rope_append_page_gauge": (
        c_i32,
        [c_vp] * 14 + [c_i64] * 4 + [c_i32] * 3 + [c_i64] * 4 + [c_vp, c_i64, c_i64, c_vp],
    ),
    "pg_rope_append_fp16_batched": (c_i32, [c_vp] * 8 + [c_i64] * 3 + [c_i32] * 3 + [c_i64, c_vp, c_i64, c_i64, c_vp]),
    "pg_rope_append_page_gauge_batched": (
        c_i32,
        [c_vp] * 14 + [c_i64] * 4 + [c_i32] * 3 + [c_i64] * 3 + [c_vp, c_i64, c_i64, c_i32, c_vp],
    ),
    "pg_rope_append_page_gauge_served": (
        c_i32, [c_vp] * 15 + [c_i64] * 3 + [c_i32] * 3 + [c_i64] * 3 + [c_vp] * 4 + [c_i64, c_i64, c_vp],
    ),
    "pg_zero_pool_pages": (c_i32, [c_vp] * 4 + [c_i64, c_i32, c_vp, c_i32, c_vp]),
    "pg_exact_tail_merge_center": (
        c_i32,
        [c_vp, c_vp, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32,
         ctypes.c_double, c_vp],
    ),
    "pg_decode_plan": (
        c_i32,
        [c_i32, c_i32, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_i64, c_vp,
         ctypes.POINTER(PgPlanInfo)],
    ),
    "pg_decode_run": (c_i32, [ctypes.POINTER(PgDecodeArgs), c_vp]),
    "pg_decode_max_clusters": (c_i32, [c_i32, c_i32, c_i32p]),
    "pg_decode_static": (c_i32, [ctypes.POINTER(PgDecodeArgs), c_vp, c_vp, c_i32, c_i32, c_i32, c_vp]),
    "pg_merge_state_in_place": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "pg_add_rmsnorm": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_i64, c_i64, c_i64,
                               ctypes.c_float, c_vp]),
    "pg_silu_mul": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_i64, c_i64, c_vp]),
    "pg_step_positions": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_vp]),
    "pg_argmax_rows": (c_i32, [c_vp, c_i64, c_i32, c_i32, c_i64, c_vp, c_vp, c_vp]),
    "pg_pack_weight": (c_i32, [c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp]),
    "pg_skinny_gemm_workspace": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,
                                         ctypes.POINTER(c_i64), c_i32p]),
    "pg_skinny_gemm": (c_i32, [ctypes.POINTER(PgGemmArgs), c_vp]),
    "pg_quantize_pages": (c_i32, [c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_vp]),
    "pg_quantize_affine_group16": (c_i32, [c_vp, c_i64, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None


def library_path() -> Path:
    override = os.environ.get("PAGEGAUGE_B200_LIB")
    return Path(override) if override else LIB_PATH


def load() -> ctypes.CDLL:
    """Load the CUDA library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.is_file():
        raise RuntimeError(
            f"PageGauge CUDA library not found at {path}; build it with "
            "`python -m pagegauge_b200.build` (no CPU fallback exists)"
        )
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    # The argument blocks cross the boundary by pointer: their layouts must
    # match the library's exactly.
    sizes = (c_i64 * 5)()
    if lib.pg_struct_sizes(sizes, 5) != 0:
        raise RuntimeError("pg_struct_sizes failed")
    mine = (ctypes.sizeof(PgDecodeArgs), ctypes.sizeof(PgGemmArgs), ctypes.sizeof(PgSegment),
            ctypes.sizeof(PgPlanInfo), ctypes.sizeof(PgDecodeItem))
    if tuple(sizes) != mine:
        raise RuntimeError(f"C ABI structure sizes {tuple(sizes)} differ from the binding's {mine}")
    _lib = lib
    return lib


def check(rc: int) -> None:
    """Translate a non-zero status into RuntimeError with the library message."""
    if rc != 0:
        msg = load().pg_last_error().decode("utf-8", "replace")
        raise RuntimeError(msg or f"pagegauge_b200 call failed with status {rc}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))


def kernel_pointer(t, name: str) -> int:
    """Address a kernel may use for tensor ``t``: its device address, or for
    a page-locked host tensor the mapped device address of the host buffer
    (read or written over the host link, zero copy)."""
    if t.is_cuda:
        return t.data_ptr()
    if t.is_pinned():
        out = c_vp()
        check(load().pg_host_device_pointer(c_vp(t.data_ptr()), ctypes.byref(out)))
        return int(out.value)
    raise RuntimeError(f"{name} must be CUDA or page-locked host memory")
