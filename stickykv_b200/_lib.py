"""ctypes binding of the native C ABI (``include/stickykv_b200.h``).

The library ``_native/libstickykv_b200.so`` is built in-tree by
``python -m stickykv_b200.build``.  There is no fallback: if the library is
missing every kernel call raises ``NativeLibraryError``.
"""

from __future__ import annotations

import ctypes as C
import os
import threading
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_native", "libstickykv_b200.so")

SKV_OK = 0
SKV_F32, SKV_F16, SKV_BF16 = 0, 1, 2
PAGE_TOKENS = 8
QGROUP = 32

# Every symbol the header declares (checked by the CPU test-suite).
EXPORTS = (
    "skv_abi_version", "skv_status_string", "skv_last_cuda_error", "skv_page_bytes",
    "skv_struct_size",
    "skv_evict_plan_compute", "skv_append", "skv_decode_workspace_size", "skv_decode_attention",
    "skv_evict_workspace_size", "skv_evict", "skv_prefill_workspace_size",
    "skv_prefill_attention", "skv_pack_pages", "skv_decode_attention_noalloc",
    "skv_decode_attention_append", "skv_materialize", "skv_evict_append",
)
NOALLOC_SCRATCH_BYTES = 16 << 20


class NativeLibraryError(RuntimeError):
    """The native library is missing or a native call failed."""


class LayerDesc(C.Structure):
    _fields_ = [
        ("batch", C.c_int32), ("num_kv_heads", C.c_int32), ("num_q_heads", C.c_int32),
        ("head_dim", C.c_int32), ("kv_dtype", C.c_int32), ("window_size", C.c_int32),
        ("num_sink", C.c_int32), ("sink_pad", C.c_int32), ("fp_capacity", C.c_int32),
        ("tier_page_capacity", C.c_int32), ("k_fp", C.c_void_p), ("v_fp", C.c_void_p),
        ("tier_pages", C.c_void_p), ("tier_table", C.c_void_p), ("rope_cos", C.c_void_p),
        ("rope_sin", C.c_void_p), ("rope_positions", C.c_int32), ("reserved", C.c_int32 * 7),
    ]


class EvictPlan(C.Structure):
    _fields_ = [
        ("local_windows", C.c_int32), ("evictable_windows", C.c_int32),
        ("kept_evictable", C.c_int32), ("retained_windows", C.c_int32),
        ("seq_len_new", C.c_int32), ("tier_pages_new", C.c_int32), ("fp_len_new", C.c_int32),
        ("reserved", C.c_int32),
    ]


class EvictArgs(C.Structure):
    _fields_ = [
        ("seq_len", C.c_int32), ("tier_pages", C.c_int32), ("num_windows", C.c_int32),
        ("top_k_windows", C.c_int32), ("local_windows", C.c_int32),
        ("scores_capacity", C.c_int32), ("scores_src", C.c_void_p), ("scores_dst", C.c_void_p),
        ("ids_src", C.c_void_p), ("ids_dst", C.c_void_p), ("retained_out", C.c_void_p),
        ("next_window_id", C.c_int64),
    ]


_lib: Optional[C.CDLL] = None
_lock = threading.Lock()


def _declare(lib: C.CDLL) -> None:
    P, I32, I64, SZ, F = C.c_void_p, C.c_int32, C.c_int64, C.c_size_t, C.c_float
    sig = {
        "skv_abi_version": (C.c_int, []),
        "skv_status_string": (C.c_char_p, [C.c_int]),
        "skv_last_cuda_error": (C.c_char_p, []),
        "skv_page_bytes": (I32, [I32]),
        "skv_struct_size": (I32, [I32]),
        "skv_evict_plan_compute": (C.c_int, [I32, I32, I32, I32, I32, I32, I32, C.POINTER(EvictPlan)]),
        "skv_append": (C.c_int, [C.POINTER(LayerDesc), I32, I32, P, P, I64, I64, I64, I32, P]),
        "skv_decode_workspace_size": (SZ, [C.POINTER(LayerDesc), I32]),
        "skv_decode_attention": (C.c_int, [C.POINTER(LayerDesc), I32, I32, P, I64, I64, P, I64,
                                           I64, F, P, I32, P, SZ, P]),
        "skv_evict_workspace_size": (SZ, [C.POINTER(LayerDesc), I32]),
        "skv_evict": (C.c_int, [C.POINTER(LayerDesc), C.POINTER(LayerDesc), C.POINTER(EvictArgs),
                                P, SZ, P]),
        "skv_evict_append": (C.c_int, [C.POINTER(LayerDesc), C.POINTER(LayerDesc), C.POINTER(EvictArgs),
                                       P, P, I64, I64, P, SZ, P]),
        "skv_prefill_workspace_size": (SZ, [C.POINTER(LayerDesc), I32]),
        "skv_prefill_attention": (C.c_int, [C.POINTER(LayerDesc), I32, P, P, P, P, F, P, I32, P,
                                            SZ, P]),
        "skv_pack_pages": (C.c_int, [C.POINTER(LayerDesc), P, P, I32, I32, P, P]),
        "skv_materialize": (C.c_int, [C.POINTER(LayerDesc), I32, I32, P, P, P]),
        "skv_decode_attention_noalloc": (C.c_int, [C.POINTER(LayerDesc), I32, I32, P, I64, I64, P,
                                                   I64, I64, F, P, I32, P]),
        "skv_decode_attention_append": (C.c_int, [C.POINTER(LayerDesc), I32, I32, P, P, I64, I64, P,
                                                  I64, I64, P, I64, I64, F, P, I32, P, SZ, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib() -> C.CDLL:
    """Load (once) and return the native library; raise if it is missing."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise NativeLibraryError(
                        f"native library not built: {LIB_PATH} (run python -m stickykv_b200.build)")
                handle = C.CDLL(LIB_PATH)
                _declare(handle)
                if handle.skv_abi_version() != 1:
                    raise NativeLibraryError("ABI version mismatch")
                for i, st in enumerate((LayerDesc, EvictPlan, EvictArgs)):
                    if handle.skv_struct_size(i) != C.sizeof(st):
                        raise NativeLibraryError(f"struct layout mismatch for {st.__name__}")
                _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != SKV_OK:
        L = lib()
        msg = L.skv_status_string(status).decode()
        if status == 5:
            msg += " (" + L.skv_last_cuda_error().decode() + ")"
        exc = {2: NotImplementedError, 4: MemoryError, 5: RuntimeError}.get(status, ValueError)
        raise exc(f"{what} failed: {msg} [status {status}]")


def evict_plan(seq_len: int, num_windows: int, num_sink: int, window_size: int, top_k: int,
               local_windows: int, tier: bool) -> EvictPlan:
    p = EvictPlan()
    check(lib().skv_evict_plan_compute(seq_len, num_windows, num_sink, window_size, top_k,
                                       local_windows, int(tier), C.byref(p)), "skv_evict_plan_compute")
    return p


def page_bytes(head_dim: int) -> int:
    return 2 * PAGE_TOKENS * (head_dim // 2 + (head_dim // QGROUP) * 4)
