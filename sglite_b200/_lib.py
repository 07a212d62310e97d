"""ctypes binding of the C-ABI library ``lib/libawqb200.so``.

The library is the only compute path: if it is missing, importing any op
raises instead of falling back to PyTorch. Status codes follow
``include/awqb200.h``: 1/2 raise ``ValueError`` (as the reference's config and
shape checks do, ``layers/quantization/awq.py:19-23,76-85``), the rest
``RuntimeError`` (``awq_marlin.py:287-291``).
"""

from __future__ import annotations

import ctypes
import os
import threading

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libawqb200.so")

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_vp = ctypes.c_void_p
c_u32p = ctypes.POINTER(ctypes.c_uint32)
c_i64p = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes)
_SIGNATURES = {
    "awqb_last_error": (ctypes.c_char_p, []),
    "awqb_abi_version": (c_int, []),
    "awqb_blob_bytes": (c_int, [c_i64, c_i64, c_i64, c_i64p]),
    "awqb_repack": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "awqb_unrepack": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp]),
    "awqb_dequant": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_vp]),
    "awqb_gemm_workspace_bytes": (c_int, [c_i64, c_i64, c_i64, c_i64, c_i64p]),
    "awqb_gemm_workspace_bytes_ex": (c_int, [c_i64, c_i64, c_i64, c_i64, c_int, c_i64, c_i64p]),
    "awqb_gemm_plan": (c_int, [c_i64, c_i64, c_i64, c_i64, c_int, c_i64, ctypes.POINTER(c_int), c_i64p,
                               ctypes.POINTER(c_int)]),
    "awqb_gemm": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp]),
    "awqb_gemm_ex": (
        c_int,
        [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_vp, c_vp, c_i64, c_int, c_i64, c_vp],
    ),
    "awqb_gemv_ex": (
        c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp]),
    "awqb_gemm_noalloc_scratch_bytes": (c_i64, []),
    "awqb_gemm_noalloc": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_vp, c_vp]),
    "awqb_moe_topk_softmax": (c_int, [c_vp, c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_vp]),
    "awqb_moe_max_padded": (c_i64, [c_i64, c_i64, c_i64]),
    "awqb_moe_align": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp]),
    "awqb_moe_align_workspace_bytes": (c_i64, [c_i64, c_i64]),
    "awqb_moe_align_ex": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp]),
    "awqb_moe_gather_rows": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "awqb_moe_grouped_workspace_bytes": (c_int, [c_i64, c_i64, c_i64, c_i64, c_int, c_i64p]),
    "awqb_gemm_silu_mul": (c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp]),
    "awqb_moe_grouped_gemm_silu_mul": (
        c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_i64, c_vp, c_vp, c_int, c_vp, c_i64, c_vp, c_i64,
                c_vp]),
    "awqb_moe_grouped_gemm": (
        c_int,
        [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_i64, c_vp, c_vp, c_int, c_vp, c_vp, c_i64,
         c_vp, c_i64, c_vp, c_i64, c_vp],
    ),
    "awqb_silu_and_mul": (c_int, [c_vp, c_i64, c_vp, c_i64, c_int, c_vp, c_vp]),
    "awqb_silu_and_mul_interleaved": (c_int, [c_vp, c_i64, c_vp, c_i64, c_int, c_vp, c_vp]),
    "awqb_rmsnorm": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, ctypes.c_float, c_int, c_vp]),
    "awqb_fused_add_rmsnorm": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, ctypes.c_float, c_int,
                                       c_vp]),
    "awqb_moe_topk_sum": (c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_int, c_vp, c_vp]),
    "awqb_nccl_unique_id_bytes": (c_int, []),
    "awqb_nccl_get_unique_id": (c_int, [c_vp]),
    "awqb_nccl_init": (c_int, [c_vp, c_int, c_int, c_i64, ctypes.POINTER(c_vp)]),
    "awqb_nccl_symmetric_buffer": (c_int, [c_vp, ctypes.POINTER(c_vp), c_i64p]),
    "awqb_nccl_all_reduce": (c_int, [c_vp, c_vp, c_i64, c_int, c_vp]),
    "awqb_nccl_destroy": (c_int, [c_vp]),
    "awqb_tp_exchange_handle_bytes": (c_int, [c_i64p]),
    "awqb_tp_exchange_create": (c_int, [c_int, c_int, c_i64, c_i64, ctypes.POINTER(c_vp)]),
    "awqb_tp_exchange_handle": (c_int, [c_vp, c_vp]),
    "awqb_tp_exchange_open": (c_int, [c_vp, c_vp]),
    "awqb_tp_exchange_set_mode": (c_int, [c_vp, c_int]),
    "awqb_tp_exchange_destroy": (c_int, [c_vp]),
    "awqb_gemm_allreduce": (
        c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp]),
    "awqb_device_error": (c_int, [c_u32p]),
    "awqb_clear_device_error": (c_int, []),
}

EXPORTED = tuple(_SIGNATURES)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> str:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load the library once; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise RuntimeError(
                    f"{_LIB_PATH} is missing: build it with `python -m sglite_b200._build` "
                    "(there is no CPU fallback)"
                )
            # torch first, so the CUDA runtime and NCCL it loads are the ones we bind to
            import torch  # noqa: F401

            handle = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(status: int) -> None:
    if status == 0:
        return
    msg = (lib().awqb_last_error() or b"").decode(errors="replace")
    if status in (1, 2):
        raise ValueError(msg)
    raise RuntimeError(f"awqb status {status}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
