"""PyTorch-facing wrappers of the C-ABI entry points.

Tensors stay owned by PyTorch; the library only receives raw pointers and the
current CUDA stream (the reference launches on the engine stream,
``model_executor/engine.py:50-51``). Nothing here falls back to PyTorch math.
"""

from __future__ import annotations

import ctypes
import threading
from typing import Dict, Optional, Tuple

import torch

from ._lib import c_i64, call, lib

DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1}


def _p(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype not in DTYPE_CODE:
        raise ValueError(f"activation dtype {dtype} not supported (float16 or bfloat16)")
    return DTYPE_CODE[dtype]


class _DeviceGuard:
    """Makes ``device`` current for the library's CUDA runtime calls."""

    def __init__(self, device: torch.device):
        self.idx = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def _check_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError("tensors must live on a CUDA device (there is no CPU path)")
        if t.device != dev:
            raise ValueError("tensors must live on the same device")
        if not t.is_contiguous():
            raise ValueError("tensors must be contiguous")
    return dev


# ---------------------------------------------------------------- repack
def blob_bytes(K: int, N: int, G: int) -> int:
    out = c_i64(0)
    call("awqb_blob_bytes", K, N, G, ctypes.byref(out))
    return out.value


def repack(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, group_size: int) -> torch.Tensor:
    """AWQ (qweight [.., K, N/8], qzeros, scales) -> blob (uint8 [.., bytes])."""
    batched = qweight.dim() == 3
    qw = qweight if batched else qweight.unsqueeze(0)
    qz = qzeros if batched else qzeros.unsqueeze(0)
    sc = scales if batched else scales.unsqueeze(0)
    E, K, N8 = qw.shape
    N = N8 * 8
    G = K if group_size == -1 else group_size
    if qw.dtype != torch.int32 or qz.dtype != torch.int32:
        raise ValueError("qweight and qzeros must be int32")
    if sc.dtype not in DTYPE_CODE:
        raise ValueError("scales must be float16 or bfloat16")
    if qz.shape != (E, K // G, N8) or sc.shape != (E, K // G, N):
        raise ValueError(f"inconsistent AWQ shapes {tuple(qw.shape)} {tuple(qz.shape)} {tuple(sc.shape)}")
    dev = _check_cuda(qw, qz, sc)
    nb = blob_bytes(K, N, G)
    blob = torch.empty((E, nb), dtype=torch.uint8, device=dev)
    with _DeviceGuard(dev):
        call("awqb_repack", _p(qw), _p(qz), _p(sc), E, K, N, G, _p(blob), _stream(dev))
    return blob if batched else blob[0]


def unrepack(blob: torch.Tensor, K: int, N: int, G: int, scale_dtype: torch.dtype
             ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    batched = blob.dim() == 2
    b = blob if batched else blob.unsqueeze(0)
    E = b.shape[0]
    dev = _check_cuda(b)
    qw = torch.empty((E, K, N // 8), dtype=torch.int32, device=dev)
    qz = torch.empty((E, K // G, N // 8), dtype=torch.int32, device=dev)
    sc = torch.empty((E, K // G, N), dtype=scale_dtype, device=dev)
    with _DeviceGuard(dev):
        call("awqb_unrepack", _p(b), E, K, N, G, _p(qw), _p(qz), _p(sc), _stream(dev))
    if not batched:
        return qw[0], qz[0], sc[0]
    return qw, qz, sc


def dequant(blob: torch.Tensor, K: int, N: int, G: int, dtype: torch.dtype) -> torch.Tensor:
    """W = (q - z) * s in ``dtype``: [.., K, N]."""
    batched = blob.dim() == 2
    b = blob if batched else blob.unsqueeze(0)
    E = b.shape[0]
    dev = _check_cuda(b)
    w = torch.empty((E, K, N), dtype=dtype, device=dev)
    with _DeviceGuard(dev):
        call("awqb_dequant", _p(b), E, K, N, G, _dtype_code(dtype), _p(w), _stream(dev))
    return w if batched else w[0]


# ---------------------------------------------------------------- workspace
class _WorkspacePool:
    """One zero-filled scratch buffer per device, grown on demand.

    The GEMM leaves its counters at zero after every call, so the buffer is
    zeroed only when it is (re)allocated. Growing is refused while a CUDA graph
    is being captured: size it first (``reserve``) with the largest call.
    """

    def __init__(self):
        self._bufs: Dict[int, torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        buf = self._bufs.get(idx)
        if buf is not None and buf.numel() >= nbytes:
            return buf
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("AWQ GEMM workspace must be reserved before CUDA graph capture")
        with self._lock:
            buf = self._bufs.get(idx)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 20)
                if buf is not None:
                    size = max(size, 2 * buf.numel())
                buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
                self._bufs[idx] = buf
        return buf

    def reserve(self, device: torch.device, nbytes: int) -> None:
        self.get(device, nbytes)


workspace_pool = _WorkspacePool()


def gemm_workspace_bytes(M: int, K: int, N: int, G: int, ntok: int = 0, ctas: int = 0) -> int:
    out = c_i64(0)
    call("awqb_gemm_workspace_bytes_ex", M, K, N, G, ntok, ctas, ctypes.byref(out))
    return out.value


# ---------------------------------------------------------------- GEMM
def gemm(x: torch.Tensor, blob: torch.Tensor, K: int, N: int, G: int,
         bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
         ntok: int = 0, ctas: int = 0, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y[..., N] = x[..., K] @ dequant(blob) (+ bias), fp32 accumulation."""
    if x.shape[-1] != K:
        raise ValueError(f"x has {x.shape[-1]} features, expected K={K}")
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    M = x2.shape[0]
    code = _dtype_code(x.dtype)
    dev = _check_cuda(x2, blob)
    if bias is not None:
        _check_cuda(bias)
        if bias.dtype != x.dtype or bias.numel() != N:
            raise ValueError("bias must be [N] in the activation dtype")
    if out is None:
        out = torch.empty((M, N), dtype=x.dtype, device=dev)
    elif out.shape[-1] != N or out.numel() != M * N or out.dtype != x.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous [M, N] tensor of the activation dtype")
    if M == 0:
        return out.reshape(*x.shape[:-1], N)
    nbytes = gemm_workspace_bytes(M, K, N, G, ntok, ctas)
    ws = workspace if workspace is not None else workspace_pool.get(dev, nbytes)
    with _DeviceGuard(dev):
        call("awqb_gemm_ex", _p(x2), M, K, N, G, code, _p(blob), _p(bias), _p(out), _p(ws),
             ws.numel(), ntok, ctas, _stream(dev))
    return out.reshape(*x.shape[:-1], N)


def device_error(clear: bool = True) -> int:
    """Bits set by kernels whose bounded waits gave up (synchronises)."""
    v = ctypes.c_uint32(0)
    call("awqb_device_error", ctypes.byref(v))
    if clear and v.value:
        call("awqb_clear_device_error")
    return v.value


def abi_version() -> int:
    return lib().awqb_abi_version()
