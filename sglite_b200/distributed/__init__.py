"""Tensor-parallel communication for the row-parallel projections.

Two paths: NCCL (``init_nccl``, any size) and, for decode-sized M, the GEMM fused
with its all-reduce over peer memory (``init_peer_exchange``).

``init_nccl`` follows the reference's ``init_pynccl`` (kernels/pynccl.py:50-83):
rank 0 creates the NCCL unique id, the id travels over the CPU (gloo) process
group with ``broadcast_object_list``, and every rank builds its communicator
through the C-ABI. ``NcclCommunicator.all_reduce`` is the in-place SUM of
``PyNCCLCommunicator.all_reduce`` (communicator.py:62-65, pynccl.cu:96-138).
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from .._lib import c_i64, call, lib
from ..ops import DTYPE_CODE, _DeviceGuard, _p, _stream


class NcclCommunicator:
    def __init__(self, rank: int, world: int, uid: bytes, device: torch.device, max_size_bytes: int = 0):
        self.rank = rank
        self.world = world
        self.device = device
        self._comm = ctypes.c_void_p(0)
        buf = ctypes.create_string_buffer(uid, len(uid))
        with _DeviceGuard(device):
            call("awqb_nccl_init", buf, rank, world, max_size_bytes, ctypes.byref(self._comm))

    def all_reduce(self, x: torch.Tensor, op: str = "sum") -> torch.Tensor:
        """In-place SUM over the group; returns ``x``."""
        if op != "sum":
            raise ValueError(f"only sum is supported, got {op!r}")
        if x.dtype not in DTYPE_CODE:
            raise ValueError(f"all-reduce supports float16/bfloat16, got {x.dtype}")
        if not x.is_contiguous():
            raise ValueError("all-reduce needs a contiguous tensor")
        with _DeviceGuard(x.device):
            call("awqb_nccl_all_reduce", self._comm, _p(x), x.numel(), DTYPE_CODE[x.dtype], _stream(x.device))
        return x

    def symmetric_buffer(self) -> Optional[torch.Tensor]:
        """The registered symmetric buffer as a uint8 tensor view (or None)."""
        ptr = ctypes.c_void_p(0)
        nbytes = c_i64(0)
        call("awqb_nccl_symmetric_buffer", self._comm, ctypes.byref(ptr), ctypes.byref(nbytes))
        if not ptr.value or nbytes.value == 0:
            return None
        return _wrap_device_ptr(ptr.value, nbytes.value, self.device)

    def destroy(self) -> None:
        if self._comm.value:
            with _DeviceGuard(self.device):
                call("awqb_nccl_destroy", self._comm)
            self._comm = ctypes.c_void_p(0)


def _wrap_device_ptr(ptr: int, nbytes: int, device: torch.device) -> torch.Tensor:
    class _Holder:
        __cuda_array_interface__ = {
            "shape": (nbytes,),
            "typestr": "|u1",
            "data": (ptr, False),
            "version": 3,
            "strides": None,
        }

    with torch.cuda.device(device):
        return torch.as_tensor(_Holder(), device=device)


def get_unique_id() -> bytes:
    n = lib().awqb_nccl_unique_id_bytes()
    buf = ctypes.create_string_buffer(n)
    call("awqb_nccl_get_unique_id", buf)
    return buf.raw


def init_nccl(*, tp_rank: int, tp_size: int, tp_cpu_group, device: torch.device,
              max_size_bytes: int = 0) -> NcclCommunicator:
    """Create the TP communicator; the unique id goes over the CPU group."""
    import torch.distributed as dist

    ids = [get_unique_id() if tp_rank == 0 else None]
    dist.broadcast_object_list(ids, src=0, group=tp_cpu_group)
    if ids[0] is None:
        raise RuntimeError(f"Failed to get NCCL unique ID on tp_rank={tp_rank}")
    return NcclCommunicator(tp_rank, tp_size, ids[0], device, max_size_bytes)


class PeerExchange:
    """Fused row-parallel GEMM + all-reduce over peer memory (one per TP rank).

    Replaces, for M <= ``max_rows``, the reference's row-parallel pair: the
    quantised GEMM followed by ``PyNCCLCommunicator.all_reduce``
    (layers/linear.py:189-194, pynccl.cu:96-138). Every rank must call
    ``gemm_allreduce`` in the same order with the same shapes.
    """

    def __init__(self, rank: int, world: int, device: torch.device, max_rows: int, max_n: int):
        self.rank, self.world, self.device = rank, world, device
        self.max_rows, self.max_n = max_rows, max_n
        self._ctx = ctypes.c_void_p(0)
        with _DeviceGuard(device):
            call("awqb_tp_exchange_create", rank, world, max_rows, max_n, ctypes.byref(self._ctx))

    def handle(self) -> bytes:
        n = c_i64(0)
        call("awqb_tp_exchange_handle_bytes", ctypes.byref(n))
        buf = ctypes.create_string_buffer(n.value)
        call("awqb_tp_exchange_handle", self._ctx, buf)
        return buf.raw

    def open(self, handles) -> None:
        blob = b"".join(handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        with _DeviceGuard(self.device):
            call("awqb_tp_exchange_open", self._ctx, buf)

    MODES = {"auto": 0, "all_to_all": 1, "reduce_scatter": 2}

    def set_mode(self, mode: str) -> None:
        """Exchange pattern: "auto", "all_to_all" or "reduce_scatter" (same on
        every rank; results are bit-identical across patterns)."""
        if mode not in self.MODES:
            raise ValueError(f"mode must be one of {sorted(self.MODES)}")
        call("awqb_tp_exchange_set_mode", self._ctx, self.MODES[mode])

    def gemm_allreduce(self, x: torch.Tensor, blob: torch.Tensor, K: int, N: int, G: int,
                       bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y[..., N] = sum over ranks of x_r[..., K] @ dequant(blob_r) (+ bias), on every rank."""
        from ..ops import _check_cuda, _dtype_code, gemm_workspace_bytes, workspace_pool

        if x.shape[-1] != K:
            raise ValueError(f"x has {x.shape[-1]} features, expected K={K}")
        x2 = x.reshape(-1, K)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        M = x2.shape[0]
        if M > self.max_rows or N > self.max_n:
            raise ValueError(f"exchange sized for M <= {self.max_rows}, N <= {self.max_n}")
        code = _dtype_code(x.dtype)
        dev = _check_cuda(x2, blob)
        if bias is not None and (bias.dtype != x.dtype or bias.numel() != N):
            raise ValueError("bias must be [N] in the activation dtype")
        if out is None:
            out = torch.empty((M, N), dtype=x.dtype, device=dev)
        elif out.numel() != M * N or out.dtype != x.dtype or not out.is_contiguous():
            raise ValueError("out must be a contiguous [M, N] tensor of the activation dtype")
        if M == 0:
            return out.reshape(*x.shape[:-1], N)
        ws = workspace_pool.get(dev, gemm_workspace_bytes(M, K, N, G))
        with _DeviceGuard(dev):
            call("awqb_gemm_allreduce", _p(x2), M, K, N, G, code, _p(blob), _p(bias), _p(out), _p(ws),
                 ws.numel(), self._ctx, _stream(dev))
        return out.reshape(*x.shape[:-1], N)

    def destroy(self) -> None:
        if self._ctx.value:
            with _DeviceGuard(self.device):
                call("awqb_tp_exchange_destroy", self._ctx)
            self._ctx = ctypes.c_void_p(0)


def init_peer_exchange(*, tp_rank: int, tp_size: int, tp_cpu_group, device: torch.device,
                       max_rows: int = 64, max_n: int = 8192) -> PeerExchange:
    """Create the exchange on every rank and map the peers' buffers (handles
    travel over the CPU group)."""
    import torch.distributed as dist

    ex = PeerExchange(tp_rank, tp_size, device, max_rows, max_n)
    handles = [None] * tp_size
    if tp_size > 1:
        dist.all_gather_object(handles, ex.handle(), group=tp_cpu_group)
    else:
        handles = [ex.handle()]
    ex.open(handles)
    return ex


__all__ = ["NcclCommunicator", "PeerExchange", "get_unique_id", "init_nccl", "init_peer_exchange"]
