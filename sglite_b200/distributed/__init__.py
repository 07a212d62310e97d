"""Tensor-parallel communication for the row-parallel projections.

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


__all__ = ["NcclCommunicator", "get_unique_id", "init_nccl"]
