"""RMSNorm layers over the library's kernels, with the interface of the
reference's ``srt/model_executor/layers/norm.py:10-47`` (``RMSNorm``,
``RMSNormFused``). After a row-parallel projection whose all-reduce is fused
into the GEMM (``distributed.PeerExchange.gemm_allreduce``), the residual add
and the norm run as one more kernel, launched so that it overlaps the GEMM's
tail (programmatic dependent launch)."""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import ops


class RMSNorm:
    """RMSNorm over the last dimension (``norm.py:10-25``)."""

    def __init__(self, size: int, eps: float) -> None:
        self.eps = eps
        self.weight = torch.empty(size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rmsnorm(x, self.weight, self.eps)

    def forward_inplace(self, x: torch.Tensor) -> None:
        ops.rmsnorm(x, self.weight, self.eps, out=x)


class RMSNormFused:
    """RMSNorm with the residual add fused in (``norm.py:28-47``)."""

    def __init__(self, size: int, eps: float) -> None:
        self.eps = eps
        self.weight = torch.empty(size)

    def forward(self, x: torch.Tensor,
                residual: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Without a residual: (rmsnorm(x), x). With one: residual += x and
        x = rmsnorm(residual), both in place; returns (x, residual)."""
        if residual is None:
            return ops.rmsnorm(x, self.weight, self.eps), x
        ops.fused_add_rmsnorm(x, residual, self.weight, self.eps)
        return x, residual
