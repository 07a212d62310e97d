"""CPU oracle for RMSNorm and residual-add RMSNorm -- TEST INFRASTRUCTURE ONLY
(imported by ``tests/`` as the checker, never by the product path).

The reference (``srt/model_executor/layers/norm.py:10-47``) calls
``flashinfer.rmsnorm`` and ``flashinfer.fused_add_rmsnorm`` (third-party,
flashinfer 0.6.11.post2, ``include/flashinfer/norm.cuh``, kernels ``RMSNormKernel``
and ``FusedAddRMSNormKernel``). Their published arithmetic, restated per row:

    x        = float(input) + float(residual)          (fp32; no residual: x = float(input))
    residual = x rounded to the dtype                  (fused only)
    out      = x * rsqrt(sum(x * x) / d + eps) * float(weight), rounded to the dtype

with the sum of squares over the unrounded fp32 x. The order of that sum is an
implementation detail of each kernel, so the normalised output is compared
within a tolerance; the rounded residual is exact.

Pinned against flashinfer 0.6.11.post2 itself (installed on the GPU image):
``tests/test_gpu_norm.py::test_norm_matches_flashinfer_and_pins_the_oracle``
runs its two kernels on the same inputs and checks this restatement against
them (residual bit-identical, outputs within 8e-3 of max|ref|).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch


def rmsnorm_ref(x: torch.Tensor, weight: torch.Tensor, eps: float,
                residual: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Returns (out, new_residual) on the CPU; new_residual is None without a residual."""
    xf = x.detach().cpu().float()
    new_res = None
    if residual is not None:
        xf = xf + residual.detach().cpu().float()
        new_res = xf.to(x.dtype)
    inv = torch.rsqrt(xf.pow(2).sum(-1, keepdim=True) / xf.shape[-1] + eps)
    out = (xf * inv * weight.detach().cpu().float()).to(x.dtype)
    return out, new_res
