"""AWQ mixture-of-experts backend on the sm_100a kernels.

Same pipeline and interface as the reference's ``FusedMoe``
(``layers/fused_moe/fused.py:205-233``, ``fused_experts_impl`` ``:101-202``):
router softmax + top-k, expert sort padded to the block size, expert GEMM on
``w1`` (gate|up), SiLU-and-mul, expert GEMM on ``w2`` with the router weight
applied to its output, top-k sum written into ``hidden_states`` in place. The
expert weights are AWQ int4 (stacked ``[E, K, N/8]`` as the loader stacks them,
``model_loader/weight_loader.py:134-142``) instead of dense, and a rank may own
only the experts ``[e_begin, e_end)`` (expert parallelism; the caller then
all-reduces the output across ranks as ``MoELayer.forward`` does for TP,
``layers/moe_layer.py:62-63``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import ops

try:  # pragma: no cover - depends on the host environment
    from sglite.srt.model_executor.layers.fused_moe.base import BaseMoeBackend  # type: ignore
except Exception:
    from abc import ABC, abstractmethod

    class BaseMoeBackend(ABC):  # type: ignore[no-redef]
        """Base class for MoE backends (layers/fused_moe/base.py:8-24)."""

        @abstractmethod
        def forward(self, hidden_states, w1, w2, gating_output, topk, renormalize, activation,
                    apply_router_weight_on_input):
            ...


@dataclass
class AWQExpertWeights:
    """Repacked AWQ weights of a rank's experts for one projection."""

    blob: torch.Tensor           # uint8 [E_local, blob_bytes]
    K: int                       # input features
    N: int                       # output features
    G: int                       # group size
    act_dtype: torch.dtype
    e_begin: int = 0             # first global expert id held here
    num_global_experts: Optional[int] = None
    gate_up_interleaved: bool = False  # w1 columns interleaved gate j, up j (fused SiLU-and-mul)

    @property
    def num_experts(self) -> int:
        return self.blob.shape[0]

    @property
    def e_end(self) -> int:
        return self.e_begin + self.num_experts

    @classmethod
    def from_awq(cls, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, group_size: int,
                 e_begin: int = 0, num_global_experts: Optional[int] = None,
                 gate_up: bool = False) -> "AWQExpertWeights":
        """qweight [E, K, N/8] int32, qzeros [E, K/G, N/8] int32, scales [E, K/G, N] (device tensors).
        gate_up=True for the merged gate_up projection (w1): its columns are
        interleaved at load so the GEMM can apply SiLU-and-mul in its epilogue
        (needs the intermediate size to be a multiple of 8; otherwise the plain
        layout is kept and SiLU-and-mul runs as its own kernel)."""
        E, K, N8 = qweight.shape
        G = K if group_size == -1 else group_size
        inter = gate_up and (N8 * 8) % 16 == 0
        if inter:
            qweight, qzeros, scales = ops.interleave_gate_up(qweight, qzeros, scales)
        blob = ops.repack(qweight.contiguous(), qzeros.contiguous(), scales.contiguous(), G)
        return cls(blob, K, N8 * 8, G, scales.dtype, e_begin, num_global_experts, inter)


def choose_block_m(num_tokens: int, topk: int, num_experts: int) -> int:
    """Rows per expert block (the grouped GEMM's token tile), from the mean
    number of rows per expert. Measured on B200 (Qwen3-30B-A3B experts): a
    block of about twice the mean is fastest up to 64 (routed counts scatter
    around the mean, and an expert split over two blocks is dequantised
    twice); means of 8 / 16 / 32 / 64 rows -> blocks of 16 / 32 / 64 / 64;
    128 above."""
    mean = (num_tokens * topk + num_experts - 1) // max(1, num_experts)
    if mean <= 8:
        return 16
    if mean <= 16:
        return 32
    if mean <= 64:
        return 64
    return 128


class AWQB200MoeBackend(BaseMoeBackend):
    """MoE backend over AWQ int4 experts (registered as "awq_b200")."""

    def forward(self, hidden_states: torch.Tensor, w1: AWQExpertWeights, w2: AWQExpertWeights,
                gating_output: torch.Tensor, topk: int, renormalize: bool, activation: str = "silu",
                apply_router_weight_on_input: bool = False) -> torch.Tensor:
        if activation != "silu":
            raise ValueError(f"activation {activation!r} not supported by the AWQ B200 MoE backend")
        if apply_router_weight_on_input:
            raise ValueError("router weights are applied to the down-projection output only")
        topk_weights, topk_ids = ops.moe_topk_softmax(gating_output, topk, renormalize)
        return self.experts(hidden_states, w1, w2, topk_weights, topk_ids)

    def experts(self, hidden_states: torch.Tensor, w1: AWQExpertWeights, w2: AWQExpertWeights,
                topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
        x = hidden_states
        if not x.is_contiguous():
            raise ValueError("hidden_states must be contiguous")
        if x.dtype != w1.act_dtype or x.dtype != w2.act_dtype:
            raise ValueError("hidden_states dtype differs from the experts' scale dtype")
        M, H = x.shape
        topk = topk_ids.shape[1]
        if w1.K != H or w2.N != H or w1.N != 2 * w2.K:
            raise ValueError("expert shapes do not match: w1 [E, H, 2I], w2 [E, I, H]")
        if w1.e_begin != w2.e_begin or w1.num_experts != w2.num_experts:
            raise ValueError("w1 and w2 hold different experts")
        E_glob = w1.num_global_experts or w1.num_experts
        numel = M * topk
        block_m = choose_block_m(M, topk, E_glob)
        sorted_ids, block_expert, npp = ops.moe_align(topk_ids, w1.e_begin, w1.e_end, block_m)
        rows = sorted_ids.numel()
        xs = ops.moe_gather_rows(x, sorted_ids, npp, topk, numel)
        if w1.gate_up_interleaved and block_m <= ops.SILU_FUSE_MAX_M:
            # gate_up GEMM with SiLU-and-mul in its epilogue (measured faster for
            # small expert blocks; above, the separate kernel wins)
            a = torch.empty((rows, w1.N // 2), dtype=x.dtype, device=x.device)
            ops.moe_grouped_gemm_silu_mul(xs, w1.blob, w1.K, w1.N, w1.G, block_expert, npp, block_m, a)
        else:
            h1 = torch.empty((rows, w1.N), dtype=x.dtype, device=x.device)
            ops.moe_grouped_gemm(xs, w1.blob, w1.K, w1.N, w1.G, block_expert, npp, block_m, h1)
            a = ops.silu_and_mul(h1, rows_dev=npp, interleaved=w1.gate_up_interleaved)
        y3 = torch.empty((numel, H), dtype=x.dtype, device=x.device)
        ops.moe_grouped_gemm(a, w2.blob, w2.K, w2.N, w2.G, block_expert, npp, block_m, y3,
                             row_map=sorted_ids, row_scale=topk_weights.reshape(-1).contiguous(), num_valid=numel)
        ids = topk_ids if (w1.e_begin != 0 or w1.e_end != E_glob) else None
        ops.moe_topk_sum(y3, M, topk, ids, w1.e_begin, w1.e_end, hidden_states)
        return hidden_states


def route(gating_output: torch.Tensor, topk: int, renormalize: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    return ops.moe_topk_softmax(gating_output, topk, renormalize)
