"""Tensor-parallel AWQ projections.

Sharding follows the reference's loader for AWQ tensors
(``model_loader/weight_loader.py:40-69,121-132``): column-parallel projections
(q/k/v, gate/up) split the packed output dimension (dim 1 of qweight, qzeros
and scales), row-parallel ones (o, down) split the input dimension (dim 0, and
K/G rows of qzeros / scales), and fused projections concatenate the per-slot
shards along dim 1. Local sizes follow ``layers/linear.py:127-194``; the row
parallel output is all-reduced (``RowParallelLinear.forward``, ``:189-194``).
"""

from __future__ import annotations

from typing import Dict, List, Optional

import torch

from .quantization.awq_b200 import AWQB200LinearMethod

AWQ_KEYS = ("qweight", "qzeros", "scales")


def div_even(a: int, b: int, allow_replicate: bool = False) -> int:
    """utils/misc.py:6-12."""
    if allow_replicate and b > a:
        if b % a:
            raise ValueError(f"{b} must be divisible by {a} for replication")
        return 1
    if a % b:
        raise ValueError(f"{a} must be divisible by {b}")
    return a // b


def shard_awq(tensors: Dict[str, torch.Tensor], parallel: str, rank: int, world: int) -> Dict[str, torch.Tensor]:
    """Rank ``rank``'s shard of one AWQ projection: parallel = "column" | "row"."""
    if parallel not in ("column", "row"):
        raise ValueError(parallel)
    dim = 1 if parallel == "column" else 0
    out = {}
    for k in AWQ_KEYS:
        t = tensors[k]
        if t.shape[dim] % world:
            raise ValueError(f"{k} dim {dim} ({t.shape[dim]}) is not divisible by tp={world}")
        out[k] = t.chunk(world, dim=dim)[rank].contiguous()
    return out


def merge_awq(parts: List[Dict[str, torch.Tensor]]) -> Dict[str, torch.Tensor]:
    """Fused projection (qkv / gate_up): concatenate the slots on dim 1."""
    return {k: torch.cat([p[k] for p in parts], dim=1) for k in AWQ_KEYS}


def qkv_local_size(num_qo_heads: int, num_kv_heads: int, head_dim: int, tp: int) -> int:
    return (div_even(num_qo_heads, tp) + 2 * div_even(num_kv_heads, tp, allow_replicate=True)) * head_dim


class _AWQLinear:
    """A projection holding this rank's AWQ weights behind the linear method."""

    def __init__(self, method: AWQB200LinearMethod, local_in: int, local_out: int,
                 bias: Optional[torch.Tensor] = None):
        self.method = method
        self.weights = method.create_weights(local_in, local_out)
        self.local_input_size = local_in
        self.local_output_size = local_out
        self.bias = bias

    def load(self, shard: Dict[str, torch.Tensor]) -> None:
        for k in AWQ_KEYS:
            if tuple(shard[k].shape) != tuple(self.weights[k].shape):
                raise ValueError(f"{k}: shard {tuple(shard[k].shape)} != expected {tuple(self.weights[k].shape)}")
            self.weights[k] = shard[k]
        self.weights = self.method.process_weights_after_loading(self.weights)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.method.apply_weights(self.weights, x, self.bias)


class ColumnParallelAWQLinear(_AWQLinear):
    """QKV / merged gate_up: output features split across ranks, no collective."""

    def __init__(self, method, input_size: int, local_output_size: int, bias=None):
        super().__init__(method, input_size, local_output_size, bias)


class RowParallelAWQLinear(_AWQLinear):
    """O / down: input features split across ranks, output all-reduced
    (``RowParallelLinear.forward``, layers/linear.py:189-194).

    With a ``PeerExchange`` and no bias, decode-sized batches (M <= its
    max_rows) run the GEMM fused with the all-reduce in one kernel over peer
    memory; otherwise the GEMM is followed by the NCCL all-reduce. (The
    reference adds the bias on every rank before reducing; that case keeps the
    NCCL path so the semantics stay identical.)"""

    def __init__(self, method, input_size: int, output_size: int, tp_size: int, comm=None, bias=None,
                 exchange=None):
        super().__init__(method, div_even(input_size, tp_size), output_size, bias)
        self.tp_size = tp_size
        self.comm = comm
        self.exchange = exchange

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp_size > 1 and self.exchange is not None and self.bias is None:
            M = x.numel() // self.local_input_size
            if M <= self.exchange.max_rows and self.local_output_size <= self.exchange.max_n:
                w = self.weights
                if x.dtype != w["_act_dtype"]:
                    raise ValueError(f"activations are {x.dtype}, weights were loaded for {w['_act_dtype']}")
                return self.exchange.gemm_allreduce(x, w["qweight"], self.local_input_size,
                                                    self.local_output_size, w["_group_size"])
        y = super().forward(x)
        if self.tp_size > 1:
            y = self.comm.all_reduce(y)
        return y
