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

import re
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

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


# ---------------------------------------------------------------------------
# AWQ MoE layer wiring: the checkpoint tensors of the experts, their loading
# and the forward of the reference's MoELayer (layers/moe_layer.py:12-63) for
# AWQ experts.

AWQ_SUFFIXES = (".qweight", ".qzeros", ".scales")
_EXPERT_KEY = re.compile(r"^(?P<prefix>.+\.experts)\.(?P<idx>\d+)\.(?P<name>.+)$")


def shard_expert_tensor(key: str, value: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank ``rank``'s shard of one AWQ expert tensor, as the reference loader
    cuts it (model_loader/weight_loader.py:40-69): gate / up projections split
    their packed output columns (dim 1), the down projection its input rows
    (dim 0, and the K/G rows of qzeros / scales)."""
    if world == 1:
        return value
    if ".gate_proj" in key or ".up_proj" in key:
        return value.chunk(world, dim=1)[rank].contiguous()
    if ".down_proj" in key:
        return value.chunk(world, dim=0)[rank].contiguous()
    return value


def stack_awq_experts(tensors: Dict[str, torch.Tensor], num_experts: int, rank: int = 0,
                      world: int = 1) -> Dict[str, torch.Tensor]:
    """Checkpoint AWQ expert tensors -> the loader's packed runtime tensors.

    Restates model_loader/weight_loader.py:121-142 for AWQ experts: each
    ``<prefix>.experts.<e>.{gate,up,down}_proj.{qweight,qzeros,scales}`` is
    sharded for this rank, gate and up are concatenated on the packed column
    dimension into ``gate_up_proj`` (``[gate_r | up_r]``), and the experts are
    stacked on a new leading dimension: ``<prefix>.experts.gate_up_proj.qweight``
    ``[E, H, 2 I / tp / 8]``, ``<prefix>.experts.down_proj.qweight``
    ``[E, I / tp, H / 8]`` (and likewise qzeros / scales). Tensors that are not
    expert tensors pass through unchanged."""
    out: Dict[str, torch.Tensor] = {}
    slots: Dict[str, Dict[int, Dict[str, torch.Tensor]]] = {}
    for key, value in tensors.items():
        m = _EXPERT_KEY.match(key)
        if m is None or not key.endswith(AWQ_SUFFIXES):
            out[key] = value
            continue
        name = m.group("name")  # e.g. gate_proj.qweight
        proj, suffix = name.rsplit(".", 1)
        t = shard_expert_tensor(key, value, rank, world)
        merged = "gate_up_proj" if proj in ("gate_proj", "up_proj") else proj
        per = slots.setdefault(f"{m.group('prefix')}.{merged}.{suffix}", {}).setdefault(int(m.group("idx")), {})
        per[proj] = t
    for packed, experts in slots.items():
        if sorted(experts) != list(range(num_experts)):
            raise ValueError(f"{packed}: expected experts 0..{num_experts - 1}, got {sorted(experts)}")
        parts = []
        for e in range(num_experts):
            d = experts[e]
            if "gate_up_proj" in packed:
                if set(d) != {"gate_proj", "up_proj"}:
                    raise ValueError(f"{packed}: expert {e} needs both gate_proj and up_proj")
                parts.append(torch.cat([d["gate_proj"], d["up_proj"]], dim=1))
            else:
                (t,) = d.values()
                parts.append(t)
        out[packed] = torch.stack(parts, dim=0)
    return out


class AWQB200MoEMethod:
    """Weight method of an AWQ MoE layer: the expert counterpart of the linear
    method's create_weights / process_weights_after_loading / apply
    (layers/quantization/base_config.py:22-42)."""

    def __init__(self, quant_config):
        self.quant_config = quant_config

    def _group(self, k: int) -> int:
        return k if self.quant_config.group_size == -1 else self.quant_config.group_size

    def create_weights(self, num_experts: int, hidden_size: int, intermediate_size_per_partition: int,
                       params_dtype: torch.dtype = torch.bfloat16) -> Dict[str, Dict[str, torch.Tensor]]:
        """Empty expert stacks with the loader's shapes: gate_up_proj
        [E, H, 2 I / 8] (qzeros [E, H / G, 2 I / 8], scales [E, H / G, 2 I]) and
        down_proj [E, I, H / 8] (qzeros [E, I / G, H / 8], scales [E, I / G, H])."""
        E, H, I = num_experts, hidden_size, intermediate_size_per_partition
        pf = self.quant_config.pack_factor
        G1, G2 = self._group(H), self._group(I)
        if H % G1 or I % G2:
            raise ValueError(f"hidden {H} / intermediate {I} not aligned with the group size")
        if (2 * I) % pf or H % pf:
            raise ValueError("output sizes must be multiples of the pack factor")

        def stack(k, n, G):
            return {"qweight": torch.empty(E, k, n // pf, dtype=torch.int32),
                    "qzeros": torch.empty(E, k // G, n // pf, dtype=torch.int32),
                    "scales": torch.empty(E, k // G, n, dtype=params_dtype)}

        return {"gate_up_proj": stack(H, 2 * I, G1), "down_proj": stack(I, H, G2)}

    def process_weights_after_loading(self, weights: Dict[str, Dict[str, torch.Tensor]], e_begin: int = 0,
                                      num_global_experts: Optional[int] = None
                                      ) -> Tuple[AWQExpertWeights, AWQExpertWeights]:
        """Repack the loaded stacks on the GPU (gate_up with its columns
        interleaved for the fused SiLU-and-mul epilogue)."""
        g, d = weights["gate_up_proj"], weights["down_proj"]
        H = g["qweight"].shape[1]
        I = d["qweight"].shape[1]
        w1 = AWQExpertWeights.from_awq(g["qweight"], g["qzeros"], g["scales"], self._group(H), e_begin,
                                       num_global_experts, gate_up=True)
        w2 = AWQExpertWeights.from_awq(d["qweight"], d["qzeros"], d["scales"], self._group(I), e_begin,
                                       num_global_experts)
        return w1, w2


class _AWQTensors:
    """qweight / qzeros / scales of one expert projection (a state-dict node)."""

    def __init__(self, tensors: Dict[str, torch.Tensor]):
        self.qweight = tensors["qweight"]
        self.qzeros = tensors["qzeros"]
        self.scales = tensors["scales"]

    def as_dict(self) -> Dict[str, torch.Tensor]:
        return {"qweight": self.qweight, "qzeros": self.qzeros, "scales": self.scales}


class AWQMoELayer:
    """The reference's MoELayer (layers/moe_layer.py:12-63) over AWQ experts.

    State-dict keys are those the reference loader produces for AWQ MoE
    checkpoints: ``gate_up_proj.{qweight,qzeros,scales}`` and
    ``down_proj.{...}`` under the layer's prefix (e.g.
    ``model.layers.0.mlp.experts``), with the intermediate size already split
    for tensor parallelism by the loader. With expert parallelism
    (``ep_size > 1``) the layer keeps only its experts
    ``[ep_rank * E / ep_size, (ep_rank + 1) * E / ep_size)`` at load; every
    rank computes its experts' weighted outputs for all tokens, and the partial
    outputs are all-reduced, as ``MoELayer.forward`` does for TP
    (moe_layer.py:62-63)."""

    def __init__(self, num_experts: int, top_k: int, hidden_size: int, intermediate_size: int, quant_config,
                 renormalize: bool = True, activation: str = "silu", apply_router_weight_on_input: bool = False,
                 tp_size: int = 1, ep_rank: int = 0, ep_size: int = 1, comm=None):
        if num_experts % ep_size:
            raise ValueError(f"{num_experts} experts do not split over {ep_size} ranks")
        if intermediate_size % tp_size:
            raise ValueError(f"intermediate size {intermediate_size} does not split over {tp_size} ranks")
        self.num_experts = num_experts
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.renormalize = renormalize
        self.activation = activation
        self.apply_router_weight_on_input = apply_router_weight_on_input
        self._tp_size, self._ep_size = tp_size, ep_size
        self._e_begin = ep_rank * (num_experts // ep_size)
        self._e_local = num_experts // ep_size
        self._comm = comm
        self._method = AWQB200MoEMethod(quant_config)
        w = self._method.create_weights(num_experts, hidden_size, intermediate_size // tp_size)
        self.gate_up_proj = _AWQTensors(w["gate_up_proj"])
        self.down_proj = _AWQTensors(w["down_proj"])
        self._w1: Optional[AWQExpertWeights] = None
        self._w2: Optional[AWQExpertWeights] = None
        self._backend = AWQB200MoeBackend()

    # state dict with the semantics of layers/base.py:18-62
    def state_dict(self, *, prefix: str = "", result=None) -> Dict[str, torch.Tensor]:
        result = result if result is not None else {}
        for proj in ("gate_up_proj", "down_proj"):
            for k, v in getattr(self, proj).as_dict().items():
                result[f"{prefix}.{proj}.{k}" if prefix else f"{proj}.{k}"] = v
        return result

    def load_state_dict(self, state_dict: Dict[str, torch.Tensor], *, prefix: str = "",
                        _internal: bool = False) -> None:
        for proj in ("gate_up_proj", "down_proj"):
            node = getattr(self, proj)
            for k in ("qweight", "qzeros", "scales"):
                key = f"{prefix}.{proj}.{k}" if prefix else f"{proj}.{k}"
                item = state_dict.pop(key)
                cur = getattr(node, k)
                if tuple(item.shape) != tuple(cur.shape) or item.dtype != cur.dtype:
                    raise ValueError(f"{key}: got {tuple(item.shape)} {item.dtype}, "
                                     f"expected {tuple(cur.shape)} {cur.dtype}")
                setattr(node, k, item)
        if not _internal and state_dict:
            raise RuntimeError(f"Unexpected keys in state_dict: {list(state_dict.keys())}")

    def process_weights_after_loading(self) -> None:
        """Keep this rank's experts and repack them (once, on the GPU)."""
        lo, hi = self._e_begin, self._e_begin + self._e_local
        local = {p: {k: v[lo:hi].contiguous() for k, v in getattr(self, p).as_dict().items()}
                 for p in ("gate_up_proj", "down_proj")}
        self._w1, self._w2 = self._method.process_weights_after_loading(local, lo, self.num_experts)
        empty = {k: v[:0] for k, v in self.gate_up_proj.as_dict().items()}
        self.gate_up_proj = _AWQTensors(empty)  # the blobs replace the checkpoint tensors
        self.down_proj = _AWQTensors({k: v[:0] for k, v in self.down_proj.as_dict().items()})

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        if self._w1 is None:
            raise RuntimeError("process_weights_after_loading must run before forward")
        out = self._backend.forward(hidden_states=hidden_states.contiguous(), w1=self._w1, w2=self._w2,
                                    gating_output=router_logits, topk=self.top_k, renormalize=self.renormalize,
                                    activation=self.activation,
                                    apply_router_weight_on_input=self.apply_router_weight_on_input)
        if (self._tp_size > 1 or self._ep_size > 1) and self._comm is not None:
            out = self._comm.all_reduce(out)
        return out
