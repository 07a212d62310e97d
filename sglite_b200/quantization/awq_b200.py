"""AWQ quantization config and linear method backed by the sm_100a kernels.

Same weight interface as the reference's AWQ methods: ``create_weights``
allocates the checkpoint tensors ``qweight`` / ``qzeros`` / ``scales`` with the
loader attributes of ``layers/quantization/awq.py:87-124``;
``process_weights_after_loading`` repacks them once on the GPU (the role of
``AWQMarlinLinearMethod.process_weights_after_loading``, ``awq_marlin.py:270-334``);
``apply_weights`` runs the W4A16 GEMM (``awq.py:126-147``).
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional

import torch
from torch.nn.parameter import Parameter

from .. import ops
from .base_config import LinearMethodBase, QuantizationConfig, set_weight_attrs

SUPPORTED_GROUP_SIZES = (-1, 32, 64, 128)
# decode batches are captured in CUDA graphs up to this many tokens
# (model_executor/cuda_graph.py:76); their GEMM workspace is reserved at load
GRAPH_MAX_TOKENS = 256


def _kernel_group_ok(G: int) -> bool:
    return G in (32, 64) or (G >= 128 and G % 128 == 0)


class AWQB200Config(QuantizationConfig):
    """Config for AWQ int4 weights (group-wise zero point and scale) on B200."""

    def __init__(self, weight_bits: int, group_size: int, zero_point: bool) -> None:
        self.weight_bits = weight_bits
        self.group_size = group_size
        self.zero_point = zero_point
        if self.weight_bits != 4:
            raise ValueError(
                f"Currently, only 4-bit weight quantization is supported for AWQ, "
                f"but got {self.weight_bits} bits."
            )
        if group_size not in SUPPORTED_GROUP_SIZES and not (group_size > 0 and group_size % 128 == 0):
            raise ValueError(f"AWQ B200 does not support group_size={group_size}; "
                             f"use one of {SUPPORTED_GROUP_SIZES} or a multiple of 128.")
        if not zero_point:
            raise ValueError("AWQ B200 requires zero_point=True (asymmetric AWQ checkpoints).")
        self.pack_factor = 32 // self.weight_bits

    def __repr__(self) -> str:
        return (f"AWQB200Config(weight_bits={self.weight_bits}, group_size={self.group_size}, "
                f"zero_point={self.zero_point})")

    def get_name(self) -> str:
        return "awq_b200"

    def get_supported_act_dtypes(self) -> List[torch.dtype]:
        return [torch.half, torch.bfloat16]

    def get_min_capability(self) -> int:
        return 100

    @staticmethod
    def get_config_filenames() -> List[str]:
        return ["quant_config.json", "quantize_config.json"]

    @classmethod
    def from_config(cls, config: Dict[str, Any]) -> "AWQB200Config":
        weight_bits = cls.get_from_keys(config, ["w_bit", "bits"])
        group_size = cls.get_from_keys(config, ["q_group_size", "group_size"])
        zero_point = cls.get_from_keys(config, ["zero_point"])
        return cls(weight_bits, group_size, zero_point)

    @classmethod
    def is_awq_b200_compatible(cls, quant_config: Dict[str, Any]) -> bool:
        """Whether AWQ metadata can run on these kernels (config only, like
        ``AWQMarlinConfig.is_awq_marlin_compatible``, awq_marlin.py:112-143)."""
        method = str(quant_config.get("quant_method", "awq")).lower()
        bits = quant_config.get("w_bit") or quant_config.get("bits")
        group = quant_config.get("q_group_size") or quant_config.get("group_size")
        zp = quant_config.get("zero_point")
        if method != "awq" or bits != 4 or group is None or not zp:
            return False
        return group in SUPPORTED_GROUP_SIZES or (group > 0 and group % 128 == 0)

    def get_linear_method(self) -> "AWQB200LinearMethod":
        return AWQB200LinearMethod(self)

    def get_scaled_act_names(self) -> List[str]:
        return ["gelu", "gelu_fast", "gelu_new", "gelu_pytorch_tanh"]


class AWQB200LinearMethod(LinearMethodBase):
    """Linear method running AWQ weights through the sm_100a W4A16 GEMM."""

    def __init__(self, quant_config: AWQB200Config):
        self.quant_config = quant_config

    def _group(self, input_size: int) -> int:
        return input_size if self.quant_config.group_size == -1 else self.quant_config.group_size

    def create_weights(self, input_size: int, output_size: int) -> Dict[str, Any]:
        G = self._group(input_size)
        pf = self.quant_config.pack_factor
        if input_size % G != 0:
            raise ValueError(
                "The input size is not aligned with the quantized weight shape. "
                "This can be caused by too large tensor parallel size."
            )
        if output_size % pf != 0:
            raise ValueError(
                "The output size is not aligned with the quantized weight shape. "
                "This can be caused by too large tensor parallel size."
            )
        if not _kernel_group_ok(G):
            raise ValueError(f"group size {G} (input_size={input_size}) is not supported by the "
                             "B200 kernels: use 32, 64 or a multiple of 128.")
        qweight = Parameter(torch.empty(input_size, output_size // pf, dtype=torch.int32), requires_grad=False)
        set_weight_attrs(qweight, {"input_dim": 0, "output_dim": 1, "packed_dim": 1, "pack_factor": pf})
        qzeros = Parameter(torch.empty(input_size // G, output_size // pf, dtype=torch.int32), requires_grad=False)
        set_weight_attrs(qzeros, {"input_dim": 0, "output_dim": 1, "packed_dim": 1, "pack_factor": pf})
        scales = Parameter(torch.empty(input_size // G, output_size), requires_grad=False)
        set_weight_attrs(scales, {"input_dim": 0, "output_dim": 1})
        return {
            "qweight": qweight,
            "qzeros": qzeros,
            "scales": scales,
            "_input_size": input_size,
            "_output_size": output_size,
            "_group_size": G,
            "_weights_processed": False,
        }

    def process_weights_after_loading(self, weights: Dict[str, Any]) -> Dict[str, Any]:
        if weights.get("_weights_processed", False):
            return weights
        qweight, qzeros, scales = weights["qweight"], weights["qzeros"], weights["scales"]
        if qweight.device.type != "cuda":
            raise RuntimeError("AWQ B200 weights must be loaded on a CUDA device before repacking")
        K, N, G = weights["_input_size"], weights["_output_size"], weights["_group_size"]
        if scales.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError(f"scales must be float16 or bfloat16, got {scales.dtype}")
        blob = ops.repack(qweight.data.contiguous(), qzeros.data.contiguous(), scales.data.contiguous(), G)
        ops.workspace_pool.reserve(blob.device, ops.gemm_workspace_bytes(GRAPH_MAX_TOKENS, K, N, G))
        return {
            # the blob replaces the checkpoint tensors (as Marlin's repack does)
            "qweight": Parameter(blob, requires_grad=False),
            "qzeros": Parameter(torch.empty(0, dtype=torch.int32, device=blob.device), requires_grad=False),
            "scales": Parameter(torch.empty(0, dtype=scales.dtype, device=blob.device), requires_grad=False),
            "_input_size": K,
            "_output_size": N,
            "_group_size": G,
            "_act_dtype": scales.dtype,
            "_weights_processed": True,
        }

    def apply_weights(self, weights: Dict[str, Any], x: torch.Tensor,
                      bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not weights.get("_weights_processed", False):
            raise RuntimeError("process_weights_after_loading must run before apply_weights")
        if x.dtype != weights["_act_dtype"]:
            raise ValueError(f"activation dtype {x.dtype} differs from the scales dtype "
                             f"{weights['_act_dtype']} the weights were loaded with")
        # out: optional preallocated [..., N] result (e.g. a slice of a buffer the
        # caller copies to the host in one piece)
        return ops.gemm(x, weights["qweight"], weights["_input_size"], weights["_output_size"],
                        weights["_group_size"], bias=bias, out=out)
