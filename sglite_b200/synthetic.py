"""Seeded synthetic AWQ inputs shaped like the benchmark configurations.

There is no public dataset on this path: weights are random 4-bit values
packed the way AWQ checkpoints store them, zero points likewise, scales uniform
in [1e-3, 1e-2], activations N(0, 1), router logits N(0, 1). Everything is
generated on the CPU with ``torch.Generator`` so a seed fixes every bit.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch

# AWQ packs logical column 8j + AWQ_PACK_ORDER[p] into bits [4p, 4p+4) of word j
# (marlin_utils.py:304,341); the unpack uses the inverse order [0,4,1,5,2,6,3,7]
# (awq_triton.py:53-62).
AWQ_PACK_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)


def pack_awq(nibbles: torch.Tensor) -> torch.Tensor:
    """int tensor [..., N] with values 0..15 -> int32 [..., N/8] in AWQ order."""
    if nibbles.shape[-1] % 8:
        raise ValueError("last dimension must be a multiple of 8")
    v = nibbles.to(torch.int64).reshape(*nibbles.shape[:-1], -1, 8)
    out = torch.zeros(v.shape[:-1], dtype=torch.int64)
    for p, i in enumerate(AWQ_PACK_ORDER):
        out |= (v[..., i] & 0xF) << (4 * p)
    out = torch.where(out >= 2**31, out - 2**32, out)
    return out.to(torch.int32)


def make_awq_weights(K: int, N: int, group_size: int, dtype: torch.dtype, seed: int,
                     batch: Optional[int] = None) -> Dict[str, torch.Tensor]:
    """AWQ tensors for a [K, N] projection (or [batch, K, N] stacked experts)."""
    G = K if group_size == -1 else group_size
    g = torch.Generator().manual_seed(seed)
    lead = () if batch is None else (batch,)
    q = torch.randint(0, 16, (*lead, K, N), generator=g, dtype=torch.int32)
    z = torch.randint(0, 16, (*lead, K // G, N), generator=g, dtype=torch.int32)
    s = (torch.rand((*lead, K // G, N), generator=g) * 9e-3 + 1e-3).to(dtype)
    return {"qweight": pack_awq(q), "qzeros": pack_awq(z), "scales": s}


def make_activations(M: int, K: int, dtype: torch.dtype, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn((M, K), generator=g).to(dtype)


def make_router_logits(M: int, E: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn((M, E), generator=g, dtype=torch.float32)


# Shapes of the benchmark configurations.
LLAMA3_8B_DECODE = {  # config 1: name -> (K, N)
    "qkv": (4096, 6144),
    "o": (4096, 4096),
    "gate_up": (4096, 28672),
    "down": (14336, 4096),
}
LLAMA3_8B_DECODE_M = (1, 8, 32, 64)

QWEN3_4B_PREFILL = {  # config 2
    "qkv": (2560, 6144),
    "o": (4096, 2560),
    "gate_up": (2560, 19456),
    "down": (9728, 2560),
}
QWEN3_4B_PREFILL_M = (512, 2048, 8192)


def llama70b_tp_shapes(tp: int) -> Dict[str, tuple]:
    """Config 3: per-rank (K, N) of the Llama-3.1-70B layer under TP=tp."""
    return {
        "qkv": (8192, 10240 // tp),
        "o": (8192 // tp, 8192),
        "gate_up": (8192, 57344 // tp),
        "down": (28672 // tp, 8192),
    }


LLAMA70B_M = (1, 32, 256, 4096)

QWEN3_30B_A3B_MOE = {"experts": 128, "topk": 8, "hidden": 2048, "intermediate": 768}
QWEN3_30B_A3B_MOE_M = (16, 256, 4096)
