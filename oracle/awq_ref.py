"""CPU oracle for the AWQ W4A16 path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker (or the timed CPU
baseline). It is never part of the product path.

It restates the reference's algorithm:
  * unpack (``layers/quantization/awq_triton.py:53-62,94-96,107-109,119-120``):
    logical column i of a packed int32 sits at bits 4*[0,4,1,5,2,6,3,7][i];
  * dequantise (``awq_triton.py:119-122``): W = (q - z) * s, rounded once to the
    activation dtype (computed here as an fp32 product rounded to the dtype,
    which gives the same bits because q - z and s are exact);
  * GEMM with fp32 accumulation (``awq.py:126-147``; the comparison target
    named by the task, ``max|err| <= 1e-2 * max|ref|``);
  * MoE routing and expert pipeline (``layers/fused_moe/fused.py:11-61,101-202``,
    ``kernels/triton/fused_moe.py:7-50,155-285``).

Integer unpacking is numpy; floating-point work uses torch on the CPU (numpy has
no bfloat16). Parity of this restatement is pinned against the reference's own
Triton kernel run under TRITON_INTERPRET=1 (fixtures in ``tests/golden``).
"""

from __future__ import annotations

from typing import Optional, Tuple

import numpy as np
import torch

AWQ_SHIFTS = np.array([0, 4, 1, 5, 2, 6, 3, 7], dtype=np.int64) * 4  # awq_triton.py:53-60


def unpack_awq(packed: torch.Tensor) -> torch.Tensor:
    """int32 [..., C] -> int32 [..., 8C] nibbles in logical column order."""
    a = packed.cpu().numpy().astype(np.int64) & 0xFFFFFFFF
    v = (a[..., None] >> AWQ_SHIFTS) & 0xF
    return torch.from_numpy(v.reshape(*a.shape[:-1], a.shape[-1] * 8).astype(np.int32))


def dequant_ref(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                group_size: int) -> torch.Tensor:
    """W[.., K, N] = ((q - z) * s) in scales.dtype (awq_triton.py:119-122)."""
    G = qweight.shape[-2] if group_size == -1 else group_size
    q = unpack_awq(qweight)
    z = unpack_awq(qzeros).repeat_interleave(G, dim=-2)
    s = scales.cpu().repeat_interleave(G, dim=-2)
    return ((q - z).to(torch.float32) * s.to(torch.float32)).to(scales.dtype)


def gemm_ref(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp32-accumulated x @ w (+ bias), returned in fp32."""
    y = x.cpu().to(torch.float32) @ w.cpu().to(torch.float32)
    if bias is not None:
        y = y + bias.cpu().to(torch.float32)
    return y


def awq_linear_ref(x, qweight, qzeros, scales, group_size, bias=None) -> torch.Tensor:
    return gemm_ref(x, dequant_ref(qweight, qzeros, scales, group_size), bias)


def rel_err(y: torch.Tensor, ref: torch.Tensor) -> float:
    """max|y - ref| / max|ref| (the task's tolerance metric)."""
    y = y.cpu().to(torch.float32)
    ref = ref.cpu().to(torch.float32)
    den = ref.abs().max().item()
    return (y - ref).abs().max().item() / (den if den > 0 else 1.0)


# ---------------------------------------------------------------------- MoE
def topk_softmax_ref(logits: torch.Tensor, topk: int, renormalize: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    """fused_topk (fused.py:11-31): softmax, top-k (ties to the lower index),
    renormalise by the top-k sum, then divide again by (sum + 1e-8)."""
    lg = logits.cpu().to(torch.float32)
    p = torch.softmax(lg, dim=-1)
    # stable selection on the logits: sort by (-logit, index)
    order = np.lexsort((np.broadcast_to(np.arange(lg.shape[1]), lg.shape), -lg.numpy()), axis=-1)
    ids = torch.from_numpy(order[:, :topk].astype(np.int32))
    w = torch.gather(p, 1, ids.long())
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
        w = w / (w.sum(dim=-1, keepdim=True) + 1e-8)
    return w, ids


def moe_align_ref(topk_ids: torch.Tensor, block_m: int, e_begin: int, e_end: int):
    """moe_align_block_size (fused.py:34-61) restricted to experts [e_begin, e_end):
    stable sort of flat (token, k) indices by expert, each expert padded to
    block_m with the sentinel numel. Returns (sorted_ids, block_expert, num_post_pad)."""
    flat = topk_ids.cpu().reshape(-1).numpy()
    numel = flat.size
    sorted_ids, block_expert = [], []
    for e in range(e_begin, e_end):
        idx = np.nonzero(flat == e)[0].tolist()
        if not idx:
            continue
        pad = (-len(idx)) % block_m
        sorted_ids.extend(idx + [numel] * pad)
        block_expert.extend([e - e_begin] * ((len(idx) + pad) // block_m))
    return (torch.tensor(sorted_ids, dtype=torch.int32), torch.tensor(block_expert, dtype=torch.int32),
            len(sorted_ids))


def silu_and_mul_ref(h: torch.Tensor) -> torch.Tensor:
    hf = h.to(torch.float32)
    I = hf.shape[-1] // 2
    g, u = hf[..., :I], hf[..., I:]
    return (g / (1.0 + torch.exp(-g)) * u).to(h.dtype)


def moe_ref(x: torch.Tensor, w1: dict, w2: dict, logits: torch.Tensor, topk: int,
            renormalize: bool, group_size: int, e_begin: int = 0, e_end: Optional[int] = None
            ) -> torch.Tensor:
    """AWQ MoE layer restating fused_experts_impl (fused.py:101-202) with
    dequantised expert weights w1 [E, H, 2I] and w2 [E, I, H] (AWQ dicts with
    qweight/qzeros/scales). Intermediates are rounded to the activation dtype
    where the reference stores them (cache1, cache2, cache3); the router weight
    multiplies the down-projection output (MUL_ROUTED_WEIGHT); the top-k sum
    accumulates in fp32. Only experts in [e_begin, e_end) contribute."""
    dt = x.dtype
    xf = x.cpu()
    W1 = dequant_ref(w1["qweight"], w1["qzeros"], w1["scales"], group_size)
    W2 = dequant_ref(w2["qweight"], w2["qzeros"], w2["scales"], group_size)
    E = W1.shape[0]
    e_end = E if e_end is None else e_end
    w, ids = topk_softmax_ref(logits, topk, renormalize)
    M = xf.shape[0]
    H = W2.shape[-1]
    out = torch.zeros((M, topk, H), dtype=torch.float32)
    for e in range(e_begin, e_end):
        sel = (ids == e).nonzero()
        if sel.numel() == 0:
            continue
        t, k = sel[:, 0], sel[:, 1]
        h1 = (xf[t].to(torch.float32) @ W1[e].to(torch.float32)).to(dt)
        a = silu_and_mul_ref(h1)
        y = (a.to(torch.float32) @ W2[e].to(torch.float32)) * w[t, k].unsqueeze(-1)
        out[t, k] = y.to(dt).to(torch.float32)
    return out.sum(dim=1).to(dt)


def cpu_awq_linear(x: torch.Tensor, qweight, qzeros, scales, group_size: int,
                   compute_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """The CPU baseline: dequantise on every call, then matmul (BASELINE plan)."""
    G = qweight.shape[-2] if group_size == -1 else group_size
    shifts = torch.tensor([0, 4, 1, 5, 2, 6, 3, 7], dtype=torch.int32) * 4
    q = ((qweight.unsqueeze(-1) >> shifts) & 0xF).reshape(qweight.shape[0], -1)
    z = ((qzeros.unsqueeze(-1) >> shifts) & 0xF).reshape(qzeros.shape[0], -1)
    w = (q - z.repeat_interleave(G, 0)).to(compute_dtype) * scales.repeat_interleave(G, 0).to(compute_dtype)
    return (x.to(compute_dtype) @ w).to(x.dtype)
