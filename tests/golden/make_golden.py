"""Generate golden fixtures from the reference's own kernels (run once, offline).

The reference has no tests or golden vectors for this path, so the fixtures are
produced by running its kernels on the CPU under TRITON_INTERPRET=1:

* ``awq_triton.awq_gemm_triton`` (layers/quantization/awq_triton.py:144-195) with
  identity activations -> the reference's own dequantised weights, bit for bit
  (each output element is 1.0 * W[k, n] plus exact zeros);
* the same kernel on random fp16 activations -> reference GEMM outputs;
* ``fused_moe_kernel`` and ``moe_sum_reduce_kernel``
  (kernels/triton/fused_moe.py:7-50,155-285), launched with the grid and
  arguments of kernels/moe_triton.py:8-102, on dense expert weights obtained by
  dequantising AWQ experts; routing comes from the oracle because the
  reference's topk_softmax / moe_align_block_size live in the absent sgl_kernel.

Usage (needs the reference checkout; never run by the tests):
    python tests/golden/make_golden.py /path/to/reference
"""

from __future__ import annotations

import importlib.util
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.awq_ref import dequant_ref, moe_align_ref, topk_softmax_ref  # noqa: E402
from sglite_b200.synthetic import make_activations, make_awq_weights, make_router_logits  # noqa: E402


def _load(name: str, path: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(ref_root: str) -> None:
    qdir = os.path.join(ref_root, "python/sglite/srt/model_executor/layers/quantization")
    at = _load("ref_awq_triton", os.path.join(qdir, "awq_triton.py"))
    fm = _load("ref_fused_moe", os.path.join(ref_root, "python/sglite/kernels/triton/fused_moe.py"))

    out = {}
    # 1) dequantised weights through the reference kernel (identity activations)
    for G in (32, 64, 128):
        K, N = 256, 128
        w = make_awq_weights(K, N, G, torch.float16, seed=100 + G)
        eye = torch.eye(K, dtype=torch.float16)
        W = at.awq_gemm_triton(eye, w["qweight"], w["scales"], w["qzeros"], 8)
        key = f"deq_g{G}"
        out[key + "_qweight"] = w["qweight"].numpy()
        out[key + "_qzeros"] = w["qzeros"].numpy()
        out[key + "_scales"] = w["scales"].view(torch.int16).numpy()
        out[key + "_W"] = W.view(torch.int16).numpy()
        assert torch.equal(W, dequant_ref(w["qweight"], w["qzeros"], w["scales"], G)), key

    # 2) GEMM outputs of the reference kernel
    for i, (M, K, N, G) in enumerate([(1, 512, 256, 128), (5, 512, 256, 64), (33, 256, 384, 128)]):
        w = make_awq_weights(K, N, G, torch.float16, seed=200 + i)
        x = make_activations(M, K, torch.float16, seed=300 + i)
        y = at.awq_gemm_triton(x, w["qweight"], w["scales"], w["qzeros"], 8)
        key = f"gemm{i}"
        out[key + "_shape"] = np.array([M, K, N, G], dtype=np.int64)
        out[key + "_x"] = x.view(torch.int16).numpy()
        out[key + "_qweight"] = w["qweight"].numpy()
        out[key + "_qzeros"] = w["qzeros"].numpy()
        out[key + "_scales"] = w["scales"].view(torch.int16).numpy()
        out[key + "_y"] = y.view(torch.int16).numpy()

    # 3) MoE: reference grouped kernels on dense (dequantised) experts
    E, topk, H, I, M, BM, G = 8, 2, 128, 128, 5, 16, 128
    w1 = make_awq_weights(H, 2 * I, G, torch.float16, seed=400, batch=E)
    w2 = make_awq_weights(I, H, G, torch.float16, seed=401, batch=E)
    x = make_activations(M, H, torch.float16, seed=402)
    logits = make_router_logits(M, E, seed=403)
    tw, tid = topk_softmax_ref(logits, topk, True)
    sorted_ids, block_expert, npp = moe_align_ref(tid, BM, 0, E)
    W1 = dequant_ref(w1["qweight"], w1["qzeros"], w1["scales"], G)  # [E, H, 2I]
    W2 = dequant_ref(w2["qweight"], w2["qzeros"], w2["scales"], G)  # [E, I, H]
    B1 = W1.transpose(1, 2).contiguous()  # reference layout [E, N, K]
    B2 = W2.transpose(1, 2).contiguous()
    num_post = torch.tensor([npp], dtype=torch.int32)
    cache1 = torch.zeros((M, topk, 2 * I), dtype=torch.float16)
    cache3 = torch.zeros((M, topk, H), dtype=torch.float16)
    cfg = dict(BLOCK_SIZE_M=BM, BLOCK_SIZE_N=32, BLOCK_SIZE_K=64, GROUP_SIZE_M=1)

    def run(A, B, C, mul_w, top_k):
        grid = ((sorted_ids.shape[0] + BM - 1) // BM * ((B.shape[1] + 31) // 32),)
        fm.fused_moe_kernel[grid](
            A, B, C, tw, sorted_ids, block_expert, num_post, B.shape[1], B.shape[2],
            sorted_ids.shape[0], tid.numel(), A.stride(0), A.stride(1), B.stride(0), B.stride(2),
            B.stride(1), C.stride(1), C.stride(2), MUL_ROUTED_WEIGHT=mul_w, top_k=top_k,
            compute_type=fm.tl.float16, even_Ks=True, **cfg)

    run(x, B1, cache1, False, topk)
    h = cache1.view(-1, 2 * I).float()
    act = (h[:, :I] / (1 + torch.exp(-h[:, :I])) * h[:, I:]).to(torch.float16)
    run(act, B2, cache3, True, 1)
    y = torch.zeros((M, H), dtype=torch.float16)
    fm.moe_sum_reduce_kernel[(M, 1)](cache3, *cache3.stride(), y, *y.stride(), token_num=M, topk_num=topk,
                                     hidden_dim=H, BLOCK_M=1, BLOCK_DIM=2048, NUM_STAGE=1)
    for k, v in w1.items():
        out["moe_w1_" + k] = (v.view(torch.int16) if v.dtype == torch.float16 else v).numpy()
    for k, v in w2.items():
        out["moe_w2_" + k] = (v.view(torch.int16) if v.dtype == torch.float16 else v).numpy()
    out["moe_shape"] = np.array([E, topk, H, I, M, BM, G], dtype=np.int64)
    out["moe_x"] = x.view(torch.int16).numpy()
    out["moe_logits"] = logits.numpy()
    out["moe_y"] = y.view(torch.int16).numpy()

    path = os.path.join(HERE, "awq_reference_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the SGLite source checkout>")
    main(sys.argv[1])
