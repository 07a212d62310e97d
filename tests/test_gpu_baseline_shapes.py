"""Parity at the benchmark configurations' own shapes (1, 2
and 4, plus the row-count edges 4097 and 8191) against the oracle.

Large weights are generated on the GPU as uniformly random int32 words (that is,
uniformly random nibbles, as the benchmark does); the oracle dequantises the
checked column slices on the CPU from the same tensors. Tolerance (task
contract): max|y - ref| <= 1e-2 * max|ref|."""

import pytest
import torch

from oracle.awq_ref import (awq_linear_ref, dequant_ref, gemm_ref, rel_err, silu_and_mul_ref,
                            topk_softmax_ref)
from sglite_b200 import ops
from sglite_b200.synthetic import make_activations, make_awq_weights

pytestmark = pytest.mark.gpu

TOL = 1e-2
G = 128


def _gpu_awq(K, N, dtype, seed, device, lead=()):
    g = torch.Generator(device=device).manual_seed(seed)
    qw = torch.randint(-2**31, 2**31 - 1, (*lead, K, N // 8), generator=g, device=device,
                       dtype=torch.int64).to(torch.int32)
    qz = torch.randint(-2**31, 2**31 - 1, (*lead, K // G, N // 8), generator=g, device=device,
                       dtype=torch.int64).to(torch.int32)
    sc = (torch.rand((*lead, K // G, N), generator=g, device=device) * 9e-3 + 1e-3).to(dtype)
    return {"qweight": qw, "qzeros": qz, "scales": sc}


def _slice_ref(x_cpu, w, c0, c1):
    Wsl = dequant_ref(w["qweight"][:, c0 // 8:c1 // 8].cpu(), w["qzeros"][:, c0 // 8:c1 // 8].cpu(),
                      w["scales"][:, c0:c1].cpu(), G)
    return gemm_ref(x_cpu, Wsl)


def test_config0_single_linear_fp16(cuda):
    """Config 0: K = N = 4096, M = 16, fp16, every output column."""
    K = N = 4096
    M = 16
    w = make_awq_weights(K, N, G, torch.float16, seed=0)
    x = make_activations(M, K, torch.float16, seed=1)
    blob = ops.repack(*(w[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G)
    y = ops.gemm(x.to(cuda), blob, K, N, G)
    assert rel_err(y, awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)) <= TOL
    assert ops.device_error() == 0


LLAMA3_8B = {"qkv": (4096, 6144), "o": (4096, 4096), "gate_up": (4096, 28672), "down": (14336, 4096)}


@pytest.mark.parametrize("name", list(LLAMA3_8B))
@pytest.mark.parametrize("M", [1, 8, 32, 64])
def test_config1_llama3_8b_decode(cuda, name, M):
    """Config 1: every projection at every decode batch, bf16; the first and
    last 256 output columns against the oracle."""
    K, N = LLAMA3_8B[name]
    w = _gpu_awq(K, N, torch.bfloat16, seed=K + N, device=cuda)
    x = make_activations(M, K, torch.bfloat16, seed=M)
    blob = ops.repack(w["qweight"], w["qzeros"], w["scales"], G)
    y = ops.gemm(x.to(cuda), blob, K, N, G).cpu()
    for c0 in (0, N - 256):
        assert rel_err(y[:, c0:c0 + 256], _slice_ref(x, w, c0, c0 + 256)) <= TOL, (name, M, c0)
    assert ops.device_error() == 0


QWEN3_4B = {"qkv": (2560, 6144), "o": (4096, 2560), "gate_up": (2560, 19456), "down": (9728, 2560)}


@pytest.mark.parametrize("name", list(QWEN3_4B))
@pytest.mark.parametrize("M", [512, 2048, 8192])
def test_config2_qwen3_4b_prefill(cuda, name, M):
    """Config 2: prefill shapes in fp16 (the 128-token tile, long K for down);
    128 columns at each end of the output against the oracle."""
    K, N = QWEN3_4B[name]
    w = _gpu_awq(K, N, torch.float16, seed=K * 3 + N, device=cuda)
    x = make_activations(M, K, torch.float16, seed=M + K)
    blob = ops.repack(w["qweight"], w["qzeros"], w["scales"], G)
    y = ops.gemm(x.to(cuda), blob, K, N, G).cpu()
    for c0 in (0, N - 128):
        assert rel_err(y[:, c0:c0 + 128], _slice_ref(x, w, c0, c0 + 128)) <= TOL, (name, M, c0)
    assert ops.device_error() == 0


@pytest.mark.parametrize("M", [4097, 8191])
def test_row_count_edges(cuda, M):
    """Row counts one above / below a power of two (ragged last token tile)."""
    K, N = 2560, 6144
    w = _gpu_awq(K, N, torch.bfloat16, seed=M, device=cuda)
    x = make_activations(M, K, torch.bfloat16, seed=M + 1)
    blob = ops.repack(w["qweight"], w["qzeros"], w["scales"], G)
    y = ops.gemm(x.to(cuda), blob, K, N, G).cpu()
    for c0 in (0, N - 128):
        assert rel_err(y[:, c0:c0 + 128], _slice_ref(x, w, c0, c0 + 128)) <= TOL
    assert ops.device_error() == 0


def test_config4_moe_4096_tokens(cuda):
    """Config 4 at its largest batch: the whole M = 4096 layer runs on the GPU;
    the first 8 tokens are checked against the oracle's restatement of the
    expert pipeline (fused.py:101-202) over their routed experts."""
    from sglite_b200.moe import AWQB200MoeBackend, AWQExpertWeights

    E, k, H, I, M = 128, 8, 2048, 768, 4096
    dt = torch.bfloat16
    w1 = _gpu_awq(H, 2 * I, dt, seed=11, device=cuda, lead=(E,))
    w2 = _gpu_awq(I, H, dt, seed=12, device=cuda, lead=(E,))
    e1 = AWQExpertWeights.from_awq(w1["qweight"], w1["qzeros"], w1["scales"], G, gate_up=True)
    e2 = AWQExpertWeights.from_awq(w2["qweight"], w2["qzeros"], w2["scales"], G)
    x = make_activations(M, H, dt, seed=13)
    logits = torch.randn((M, E), generator=torch.Generator().manual_seed(14))
    out = x.to(cuda).clone()
    AWQB200MoeBackend().forward(out, e1, e2, logits.to(cuda), k, True)
    out = out.cpu()
    T = 8
    tw, ti = topk_softmax_ref(logits[:T], k, True)
    ref = torch.zeros((T, H), dtype=torch.float32)
    cache = {}
    for t in range(T):
        for j in range(k):
            e = int(ti[t, j])
            if e not in cache:
                cache[e] = (dequant_ref(w1["qweight"][e].cpu(), w1["qzeros"][e].cpu(), w1["scales"][e].cpu(), G),
                            dequant_ref(w2["qweight"][e].cpu(), w2["qzeros"][e].cpu(), w2["scales"][e].cpu(), G))
            W1, W2 = cache[e]
            h1 = (x[t:t + 1].float() @ W1.float()).to(dt)
            a = silu_and_mul_ref(h1)
            y = ((a.float() @ W2.float()) * tw[t, j]).to(dt)
            ref[t] += y[0].float()
    assert rel_err(out[:T], ref) <= TOL
    assert ops.device_error() == 0
