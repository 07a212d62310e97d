"""The small-batch (decode) kernel on the GPU against the fp32-accumulated
oracle: every feature slice per CTA, ring depth, group size, both dtypes,
ragged K and N, bias, fused SiLU-and-mul, and the full Llama-3-8B decode
shapes. Tolerance (task contract): max|y - ref| <= 1e-2 * max|ref|."""

import pytest
import torch

from oracle.awq_ref import awq_linear_ref, dequant_ref, gemm_ref, rel_err
from sglite_b200 import ops
from sglite_b200.synthetic import make_activations, make_awq_weights

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _setup(cuda, M, K, N, G, dtype, seed):
    w = make_awq_weights(K, N, G, dtype, seed=seed)
    x = make_activations(M, K, dtype, seed=seed + 1)
    blob = ops.repack(*(w[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G)
    return w, x, blob


FW = [(16, 16), (32, 16), (32, 8), (64, 8)]  # built (feature slice, compute warps) pairs


@pytest.mark.parametrize("F,W", FW)
@pytest.mark.parametrize("M", [1, 3, 8, 9, 16, 17, 32])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemv_slices_and_rows(cuda, F, W, M, dtype):
    K, N, G = 4096, 384, 128
    if 2 * (W * 4 * M * 64 + W * 4 * F * 16 + 1024) + 1280 > 227 * 1024:
        pytest.skip("two load stages of this configuration exceed shared memory (rejected by the plan)")
    w, x, blob = _setup(cuda, M, K, N, G, dtype, seed=F + W + M)
    y = ops.gemv(x.to(cuda), blob, K, N, G, features_per_cta=F, warps=W)
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
    assert y.shape == (M, N) and y.dtype == dtype
    assert rel_err(y, ref) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("K,N,G", [(256, 136, 32), (320, 256, 64), (1024, 512, 1024), (128, 128, 128),
                                   (640, 200, 128), (96, 64, 32), (2048, 1000, 256), (768, 1536, 64)])
@pytest.mark.parametrize("F,W", FW)
def test_gemv_groups_and_ragged_sizes(cuda, K, N, G, F, W):
    M = 5
    dtype = torch.bfloat16
    w, x, blob = _setup(cuda, M, K, N, G, dtype, seed=K + N + F + W)
    y = ops.gemv(x.to(cuda), blob, K, N, G, features_per_cta=F, warps=W)
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
    assert rel_err(y, ref) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("ring", [1, 2, 3, 5, 8])
def test_gemv_ring_wraparound(cuda, ring):
    """Many more stages than ring slots (16 stages of 8 k-blocks): every slot
    is reused with both barrier parities; the result must not depend on the
    ring depth."""
    M, K, N, G = 4, 16384, 256, 128
    w, x, blob = _setup(cuda, M, K, N, G, torch.bfloat16, seed=ring)
    y = ops.gemv(x.to(cuda), blob, K, N, G, features_per_cta=32, warps=8, ring=ring)
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
    assert rel_err(y, ref) <= TOL
    y2 = ops.gemv(x.to(cuda), blob, K, N, G, features_per_cta=32, warps=8, ring=2)
    assert torch.equal(y, y2)
    assert ops.device_error() == 0


def test_gemv_bias_batch_dims_and_default_dispatch(cuda):
    M, K, N, G = 6, 512, 256, 128
    dtype = torch.float16
    w, x, blob = _setup(cuda, M, K, N, G, dtype, seed=3)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(4)).to(dtype)
    assert ops.gemm_plan(M, K, N, G)["cluster"] == 0  # the default path for M <= 16 is this kernel
    y = ops.gemm(x.view(2, 3, K).to(cuda), blob, K, N, G, bias=bias.to(cuda))
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G, bias=bias)
    assert y.shape == (2, 3, N)
    assert rel_err(y.view(M, N), ref) <= TOL
    assert torch.equal(y.view(M, N), ops.gemv(x.to(cuda), blob, K, N, G, bias=bias.to(cuda)))


@pytest.mark.parametrize("M", [1, 7, 16])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemv_silu_mul(cuda, M, dtype):
    K, I, G = 1024, 384, 128
    w = make_awq_weights(K, 2 * I, G, dtype, seed=I + M)
    x = make_activations(M, K, dtype, seed=M)
    qw, qz, sc = ops.interleave_gate_up(*(w[k].to(cuda) for k in ("qweight", "qzeros", "scales")))
    blob = ops.repack(qw, qz, sc, G)
    y = ops.gemm_silu_mul(x.to(cuda), blob, K, 2 * I, G)
    W = dequant_ref(w["qweight"], w["qzeros"], w["scales"], G).float()
    h = x.float() @ W
    ref = torch.nn.functional.silu(h[:, :I]) * h[:, I:]
    assert y.shape == (M, I)
    assert rel_err(y, ref) <= TOL
    y2 = ops.gemv(x.to(cuda), blob, K, 2 * I, G, features_per_cta=32, warps=8, silu_mul=True)
    assert rel_err(y2, ref) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("name,K,N", [("qkv", 4096, 6144), ("o", 4096, 4096), ("gate_up", 4096, 28672),
                                      ("down", 14336, 4096)])
@pytest.mark.parametrize("M", [1, 8, 16])
def test_gemv_llama8b_decode_shapes(cuda, name, K, N, M):
    """BASELINE config 1 shapes through the default dispatch: a slice of 256
    output features against the oracle, plus linearity over the whole output."""
    G = 128
    dtype = torch.bfloat16
    w, x, blob = _setup(cuda, M, K, N, G, dtype, seed=K + N + M)
    xa = x.to(cuda)
    xb = make_activations(M, K, dtype, seed=K + M + 99).to(cuda)
    ya = ops.gemm(xa, blob, K, N, G).float()
    yb = ops.gemm(xb, blob, K, N, G).float()
    yab = ops.gemm((xa.float() + xb.float()).to(dtype), blob, K, N, G).float()
    assert rel_err(yab, ya + yb) <= 2 * TOL
    for c0 in (0, N - 256):
        cols = slice(c0, c0 + 256)
        Wsl = dequant_ref(w["qweight"][:, c0 // 8:(c0 + 256) // 8], w["qzeros"][:, c0 // 8:(c0 + 256) // 8],
                          w["scales"][:, cols], G)
        assert rel_err(ya[:, cols], gemm_ref(x, Wsl)) <= TOL
    assert torch.equal(ops.gemm(xa, blob, K, N, G).float(), ya)  # deterministic
    assert ops.device_error() == 0
