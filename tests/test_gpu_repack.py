"""Repack / unrepack / dequantise on the GPU against the oracle and the
reference's own dequantised weights (bit-exact)."""

import numpy as np
import pytest
import torch

from oracle.awq_ref import dequant_ref
from sglite_b200 import ops
from sglite_b200.synthetic import make_awq_weights

pytestmark = pytest.mark.gpu

SHAPES = [
    (128, 128, 128),
    (256, 384, 64),
    (512, 136, 32),     # N not a multiple of 128 (padded features)
    (320, 256, 64),     # K not a multiple of 128 (padded k)
    (96, 64, 32),       # K < 128, N < 128
    (1024, 256, 1024),  # one group spanning several blocks (G = K)
    (768, 1536, 128),
]


@pytest.mark.parametrize("K,N,G", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_repack_roundtrip_and_dequant_exact(cuda, K, N, G, dtype):
    w = make_awq_weights(K, N, G, dtype, seed=K * 7 + N + G)
    qw, qz, sc = (w[k].to(cuda) for k in ("qweight", "qzeros", "scales"))
    blob = ops.repack(qw, qz, sc, G)
    assert blob.numel() == ops.blob_bytes(K, N, G)
    qw2, qz2, sc2 = ops.unrepack(blob, K, N, G, dtype)
    assert torch.equal(qw2, qw) and torch.equal(qz2, qz) and torch.equal(sc2.view(torch.int16), sc.view(torch.int16))
    W = ops.dequant(blob, K, N, G, dtype).cpu()
    ref = dequant_ref(w["qweight"], w["qzeros"], w["scales"], G)
    assert torch.equal(W.view(torch.int16), ref.view(torch.int16))


def test_batched_experts_exact(cuda):
    E, K, N, G = 4, 256, 384, 128
    w = make_awq_weights(K, N, G, torch.bfloat16, seed=5, batch=E)
    blob = ops.repack(*(w[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G)
    assert blob.shape == (E, ops.blob_bytes(K, N, G))
    W = ops.dequant(blob, K, N, G, torch.bfloat16).cpu()
    ref = dequant_ref(w["qweight"], w["qzeros"], w["scales"], G)
    assert torch.equal(W.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("G", [32, 64, 128])
def test_dequant_matches_reference_kernel_golden(cuda, golden, G):
    k = f"deq_g{G}"
    qw = torch.from_numpy(golden[k + "_qweight"]).to(cuda)
    qz = torch.from_numpy(golden[k + "_qzeros"]).to(cuda)
    sc = torch.from_numpy(golden[k + "_scales"]).view(torch.float16).to(cuda)
    K, N = qw.shape[0], qw.shape[1] * 8
    W = ops.dequant(ops.repack(qw, qz, sc, G), K, N, G, torch.float16).cpu()
    assert np.array_equal(W.view(torch.int16).numpy(), golden[k + "_W"])


def test_full_size_roundtrip(cuda):
    # Llama-3-8B gate_up at full size: repack is lossless (integer round trip)
    K, N, G = 4096, 28672, 128
    g = torch.Generator(device=cuda).manual_seed(11)
    qw = torch.randint(-2**31, 2**31 - 1, (K, N // 8), generator=g, device=cuda, dtype=torch.int64).to(torch.int32)
    qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), generator=g, device=cuda, dtype=torch.int64).to(torch.int32)
    sc = torch.rand((K // G, N), generator=g, device=cuda).to(torch.bfloat16)
    blob = ops.repack(qw, qz, sc, G)
    qw2, qz2, sc2 = ops.unrepack(blob, K, N, G, torch.bfloat16)
    assert torch.equal(qw2, qw) and torch.equal(qz2, qz) and torch.equal(sc2.view(torch.int16), sc.view(torch.int16))
