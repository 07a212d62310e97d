"""The allocation-free GEMM entry point, checked against the regular one.

Callers such as a serving host that hands out every byte of device memory from
its own arena, or code that must never call cudaMalloc (it may run inside CUDA
graph capture), cannot supply a workspace; `awqb_gemm_noalloc` serves them
from a fixed scratch array inside the library. This file is named so that
pytest collects it last; it must pass both on its own in a fresh process and
after every other test.
"""

import ctypes

import pytest
import torch

from oracle.awq_ref import awq_linear_ref, dequant_ref, gemm_ref, rel_err
from sglite_b200 import _lib, ops
from sglite_b200.synthetic import make_activations, make_awq_weights

pytestmark = pytest.mark.gpu

TOL = 1e-2  # the GEMM tolerance used by every GEMM test here


def _noalloc(x, blob, K, N, G, out):
    dev = x.device
    st = _lib.lib().awqb_gemm_noalloc(
        ctypes.c_void_p(x.data_ptr()), x.shape[0], K, N, G, ops.DTYPE_CODE[x.dtype],
        ctypes.c_void_p(blob.data_ptr()), ctypes.c_void_p(0), ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check(st)
    return out


@pytest.mark.parametrize("M,K,N", [(1, 4096, 4096), (64, 2048, 1536), (17, 14336, 4096)])
def test_noalloc_matches_workspace_entry_point_twice(cuda, M, K, N):
    G = 128
    w = make_awq_weights(K, N, G, torch.bfloat16, seed=M + K)
    blob = ops.repack(*(w[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G)
    for call in range(2):  # the scratch keeps the previous call's contents
        x = make_activations(M, K, torch.bfloat16, seed=100 * call + M)
        xd = x.to(cuda)
        ref = ops.gemm(xd, blob, K, N, G)
        y = _noalloc(xd, blob, K, N, G, torch.empty((M, N), dtype=torch.bfloat16, device=cuda))
        torch.cuda.synchronize()
        assert rel_err(y, ref.float()) <= TOL
        assert rel_err(y, awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)) <= TOL
    assert ops.device_error() == 0


def test_noalloc_stream_k_partials_in_the_scratch(cuda):
    """Stream-K plans (cluster == 1) write fp32 partial tiles and split-tile
    counters into the fixed scratch array: two such shapes, alternated twice,
    must equal the workspace entry point bit for bit (same plan, same
    reduction order) and the oracle within the GEMM tolerance."""
    G = 128
    shapes = [(64, 4096, 14336), (48, 4096, 12288)]
    setups = []
    for M, K, N in shapes:
        assert ops.gemm_plan(M, K, N, G)["cluster"] == 1, (M, K, N, ops.gemm_plan(M, K, N, G))
        w = make_awq_weights(K, N, G, torch.bfloat16, seed=N)
        setups.append((w, ops.repack(*(w[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G)))
    for rep in range(2):
        for (M, K, N), (w, blob) in zip(shapes, setups):
            x = make_activations(M, K, torch.bfloat16, seed=rep * 7 + M)
            xd = x.to(cuda)
            y = _noalloc(xd, blob, K, N, G, torch.empty((M, N), dtype=torch.bfloat16, device=cuda))
            torch.cuda.synchronize()
            assert torch.equal(y, ops.gemm(xd, blob, K, N, G)), (M, K, N, rep)
            cols = slice(N - 512, N)
            Wsl = dequant_ref(w["qweight"][:, (N - 512) // 8:], w["qzeros"][:, (N - 512) // 8:],
                              w["scales"][:, cols], G)
            assert rel_err(y[:, cols], gemm_ref(x, Wsl)) <= TOL
    assert ops.device_error() == 0


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    K, N, G, M = 8192, 57344, 128, 4096
    assert _lib.lib().awqb_gemm_noalloc_scratch_bytes() == 16 << 20
    st = _lib.lib().awqb_gemm_noalloc(ctypes.c_void_p(16), M, K, N, G, 1, ctypes.c_void_p(16),
                                      ctypes.c_void_p(0), ctypes.c_void_p(16), ctypes.c_void_p(0))
    assert st == 2
    assert b"scratch" in _lib.lib().awqb_last_error()
