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

from oracle.awq_ref import rel_err
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
        x = make_activations(M, K, torch.bfloat16, seed=100 * call + M).to(cuda)
        ref = ops.gemm(x, blob, K, N, G)
        y = _noalloc(x, blob, K, N, G, torch.empty((M, N), dtype=torch.bfloat16, device=cuda))
        torch.cuda.synchronize()
        assert rel_err(y, ref.float()) <= TOL
    assert ops.device_error() == 0


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    K, N, G, M = 8192, 57344, 128, 4096
    assert _lib.lib().awqb_gemm_noalloc_scratch_bytes() == 16 << 20
    st = _lib.lib().awqb_gemm_noalloc(ctypes.c_void_p(16), M, K, N, G, 1, ctypes.c_void_p(16),
                                      ctypes.c_void_p(0), ctypes.c_void_p(16), ctypes.c_void_p(0))
    assert st == 2
    assert b"scratch" in _lib.lib().awqb_last_error()
