"""W4A16 GEMM on the GPU against the fp32-accumulated oracle and against the
reference Triton kernel's own outputs. Tolerance (task contract):
max|y - ref| <= 1e-2 * max|ref|."""

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


EDGE_M = [1, 3, 16, 17, 63, 64, 65, 127, 200, 257, 511]


@pytest.mark.parametrize("M", EDGE_M)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gemm_edge_m(cuda, M, dtype):
    K, N, G = 512, 384, 128
    w, x, blob = _setup(cuda, M, K, N, G, dtype, seed=M)
    y = ops.gemm(x.to(cuda), blob, K, N, G)
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
    assert y.shape == (M, N) and y.dtype == dtype
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("K,N,G", [(256, 136, 32), (320, 256, 64), (1024, 512, 1024), (128, 128, 128),
                                   (768, 1536, 128), (2048, 768, 128)])
@pytest.mark.parametrize("M", [1, 33, 300])
def test_gemm_shapes_and_groups(cuda, K, N, G, M):
    dtype = torch.bfloat16
    w, x, blob = _setup(cuda, M, K, N, G, dtype, seed=K + N + M)
    y = ops.gemm(x.to(cuda), blob, K, N, G)
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
    assert rel_err(y, ref) <= TOL


@pytest.mark.parametrize("ntok", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("ctas", [1, 3, 7, 64, 0])
def test_gemm_tiles_and_stream_k_splits(cuda, ntok, ctas):
    # few CTAs force tiles to be split across contributors and fixed up
    M, K, N, G = 70, 1024, 512, 128
    w, x, blob = _setup(cuda, M, K, N, G, torch.float16, seed=ntok * 13 + ctas)
    y = ops.gemm(x.to(cuda), blob, K, N, G, ntok=ntok, ctas=ctas)
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
    assert rel_err(y, ref) <= TOL


def test_gemm_bias_and_batch_dims(cuda):
    M, K, N, G = 6, 256, 256, 128
    dtype = torch.float16
    w, x, blob = _setup(cuda, M, K, N, G, dtype, seed=3)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(4)).to(dtype)
    y = ops.gemm(x.view(2, 3, K).to(cuda), blob, K, N, G, bias=bias.to(cuda))
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G, bias=bias)
    assert y.shape == (2, 3, N)
    assert rel_err(y.view(M, N), ref) <= TOL


def test_gemm_deterministic_and_workspace_clean(cuda):
    M, K, N, G = 9, 4096, 4096, 128
    w, x, blob = _setup(cuda, M, K, N, G, torch.bfloat16, seed=21)
    xd = x.to(cuda)
    y1 = ops.gemm(xd, blob, K, N, G)
    y2 = ops.gemm(xd, blob, K, N, G)
    assert torch.equal(y1, y2)
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
    assert rel_err(y1, ref) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("i", [0, 1, 2])
def test_gemm_vs_reference_kernel_golden(cuda, golden, i):
    k = f"gemm{i}"
    M, K, N, G = (int(v) for v in golden[k + "_shape"])
    x = torch.from_numpy(golden[k + "_x"]).view(torch.float16)
    qw = torch.from_numpy(golden[k + "_qweight"])
    qz = torch.from_numpy(golden[k + "_qzeros"])
    sc = torch.from_numpy(golden[k + "_scales"]).view(torch.float16)
    y_ref_kernel = torch.from_numpy(golden[k + "_y"]).view(torch.float16)
    blob = ops.repack(qw.to(cuda), qz.to(cuda), sc.to(cuda), G)
    y = ops.gemm(x.to(cuda), blob, K, N, G)
    # the reference kernel accumulates in fp16; both must be within the contract
    # of the fp32 oracle, and of each other
    ref = gemm_ref(x, dequant_ref(qw, qz, sc, G))
    assert rel_err(y, ref) <= TOL
    assert rel_err(y_ref_kernel, ref) <= TOL
    assert rel_err(y, y_ref_kernel.float()) <= TOL


@pytest.mark.parametrize("name,K,N", [("qkv", 4096, 6144), ("down", 14336, 4096)])
@pytest.mark.parametrize("M", [1, 64])
def test_gemm_full_size_linearity(cuda, name, K, N, M):
    """Full Llama-3-8B sizes: y(a + b) = y(a) + y(b) and a column spot check
    against the oracle on a slice of output features."""
    G = 128
    dtype = torch.bfloat16
    w, x, blob = _setup(cuda, M, K, N, G, dtype, seed=K + M)
    xa = x.to(cuda)
    xb = make_activations(M, K, dtype, seed=K + M + 99).to(cuda)
    ya = ops.gemm(xa, blob, K, N, G).float()
    yb = ops.gemm(xb, blob, K, N, G).float()
    yab = ops.gemm((xa.float() + xb.float()).to(dtype), blob, K, N, G).float()
    assert rel_err(yab, ya + yb) <= 2 * TOL
    cols = slice(N - 256, N)
    Wsl = dequant_ref(w["qweight"][:, (N - 256) // 8:], w["qzeros"][:, (N - 256) // 8:], w["scales"][:, cols], G)
    ref = gemm_ref(x, Wsl)
    assert rel_err(ya[:, cols], ref) <= TOL


def test_shared_workspace_mixed_shapes(cuda):
    """Calls of different shapes and token tiles share the per-device workspace:
    each result equals the one computed with a fresh zero-filled workspace (the
    split-tile reduction order is fixed, so equality is exact)."""
    G = 128
    dtype = torch.bfloat16
    shapes = [(4096, 4096), (4096, 6144), (2048, 7168), (7168, 1024)]
    setups = [_setup(cuda, 1, K, N, G, dtype, seed=K + N) for K, N in shapes]
    for rep in range(2):
        for (K, N), (w, _, blob) in zip(shapes, setups):
            for M in (1, 40, 300):
                x = make_activations(M, K, dtype, seed=M + rep).to(cuda)
                y_shared = ops.gemm(x, blob, K, N, G)
                fresh = torch.zeros(ops.gemm_workspace_bytes(M, K, N, G), dtype=torch.uint8, device=cuda)
                y_fresh = ops.gemm(x, blob, K, N, G, workspace=fresh)
                assert torch.equal(y_shared, y_fresh), (K, N, M, rep)
    assert ops.device_error() == 0


@pytest.mark.parametrize("ntok", [64, 128, 256])
def test_gemm_data_parallel_waves(cuda, ntok):
    """Enough tiles for several waves: whole tiles are processed data-parallel
    and only the last waves are split stream-K; checked against the oracle."""
    M, K, N, G = 2304, 512, 4096, 128
    w, x, blob = _setup(cuda, M, K, N, G, torch.float16, seed=ntok)
    y = ops.gemm(x.to(cuda), blob, K, N, G, ntok=ntok)
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
    assert rel_err(y, ref) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("K,N,M", [(4096, 4096, 1), (4096, 4096, 33), (4096, 4096, 64), (8192, 1280, 5), (1024, 8192, 16),
                                   (4096, 2560, 256)])
def test_gemm_cluster_split_k(cuda, K, N, M):
    """Few feature tiles: each tile's stages are split over a thread-block
    cluster and reduced through distributed shared memory. Checked against the
    oracle and against the stream-K launch (reduction through the workspace)."""
    G = 128
    nt = 16 if M <= 16 else 0  # small M: force the tcgen05 kernel (the default is the small-batch one)
    plan = ops.gemm_plan(M, K, N, G, ntok=nt)
    assert plan["cluster"] >= 2, plan
    w, x, blob = _setup(cuda, M, K, N, G, torch.bfloat16, seed=K + N + M)
    y = ops.gemm(x.to(cuda), blob, K, N, G, ntok=nt)
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
    assert rel_err(y, ref) <= TOL
    y_sk = ops.gemm(x.to(cuda), blob, K, N, G, ctas=torch.cuda.get_device_properties(cuda).multi_processor_count)
    assert ops.gemm_plan(M, K, N, G, ctas=1)["cluster"] == 1
    assert rel_err(y, y_sk.float()) <= TOL
    assert torch.equal(y, ops.gemm(x.to(cuda), blob, K, N, G, ntok=nt))  # deterministic
    assert ops.device_error() == 0


@pytest.mark.parametrize("I", [64, 200, 768])
@pytest.mark.parametrize("M", [1, 5, 64, 300])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemm_silu_mul_fused(cuda, I, M, dtype):
    """gate_up GEMM with SiLU-and-mul in the epilogue (columns interleaved at
    load) against the oracle: silu(x W_gate) * (x W_up) in fp32."""
    from oracle.awq_ref import dequant_ref

    K, G = 512, 128
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
    assert ops.device_error() == 0


def test_clear_device_error_resets_pooled_counters(cuda):
    """Counters left non-zero in the shared workspace (as a GEMM whose bounded
    wait gave up may leave them) are zeroed by clear_device_error, after which a
    split-K GEMM on the pool equals one on a fresh workspace bit for bit."""
    M, K, N, G = 64, 4096, 14336, 128
    assert ops.gemm_plan(M, K, N, G)["cluster"] == 1  # stream-K: counters in the workspace
    w, x, blob = _setup(cuda, M, K, N, G, torch.bfloat16, seed=77)
    xd = x.to(cuda)
    ops.gemm(xd, blob, K, N, G)  # sizes the pool
    torch.cuda.synchronize()
    for buf in ops.workspace_pool._bufs.values():
        buf[:ops.COUNTER_BYTES].fill_(0x5A)  # host-side poison; no GEMM runs on it
    ops.clear_device_error()
    for buf in ops.workspace_pool._bufs.values():
        assert int(buf[:ops.COUNTER_BYTES].count_nonzero()) == 0
    y_pool = ops.gemm(xd, blob, K, N, G)
    fresh = torch.zeros(ops.gemm_workspace_bytes(M, K, N, G), dtype=torch.uint8, device=cuda)
    y_fresh = ops.gemm(xd, blob, K, N, G, workspace=fresh)
    assert torch.equal(y_pool, y_fresh)
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
    assert rel_err(y_pool, ref) <= TOL
    assert ops.device_error() == 0
