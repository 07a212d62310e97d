"""Row-parallel GEMM fused with its all-reduce over peer memory, on one GPU: an
exchange of world size 1 runs the whole protocol (landing-slot stores, system-
scope flags, rank-order sum, flag reset, device-side parity) against itself, so
its output must equal the plain GEMM bit for bit."""

import pytest
import torch

from oracle.awq_ref import awq_linear_ref, rel_err
from sglite_b200 import ops
from sglite_b200.distributed import init_peer_exchange
from sglite_b200.synthetic import make_activations, make_awq_weights

pytestmark = pytest.mark.gpu


@pytest.fixture
def exchange(cuda):
    ex = init_peer_exchange(tp_rank=0, tp_size=1, tp_cpu_group=None, device=cuda, max_rows=64, max_n=8192)
    yield ex
    ex.destroy()


def _plain(x, blob, K, N, G, bias=None):
    """The plain GEMM; the fused call runs the same kernel and plan (the
    small-batch kernel for small M, the tcgen05 kernel above), so a world of
    one must reproduce it bit for bit."""
    return ops.gemm(x, blob, K, N, G, bias=bias)


def _blob(cuda, K, N, G, dt, seed):
    w = make_awq_weights(K, N, G, dt, seed=seed)
    return w, ops.repack(*(w[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G)


@pytest.mark.parametrize("mode", ["auto", "reduce_scatter"])
@pytest.mark.parametrize("K,N", [(4096, 4096), (1024, 8192), (3584, 8192), (2048, 1000)])
def test_fused_equals_plain_gemm(cuda, exchange, K, N, mode):
    G, dt = 128, torch.bfloat16
    exchange.set_mode(mode)
    w, blob = _blob(cuda, K, N, G, dt, K + N)
    for rep in range(3):  # consecutive calls alternate the landing / flag parity
        for M in (1, 5, 8, 16, 17, 33, 64):
            x = make_activations(M, K, dt, seed=M + rep).to(cuda)
            y = exchange.gemm_allreduce(x, blob, K, N, G)
            assert torch.equal(y, _plain(x, blob, K, N, G)), (K, N, M, rep, ops.gemm_plan(M, K, N, G))
    x = make_activations(7, K, dt, seed=3)
    ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
    assert rel_err(exchange.gemm_allreduce(x.to(cuda), blob, K, N, G), ref) <= 1e-2
    assert ops.device_error() == 0


def test_fused_bias_and_fp16(cuda, exchange):
    G, dt, K, N = 128, torch.float16, 2048, 4096
    _, blob = _blob(cuda, K, N, G, dt, 5)
    bias = torch.randn(N, device=cuda).to(dt)
    x = make_activations(9, K, dt, seed=1).to(cuda)
    assert torch.equal(exchange.gemm_allreduce(x, blob, K, N, G, bias=bias), _plain(x, blob, K, N, G, bias=bias))
    assert ops.device_error() == 0


def test_fused_inside_cuda_graph_odd_call_count(cuda, exchange):
    """The parity lives on the device, so a graph holding an odd number of
    fused calls still alternates buffers from one replay to the next."""
    G, dt = 128, torch.bfloat16
    shapes = [(4096, 4096), (3584, 8192), (1024, 8192)]
    blobs = [_blob(cuda, K, N, G, dt, i)[1] for i, (K, N) in enumerate(shapes)]
    xs = [make_activations(4, K, dt, seed=i).to(cuda) for i, (K, N) in enumerate(shapes)]
    outs = [torch.empty(4, N, dtype=dt, device=cuda) for K, N in shapes]
    for (K, N), b, x, o in zip(shapes, blobs, xs, outs):  # reserve the workspace before capture
        exchange.gemm_allreduce(x, b, K, N, G, out=o)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for (K, N), b, x, o in zip(shapes, blobs, xs, outs):
            exchange.gemm_allreduce(x, b, K, N, G, out=o)
    for _ in range(5):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for (K, N), b, x, o in zip(shapes, blobs, xs, outs):
            assert torch.equal(o, _plain(x, b, K, N, G))
    del g
    assert ops.device_error() == 0


def test_fused_rejects_oversized_batches(cuda, exchange):
    G, K, N = 128, 1024, 1024
    _, blob = _blob(cuda, K, N, G, torch.bfloat16, 1)
    x = make_activations(65, K, torch.bfloat16, seed=1).to(cuda)
    with pytest.raises(ValueError):
        exchange.gemm_allreduce(x, blob, K, N, G)


def test_fused_stream_k_epilogue_up_to_256_rows(cuda):
    """An exchange sized for 256 rows: M = 256 over N = 8192 has more tiles than
    half the SMs, so the fused all-reduce runs in the stream-K epilogue
    (tp_put / tp_finish); three calls alternate both landing parities and must
    equal the plain GEMM of the same plan bit for bit."""
    G, dt, K, N, M = 128, torch.bfloat16, 1024, 8192, 256
    ex = init_peer_exchange(tp_rank=0, tp_size=1, tp_cpu_group=None, device=cuda, max_rows=256, max_n=N)
    try:
        assert ops.gemm_plan(M, K, N, G)["cluster"] == 1
        w, blob = _blob(cuda, K, N, G, dt, 11)
        for rep in range(3):
            x = make_activations(M, K, dt, seed=rep).to(cuda)
            y = ex.gemm_allreduce(x, blob, K, N, G)
            assert torch.equal(y, ops.gemm(x, blob, K, N, G)), rep
        x = make_activations(M, K, dt, seed=5)
        ref = awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)
        assert rel_err(ex.gemm_allreduce(x.to(cuda), blob, K, N, G), ref) <= 1e-2
        assert ops.device_error() == 0
    finally:
        ex.destroy()
