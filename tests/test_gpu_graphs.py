"""CUDA-graph capture of the decode calls over the reference's capture batch
list (model_executor/cuda_graph.py:76: 1, 2, 4 and multiples of 8), all graphs
sharing one memory pool (cuda_graph.py:150-160): the linear method's
apply_weights (small-batch kernel up to its crossover, tcgen05 kernel above),
gate_up fused with SiLU-and-mul, and the row-parallel GEMM fused with its
all-reduce (world size 1). Every graph is replayed with new inputs written into
its static buffers and checked against the oracle."""

import pytest
import torch

from oracle.awq_ref import awq_linear_ref, dequant_ref, rel_err
from sglite_b200 import ops
from sglite_b200.distributed import init_peer_exchange
from sglite_b200.quantization import AWQB200Config
from sglite_b200.synthetic import make_activations, make_awq_weights

pytestmark = pytest.mark.gpu

TOL = 1e-2
BS_LIST = [1, 2, 4] + list(range(8, 128 + 1, 8))


def test_graphs_over_capture_batch_list(cuda):
    G, dt = 128, torch.bfloat16
    K, N, I = 1024, 2048, 512
    method = AWQB200Config(4, G, True).get_linear_method()
    wl = make_awq_weights(K, N, G, dt, seed=1)
    lin = method.create_weights(K, N)
    lin.update({k: wl[k].to(cuda) for k in ("qweight", "qzeros", "scales")})
    lin = method.process_weights_after_loading(lin)
    wg = make_awq_weights(K, 2 * I, G, dt, seed=2)
    gu = ops.repack(*ops.interleave_gate_up(*(wg[k].to(cuda) for k in ("qweight", "qzeros", "scales"))), G)
    wr = make_awq_weights(K, N, G, dt, seed=3)
    row = ops.repack(*(wr[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G)
    ex = init_peer_exchange(tp_rank=0, tp_size=1, tp_cpu_group=None, device=cuda, max_rows=max(BS_LIST), max_n=N)
    Wg = dequant_ref(wg["qweight"], wg["qzeros"], wg["scales"], G).float()
    try:
        pool = torch.cuda.graph_pool_handle()
        graphs, bufs = {}, {}
        for bs in sorted(BS_LIST, reverse=True):  # the reference captures largest first
            xs = torch.zeros((bs, K), dtype=dt, device=cuda)
            b = {"x": xs, "y": torch.empty((bs, N), dtype=dt, device=cuda),
                 "a": torch.empty((bs, I), dtype=dt, device=cuda),
                 "r": torch.empty((bs, N), dtype=dt, device=cuda)}

            def body(b=b):
                method.apply_weights(lin, b["x"], out=b["y"])
                ops.gemm_silu_mul(b["x"], gu, K, 2 * I, G, out=b["a"])
                if b["x"].shape[0] <= ex.max_rows:
                    ex.gemm_allreduce(b["x"], row, K, N, G, out=b["r"])

            body()  # warm-up outside capture (sizes the workspace, loads kernels)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                body()
            graphs[bs], bufs[bs] = g, b
        for rep in range(2):
            for bs in BS_LIST:
                x = make_activations(bs, K, dt, seed=100 * rep + bs)
                bufs[bs]["x"].copy_(x.to(cuda))
                graphs[bs].replay()
                torch.cuda.synchronize()
                assert rel_err(bufs[bs]["y"], awq_linear_ref(x, wl["qweight"], wl["qzeros"], wl["scales"], G)) <= TOL
                h = x.float() @ Wg
                ref_a = torch.nn.functional.silu(h[:, :I]) * h[:, I:]
                assert rel_err(bufs[bs]["a"], ref_a) <= TOL, bs
                assert rel_err(bufs[bs]["r"], awq_linear_ref(x, wr["qweight"], wr["qzeros"], wr["scales"], G)) <= TOL
        del graphs
        assert ops.device_error() == 0
    finally:
        ex.destroy()
