"""Tensor parallelism on real GPUs (2 ranks, NCCL through the C ABI): the
row-parallel AWQ projection plus all-reduce equals the unsharded oracle, for a
message staged through the symmetric window and one reduced in place."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    from oracle.awq_ref import awq_linear_ref, rel_err
    from sglite_b200.distributed import init_nccl, init_peer_exchange
    from sglite_b200.quantization import AWQB200Config
    from sglite_b200.synthetic import make_activations, make_awq_weights
    from sglite_b200.tp import ColumnParallelAWQLinear, RowParallelAWQLinear, shard_awq

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    comm = ex = None
    try:
        comm = init_nccl(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD, device=dev,
                         max_size_bytes=64 * 4096 * 2)
        ex = init_peer_exchange(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD, device=dev,
                                max_rows=64, max_n=4096)
        method = AWQB200Config(4, 128, True).get_linear_method()
        G, K, N = 128, 4096, 4096
        dt = torch.bfloat16
        full = make_awq_weights(K, N, G, dt, seed=9)
        row = RowParallelAWQLinear(method, K, N, world, comm)
        row.load({k: v.to(dev) for k, v in shard_awq(full, "row", rank, world).items()})
        col = ColumnParallelAWQLinear(method, K, N // world)
        col.load({k: v.to(dev) for k, v in shard_awq(full, "column", rank, world).items()})
        rowf = RowParallelAWQLinear(method, K, N, world, comm, exchange=ex)
        rowf.load({k: v.to(dev) for k, v in shard_awq(full, "row", rank, world).items()})
        for M in (1, 64, 700):  # 700 x 4096 x 2 B exceeds the symmetric window: in-place path
            x = make_activations(M, K, dt, seed=M)
            xl = x[:, rank * K // world:(rank + 1) * K // world].contiguous().to(dev)
            y = row.forward(xl)
            ref = awq_linear_ref(x, full["qweight"], full["qzeros"], full["scales"], G)
            e = rel_err(y, ref)
            assert e <= 1e-2, (M, e)
            # fused GEMM + all-reduce over peer memory (M <= 64; NCCL above),
            # all-to-all and reduce-scatter + all-gather: identical bits
            yfs = []
            for mode in ("all_to_all", "reduce_scatter", "auto"):
                ex.set_mode(mode)
                for _ in range(3):
                    yf = rowf.forward(xl)
                    assert rel_err(yf, ref) <= 1e-2, (M, mode, rel_err(yf, ref))
                yfs.append(yf.clone())
            assert all(torch.equal(yfs[0], t) for t in yfs), M
            # every rank holds the same bits
            got = [None] * world
            dist.all_gather_object(got, yf.float().cpu().numpy().tobytes())
            assert all(g == got[0] for g in got)
            yc = col.forward(x.to(dev))
            refc = ref[:, rank * N // world:(rank + 1) * N // world]
            assert rel_err(yc, refc) <= 1e-2
        torch.cuda.synchronize()
        from sglite_b200 import ops
        assert ops.device_error() == 0
        q.put((rank, "ok"))
    except Exception as err:
        q.put((rank, repr(err)))
    finally:
        if ex is not None:
            ex.destroy()
        if comm is not None:
            comm.destroy()
        dist.destroy_process_group()


def test_tp2_row_parallel_with_nccl_all_reduce():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
