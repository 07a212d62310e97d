"""Tensor-parallel sharding logic on CPU ranks (gloo, world size 2): each rank
computes its shard with the oracle, row-parallel partials are all-reduced,
and the result equals the unsharded projection."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle.awq_ref import awq_linear_ref, rel_err
from sglite_b200.synthetic import make_activations, make_awq_weights
from sglite_b200.tp import div_even, merge_awq, qkv_local_size, shard_awq


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        G, K = 128, 512
        dt = torch.bfloat16
        x = make_activations(3, K, dt, seed=1)
        # column-parallel fused gate_up: each slot sharded, then concatenated
        gate = make_awq_weights(K, 256, G, dt, seed=2)
        up = make_awq_weights(K, 256, G, dt, seed=3)
        local = merge_awq([shard_awq(gate, "column", rank, world), shard_awq(up, "column", rank, world)])
        y_local = awq_linear_ref(x, local["qweight"], local["qzeros"], local["scales"], G)
        gathered = [torch.zeros_like(y_local) for _ in range(world)]
        dist.all_gather(gathered, y_local)
        full_gate = awq_linear_ref(x, gate["qweight"], gate["qzeros"], gate["scales"], G)
        full_up = awq_linear_ref(x, up["qweight"], up["qzeros"], up["scales"], G)
        half = 256 // world
        for r in range(world):
            g_r, u_r = gathered[r][:, :half], gathered[r][:, half:]
            assert torch.equal(g_r, full_gate[:, r * half:(r + 1) * half])
            assert torch.equal(u_r, full_up[:, r * half:(r + 1) * half])
        # row-parallel down: K split, partial outputs summed
        down = make_awq_weights(K, 384, G, dt, seed=4)
        sh = shard_awq(down, "row", rank, world)
        xs = x[:, rank * K // world:(rank + 1) * K // world]
        y = awq_linear_ref(xs, sh["qweight"], sh["qzeros"], sh["scales"], G)
        dist.all_reduce(y)
        full = awq_linear_ref(x, down["qweight"], down["qzeros"], down["scales"], G)
        assert rel_err(y, full) < 1e-5
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_tp2_sharding_matches_unsharded_on_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results


def test_local_sizes_match_reference_rules():
    # Llama-3.1-70B at tp 8: 64 q / 8 kv heads x 128 -> QKV 1280 per rank
    assert qkv_local_size(64, 8, 128, 8) == 1280
    # kv heads replicated when tp > kv heads (linear.py:160-161)
    assert qkv_local_size(32, 2, 128, 4) == (8 + 2) * 128
    assert div_even(28672, 8) == 3584
    # row shards of AWQ tensors keep whole groups: down at tp 8 -> 28 groups
    w = make_awq_weights(28672 // 8 * 2, 64, 128, torch.float16, seed=0)
    sh = shard_awq(w, "row", 1, 2)
    assert sh["qweight"].shape == (3584, 8) and sh["qzeros"].shape == (28, 8) and sh["scales"].shape == (28, 64)
