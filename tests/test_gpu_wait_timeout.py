"""A bounded device wait that runs out, in the form that faults, traps or hangs
nothing: a world-size-2 fused GEMM + all-reduce whose peer never takes part.

A helper process creates rank 1's exchange buffer, hands its IPC handle over
and then only waits (it launches no kernel); rank 0's kernel stores its
partials and waits for rank 1's words, which never arrive. Every waiting
thread gives up after the library's 2 s limit, the kernel returns, the device
error word carries the epilogue-wait bit, and the GPU keeps working: a plain
GEMM afterwards matches the oracle. The helper keeps its allocation alive until
rank 0 has closed its mapping."""

import multiprocessing as mp

import pytest
import torch

from oracle.awq_ref import awq_linear_ref, rel_err
from sglite_b200 import ops
from sglite_b200.distributed import PeerExchange
from sglite_b200.synthetic import make_activations, make_awq_weights

pytestmark = pytest.mark.gpu

ERR_WAIT_EPILOGUE = 8  # DeviceError::kErrWaitEpilogue (awqb_gemm.cuh)


def _silent_peer(q_handle, ev_done):
    import torch as _torch

    from sglite_b200.distributed import PeerExchange as _PX

    dev = _torch.device("cuda", 0)
    _torch.cuda.set_device(dev)
    ex = _PX(1, 2, dev, 8, 1024)
    q_handle.put(ex.handle())
    ev_done.wait(120)  # keep the buffer mapped until rank 0 is done with it
    ex.destroy()


def test_peer_that_never_writes_turns_into_a_device_error(cuda):
    ctx = mp.get_context("spawn")
    q, ev = ctx.Queue(), ctx.Event()
    peer = ctx.Process(target=_silent_peer, args=(q, ev))
    peer.start()
    ex = None
    try:
        h1 = q.get(timeout=120)
        ex = PeerExchange(0, 2, cuda, 8, 1024)
        ex.open([ex.handle(), h1])
        K, N, G = 512, 1024, 128
        w = make_awq_weights(K, N, G, torch.bfloat16, seed=5)
        blob = ops.repack(*(w[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G)
        x = make_activations(4, K, torch.bfloat16, seed=6)
        ops.clear_device_error()
        ex.gemm_allreduce(x.to(cuda), blob, K, N, G)
        err = ops.device_error(clear=False)
        assert err & ERR_WAIT_EPILOGUE, err
        ops.clear_device_error()
        assert ops.device_error() == 0
        # the context and the GPU still work
        y = ops.gemm(x.to(cuda), blob, K, N, G)
        assert rel_err(y, awq_linear_ref(x, w["qweight"], w["qzeros"], w["scales"], G)) <= 1e-2
    finally:
        if ex is not None:
            ex.destroy()
        ev.set()
        peer.join(timeout=120)
        if peer.is_alive():
            peer.kill()
