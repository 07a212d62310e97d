"""The CPU oracle against the reference's own kernels (fixtures produced by
tests/golden/make_golden.py from the reference's Triton kernels)."""

import numpy as np
import pytest
import torch

from oracle.awq_ref import dequant_ref, gemm_ref, moe_align_ref, moe_ref, rel_err, topk_softmax_ref, unpack_awq
from sglite_b200.synthetic import AWQ_PACK_ORDER, make_awq_weights, pack_awq


@pytest.mark.parametrize("G", [32, 64, 128])
def test_oracle_dequant_is_bit_exact_with_reference_kernel(golden, G):
    k = f"deq_g{G}"
    qw = torch.from_numpy(golden[k + "_qweight"])
    qz = torch.from_numpy(golden[k + "_qzeros"])
    sc = torch.from_numpy(golden[k + "_scales"]).view(torch.float16)
    W = dequant_ref(qw, qz, sc, G)
    assert np.array_equal(W.view(torch.int16).numpy(), golden[k + "_W"])


@pytest.mark.parametrize("i", [0, 1, 2])
def test_oracle_gemm_matches_reference_kernel(golden, i):
    k = f"gemm{i}"
    M, K, N, G = (int(v) for v in golden[k + "_shape"])
    x = torch.from_numpy(golden[k + "_x"]).view(torch.float16)
    W = dequant_ref(torch.from_numpy(golden[k + "_qweight"]), torch.from_numpy(golden[k + "_qzeros"]),
                    torch.from_numpy(golden[k + "_scales"]).view(torch.float16), G)
    y_ref_kernel = torch.from_numpy(golden[k + "_y"]).view(torch.float16)
    # the reference accumulates in fp16 (awq_triton.py:43,125): within the contract of fp32
    assert rel_err(y_ref_kernel, gemm_ref(x, W)) <= 1e-2


def test_oracle_moe_matches_reference_kernels(golden):
    E, topk, H, I, M, BM, G = (int(v) for v in golden["moe_shape"])
    w1 = {k: torch.from_numpy(golden["moe_w1_" + k]) for k in ("qweight", "qzeros", "scales")}
    w2 = {k: torch.from_numpy(golden["moe_w2_" + k]) for k in ("qweight", "qzeros", "scales")}
    w1["scales"] = w1["scales"].view(torch.float16)
    w2["scales"] = w2["scales"].view(torch.float16)
    x = torch.from_numpy(golden["moe_x"]).view(torch.float16)
    logits = torch.from_numpy(golden["moe_logits"])
    y = moe_ref(x, w1, w2, logits, topk, True, G)
    y_kernel = torch.from_numpy(golden["moe_y"]).view(torch.float16)
    assert rel_err(y, y_kernel.float()) <= 1e-2


def test_pack_order_roundtrip():
    g = torch.Generator().manual_seed(0)
    q = torch.randint(0, 16, (5, 64), generator=g, dtype=torch.int32)
    assert torch.equal(unpack_awq(pack_awq(q)), q)
    # logical column i of a word sits at bits 4 * [0,4,1,5,2,6,3,7][i] (awq_triton.py:53-62)
    one = torch.zeros(1, 8, dtype=torch.int32)
    for i in range(8):
        one.zero_()
        one[0, i] = 1
        word = int(pack_awq(one)[0, 0]) & 0xFFFFFFFF
        assert word == 1 << (4 * AWQ_PACK_ORDER.index(i))


def test_dequant_fp32_product_rounding_matches_dtype_arithmetic():
    # (q - z) and s are exact, so one fp32 product rounded to the dtype equals the
    # dtype multiply (the bit-exact contract the GPU kernels follow)
    for dt in (torch.float16, torch.bfloat16):
        w = make_awq_weights(256, 64, 128, dt, seed=3)
        q = unpack_awq(w["qweight"])
        z = unpack_awq(w["qzeros"]).repeat_interleave(128, 0)
        s = w["scales"].repeat_interleave(128, 0)
        assert torch.equal(dequant_ref(w["qweight"], w["qzeros"], w["scales"], 128), (q - z).to(dt) * s)


def test_topk_softmax_ref_properties():
    lg = torch.randn(64, 128, generator=torch.Generator().manual_seed(1))
    w, ids = topk_softmax_ref(lg, 8, True)
    assert torch.allclose(w.sum(-1), torch.ones(64), atol=1e-6)
    top = torch.topk(lg, 8, dim=-1).indices.sort(-1).values
    assert torch.equal(ids.long().sort(-1).values, top)


def test_moe_align_ref_properties():
    ids = torch.randint(0, 16, (37, 4), generator=torch.Generator().manual_seed(2), dtype=torch.int32)
    sorted_ids, block_expert, npp = moe_align_ref(ids, 8, 0, 16)
    numel = ids.numel()
    assert npp % 8 == 0 and len(block_expert) == npp // 8
    live = sorted_ids[sorted_ids < numel]
    assert sorted(live.tolist()) == list(range(numel))
    flat = ids.reshape(-1)
    for b, e in enumerate(block_expert.tolist()):
        blk = sorted_ids[b * 8:(b + 1) * 8]
        blk = blk[blk < numel]
        assert (flat[blk.long()] == e).all()
