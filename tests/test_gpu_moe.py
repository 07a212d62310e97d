"""MoE path on the GPU: routing and expert sort against the oracle (exact),
the whole AWQ expert pipeline against the oracle and the reference's own
kernels' outputs, expert-parallel partition, and the Qwen3-30B-A3B shape."""

import pytest
import torch

from oracle.awq_ref import moe_align_ref, moe_ref, rel_err, topk_softmax_ref
from sglite_b200 import ops
from sglite_b200.moe import AWQB200MoeBackend, AWQExpertWeights
from sglite_b200.synthetic import make_activations, make_awq_weights, make_router_logits

pytestmark = pytest.mark.gpu

TOL = 1e-2


@pytest.mark.parametrize("M,E,k", [(1, 128, 8), (37, 128, 8), (300, 16, 4), (5, 8, 2)])
@pytest.mark.parametrize("renorm", [True, False])
def test_topk_softmax_matches_oracle(cuda, M, E, k, renorm):
    lg = make_router_logits(M, E, seed=M + E)
    w, ids = ops.moe_topk_softmax(lg.to(cuda), k, renorm)
    w_ref, ids_ref = topk_softmax_ref(lg, k, renorm)
    assert torch.equal(ids.cpu(), ids_ref)
    assert torch.allclose(w.cpu(), w_ref, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("M,E,k,bm", [(1, 128, 8, 16), (16, 128, 8, 16), (256, 128, 8, 32), (999, 16, 4, 64),
                                      (4096, 128, 8, 128), (2050, 64, 8, 64)])
@pytest.mark.parametrize("ep", [None, (4, 12)])
@pytest.mark.parametrize("multi", [False, True])
def test_align_matches_oracle_exactly(cuda, M, E, k, bm, ep, multi):
    """Both sorts (one CTA; chunk histograms + scan + per-chunk scatter) give the
    oracle's stable order, padding and block experts."""
    ids = torch.stack([torch.randperm(E, generator=torch.Generator().manual_seed(i))[:k] for i in range(M)]).to(torch.int32)
    e0, e1 = ep if ep is not None else (0, E)
    sorted_ids, block_expert, npp = ops.moe_align(ids.to(cuda), e0, e1, bm, multi_cta=multi)
    s_ref, b_ref, n_ref = moe_align_ref(ids, bm, e0, e1)
    n = int(npp.item())
    assert n == n_ref
    assert torch.equal(sorted_ids[:n].cpu(), s_ref)
    assert torch.equal(block_expert[: n // bm].cpu(), b_ref)
    assert (sorted_ids[n:] == ids.numel()).all()  # unused tail carries the sentinel


def _experts(E, H, I, G, dtype, seed, cuda, fused=True):
    w1 = make_awq_weights(H, 2 * I, G, dtype, seed=seed, batch=E)
    w2 = make_awq_weights(I, H, G, dtype, seed=seed + 1, batch=E)
    e1 = AWQExpertWeights.from_awq(*(w1[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G, gate_up=fused)
    e2 = AWQExpertWeights.from_awq(*(w2[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G)
    assert e1.gate_up_interleaved == fused
    return w1, w2, e1, e2


@pytest.mark.parametrize("M", [1, 7, 64, 300])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("fused", [False, True])
def test_moe_pipeline_matches_oracle(cuda, M, dtype, fused):
    """fused: SiLU-and-mul inside the gate_up GEMM's epilogue (interleaved w1)."""
    E, k, H, I, G = 16, 4, 256, 128, 128
    w1, w2, e1, e2 = _experts(E, H, I, G, dtype, 11, cuda, fused)
    x = make_activations(M, H, dtype, seed=M)
    lg = make_router_logits(M, E, seed=M + 1)
    y = AWQB200MoeBackend().forward(x.to(cuda).clone(), e1, e2, lg.to(cuda), k, True)
    ref = moe_ref(x, w1, w2, lg, k, True, G)
    assert rel_err(y, ref.float()) <= TOL


def test_moe_expert_parallel_sum_equals_full(cuda):
    E, k, H, I, G, M = 16, 4, 256, 128, 128, 40
    dtype = torch.bfloat16
    w1 = make_awq_weights(H, 2 * I, G, dtype, seed=5, batch=E)
    w2 = make_awq_weights(I, H, G, dtype, seed=6, batch=E)
    x = make_activations(M, H, dtype, seed=7).to(cuda)
    lg = make_router_logits(M, E, seed=8).to(cuda)
    parts = []
    for e0, e1_ in ((0, 8), (8, 16)):
        sl = slice(e0, e1_)
        a = AWQExpertWeights.from_awq(*(w1[k_][sl].to(cuda) for k_ in ("qweight", "qzeros", "scales")), G, e0, E)
        b = AWQExpertWeights.from_awq(*(w2[k_][sl].to(cuda) for k_ in ("qweight", "qzeros", "scales")), G, e0, E)
        parts.append(AWQB200MoeBackend().forward(x.clone(), a, b, lg, k, True).float())
    ref = moe_ref(x.cpu(), w1, w2, lg.cpu(), k, True, G)
    assert rel_err(parts[0] + parts[1], ref.float()) <= TOL
    # each rank on its own matches the oracle restricted to its experts
    ref0 = moe_ref(x.cpu(), w1, w2, lg.cpu(), k, True, G, 0, 8)
    assert rel_err(parts[0], ref0.float()) <= TOL


def test_moe_matches_reference_kernels_golden(cuda, golden):
    E, topk, H, I, M, BM, G = (int(v) for v in golden["moe_shape"])
    w1 = {k: torch.from_numpy(golden["moe_w1_" + k]) for k in ("qweight", "qzeros", "scales")}
    w2 = {k: torch.from_numpy(golden["moe_w2_" + k]) for k in ("qweight", "qzeros", "scales")}
    w1["scales"] = w1["scales"].view(torch.float16)
    w2["scales"] = w2["scales"].view(torch.float16)
    e1 = AWQExpertWeights.from_awq(*(w1[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G, gate_up=True)
    e2 = AWQExpertWeights.from_awq(*(w2[k].to(cuda) for k in ("qweight", "qzeros", "scales")), G)
    x = torch.from_numpy(golden["moe_x"]).view(torch.float16)
    lg = torch.from_numpy(golden["moe_logits"])
    y = AWQB200MoeBackend().forward(x.to(cuda).clone(), e1, e2, lg.to(cuda), topk, True)
    y_kernel = torch.from_numpy(golden["moe_y"]).view(torch.float16)
    assert rel_err(y, y_kernel.float()) <= TOL


@pytest.mark.parametrize("M", [16, 256])
def test_qwen3_30b_a3b_moe_shape(cuda, M):
    E, k, H, I, G = 128, 8, 2048, 768, 128
    dtype = torch.bfloat16
    w1, w2, e1, e2 = _experts(E, H, I, G, dtype, 21, cuda)
    x = make_activations(M, H, dtype, seed=M)
    lg = make_router_logits(M, E, seed=M + 3)
    y = AWQB200MoeBackend().forward(x.to(cuda).clone(), e1, e2, lg.to(cuda), k, True)
    ref = moe_ref(x, w1, w2, lg, k, True, G)
    assert rel_err(y, ref.float()) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("interleaved", [False, True])
def test_silu_and_mul_layouts(cuda, interleaved):
    from oracle.awq_ref import silu_and_mul_ref

    rows, I = 37, 136
    h = torch.randn(rows, 2 * I, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    plain = torch.cat([h[:, 0::2], h[:, 1::2]], dim=1) if interleaved else h
    out = ops.silu_and_mul(h.to(cuda), interleaved=interleaved)
    assert torch.allclose(out.float().cpu(), silu_and_mul_ref(plain).float(), rtol=1e-2, atol=1e-2)


def test_awq_moe_layer_from_a_checkpoint_against_the_oracle(cuda):
    """The wiring end to end: a synthetic AWQ MoE checkpoint stacked by the
    restated loader rules, loaded into the AWQ MoE layer, repacked, and run
    against the oracle's MoE restatement; then the same experts split over two
    expert-parallel layers (one process), whose summed outputs must match."""
    from oracle.awq_ref import moe_ref, rel_err
    from sglite_b200.moe import AWQMoELayer, stack_awq_experts
    from sglite_b200.quantization import AWQB200Config
    from sglite_b200.synthetic import make_activations, make_awq_weights, make_router_logits

    E, k, H, I, G, M = 8, 2, 512, 256, 128, 40
    prefix = "model.layers.3.mlp.experts"
    ck = {}
    for e in range(E):
        for proj, (K, N) in (("gate_proj", (H, I)), ("up_proj", (H, I)), ("down_proj", (I, H))):
            for kk, v in make_awq_weights(K, N, G, torch.bfloat16, seed=7 * e + len(proj)).items():
                ck[f"{prefix}.{e}.{proj}.{kk}"] = v
    st = stack_awq_experts(ck, E)
    cfg = AWQB200Config(4, G, True)
    x = make_activations(M, H, torch.bfloat16, seed=1)
    logits = make_router_logits(M, E, seed=2)
    w1 = {kk: st[f"{prefix}.gate_up_proj.{kk}"] for kk in ("qweight", "qzeros", "scales")}
    w2 = {kk: st[f"{prefix}.down_proj.{kk}"] for kk in ("qweight", "qzeros", "scales")}
    ref = moe_ref(x, w1, w2, logits, k, True, G)

    layer = AWQMoELayer(E, k, H, I, cfg)
    layer.load_state_dict({kk: v.to(cuda) for kk, v in st.items()}, prefix=prefix)
    layer.process_weights_after_loading()
    y = layer.forward(x.to(cuda).clone(), logits.to(cuda))
    assert rel_err(y, ref) <= 1e-2

    parts = []
    for r in range(2):
        lr = AWQMoELayer(E, k, H, I, cfg, ep_rank=r, ep_size=2)
        lr.load_state_dict({kk: v.to(cuda) for kk, v in st.items()}, prefix=prefix)
        lr.process_weights_after_loading()
        parts.append(lr.forward(x.to(cuda).clone(), logits.to(cuda)).float())
    assert rel_err(parts[0] + parts[1], ref) <= 1e-2
    assert ops.device_error() == 0


def _vllm_ops():
    try:
        import vllm._custom_ops as vops  # noqa: F401
    except Exception as e:  # pragma: no cover - depends on the image
        pytest.skip(f"vllm custom ops unavailable: {e}")
    return vops


@pytest.mark.parametrize("M,E,k", [(1, 128, 8), (37, 128, 8), (300, 16, 4), (4096, 128, 8)])
@pytest.mark.parametrize("renorm", [True, False])
def test_topk_softmax_matches_vllm(cuda, M, E, k, renorm):
    """The reference's fused_topk (fused.py:11-31) calls sgl-kernel's
    topk_softmax, which is absent here; vllm's topk_softmax (installed on the
    GPU image) implements the same routing kernel. With the reference's Python
    renormalisation after it, ids must match exactly and weights to 1e-6."""
    vops = _vllm_ops()
    lg = make_router_logits(M, E, seed=M * 3 + E).to(cuda)
    w_v = torch.empty((M, k), dtype=torch.float32, device=cuda)
    i_v = torch.empty((M, k), dtype=torch.int32, device=cuda)
    tei = torch.empty((M, k), dtype=torch.int32, device=cuda)
    try:
        vops.topk_softmax(w_v, i_v, tei, lg.float(), renorm)
        torch.cuda.synchronize()
    except Exception as e:  # pragma: no cover
        pytest.skip(f"vllm topk_softmax failed to run here: {e}")
    if renorm:
        w_v = w_v / (w_v.sum(dim=-1, keepdim=True) + 1e-8)
    w, ids = ops.moe_topk_softmax(lg, k, renorm)
    assert torch.equal(ids.cpu(), i_v.cpu())
    assert torch.allclose(w.cpu(), w_v.cpu(), rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("M,E,k,bm", [(1, 128, 8, 16), (256, 128, 8, 32), (4096, 128, 8, 128), (999, 16, 4, 64)])
def test_align_matches_vllm(cuda, M, E, k, bm):
    """moe_align_block_size (fused.py:34-61; sgl-kernel, absent) against
    vllm's kernel of the same name: identical padded length and block experts,
    and every expert's padded region (its consecutive blocks) holds the same
    pair indices (the order inside a region is the kernel's own: ours is
    stable, which the oracle tests check; vllm's is not)."""
    vops = _vllm_ops()
    ids = torch.stack([torch.randperm(E, generator=torch.Generator().manual_seed(i))[:k]
                       for i in range(M)]).to(torch.int32).to(cuda)
    numel = ids.numel()
    cap = numel + E * (bm - 1)
    s_v = torch.full((cap,), numel, dtype=torch.int32, device=cuda)
    e_v = torch.zeros(((cap + bm - 1) // bm,), dtype=torch.int32, device=cuda)
    n_v = torch.zeros((1,), dtype=torch.int32, device=cuda)
    try:
        vops.moe_align_block_size(ids, E, bm, s_v, e_v, n_v)
        torch.cuda.synchronize()
    except Exception as e:  # pragma: no cover
        pytest.skip(f"vllm moe_align_block_size failed to run here: {e}")
    sorted_ids, block_expert, npp = ops.moe_align(ids, 0, E, bm)
    n = int(npp.item())
    assert n == int(n_v.item())
    assert torch.equal(block_expert[: n // bm].cpu(), e_v[: n // bm].cpu())
    ours, theirs = sorted_ids[:n].cpu(), s_v[:n].cpu()
    be = block_expert[: n // bm].cpu().tolist()
    b0 = 0
    while b0 < len(be):  # one expert's consecutive blocks at a time
        b1 = b0
        while b1 < len(be) and be[b1] == be[b0]:
            b1 += 1
        a, c = ours[b0 * bm:b1 * bm], theirs[b0 * bm:b1 * bm]
        assert torch.equal(torch.sort(a).values, torch.sort(c).values), be[b0]
        b0 = b1
    assert ops.device_error() == 0
