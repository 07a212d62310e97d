"""AWQ MoE wiring on the CPU: a tiny synthetic AWQ MoE checkpoint goes through
the restated loader rules (model_loader/weight_loader.py:40-69,121-142: shard,
merge gate | up on the packed columns, stack experts) into the AWQ MoE layer's
state dict (layers/moe_layer.py:37-47 with AWQ tensors)."""

import pytest
import torch

from sglite_b200.moe import AWQMoELayer, stack_awq_experts
from sglite_b200.quantization import AWQB200Config
from sglite_b200.synthetic import make_awq_weights

E, H, I, G = 4, 256, 128, 64
PREFIX = "model.layers.0.mlp.experts"


def _checkpoint(seed=0):
    ck = {}
    for e in range(E):
        for proj, (K, N) in (("gate_proj", (H, I)), ("up_proj", (H, I)), ("down_proj", (I, H))):
            w = make_awq_weights(K, N, G, torch.bfloat16, seed=seed + 10 * e + len(proj))
            for k, v in w.items():
                ck[f"{PREFIX}.{e}.{proj}.{k}"] = v
    ck["model.layers.0.mlp.gate.weight"] = torch.zeros(E, H)  # not an expert tensor: passes through
    return ck


@pytest.mark.parametrize("world", [1, 2])
def test_stacking_follows_the_loader_rules(world):
    ck = _checkpoint()
    for rank in range(world):
        st = stack_awq_experts(ck, E, rank, world)
        gu, dn = f"{PREFIX}.gate_up_proj", f"{PREFIX}.down_proj"
        assert st[f"{gu}.qweight"].shape == (E, H, 2 * I // world // 8)
        assert st[f"{gu}.qzeros"].shape == (E, H // G, 2 * I // world // 8)
        assert st[f"{gu}.scales"].shape == (E, H // G, 2 * I // world)
        assert st[f"{dn}.qweight"].shape == (E, I // world, H // 8)
        assert st[f"{dn}.qzeros"].shape == (E, I // world // G, H // 8)
        assert st[f"{dn}.scales"].shape == (E, I // world // G, H)
        for e in range(E):
            for k in ("qweight", "qzeros", "scales"):
                g = ck[f"{PREFIX}.{e}.gate_proj.{k}"].chunk(world, dim=1)[rank]
                u = ck[f"{PREFIX}.{e}.up_proj.{k}"].chunk(world, dim=1)[rank]
                assert torch.equal(st[f"{gu}.{k}"][e], torch.cat([g, u], dim=1))
                d = ck[f"{PREFIX}.{e}.down_proj.{k}"].chunk(world, dim=0)[rank]
                assert torch.equal(st[f"{dn}.{k}"][e], d)
        assert "model.layers.0.mlp.gate.weight" in st


def test_layer_state_dict_matches_the_loader_keys():
    cfg = AWQB200Config(4, G, True)
    for tp in (1, 2):
        layer = AWQMoELayer(E, 2, H, I, cfg, tp_size=tp)
        st = stack_awq_experts(_checkpoint(), E, 0, tp)
        st.pop("model.layers.0.mlp.gate.weight")
        assert sorted(layer.state_dict(prefix=PREFIX)) == sorted(st)
        layer.load_state_dict(dict(st), prefix=PREFIX)
        assert torch.equal(layer.gate_up_proj.qweight, st[f"{PREFIX}.gate_up_proj.qweight"])


def test_layer_rejects_mismatched_or_unexpected_tensors():
    cfg = AWQB200Config(4, G, True)
    layer = AWQMoELayer(E, 2, H, I, cfg)
    st = stack_awq_experts(_checkpoint(), E)
    st.pop("model.layers.0.mlp.gate.weight")
    bad = dict(st)
    bad[f"{PREFIX}.down_proj.scales"] = bad[f"{PREFIX}.down_proj.scales"][:, :1]
    with pytest.raises(ValueError):
        layer.load_state_dict(bad, prefix=PREFIX)
    extra = dict(st)
    extra["unexpected"] = torch.zeros(1)
    with pytest.raises(RuntimeError):
        AWQMoELayer(E, 2, H, I, cfg).load_state_dict(extra, prefix=PREFIX)
    with pytest.raises(ValueError):
        stack_awq_experts({k: v for k, v in _checkpoint().items() if ".3." not in k}, E)
    with pytest.raises(ValueError):
        AWQMoELayer(E, 2, H, I, cfg, ep_size=3)
