"""Host-side checks that need no GPU: the C-ABI library loads and exports every
declared symbol, argument validation reports errors through status codes, and
the linear-method boundary mirrors the reference's interface."""

import ctypes
import os
import re

import pytest
import torch

from sglite_b200 import _lib
from sglite_b200.quantization import AWQB200Config, AWQB200LinearMethod, get_quantization_config, select_awq_config

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "awqb200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(awqb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 25
    for name in names:
        assert hasattr(lib, name), name
    # and the ctypes binding covers exactly the declared API
    assert set(_lib.EXPORTED) == set(names)


def test_abi_version_and_sizes():
    lib = _lib.lib()
    assert lib.awqb_abi_version() == 1
    out = ctypes.c_int64(0)
    assert lib.awqb_blob_bytes(4096, 4096, 128, ctypes.byref(out)) == 0
    # 32 feature tiles x 32 k-blocks x (8192 + 320) bytes
    assert out.value == 32 * 32 * 8512
    assert lib.awqb_gemm_workspace_bytes(16, 4096, 4096, 128, ctypes.byref(out)) == 0
    assert out.value > 0


@pytest.mark.parametrize("K,N,G,code", [(4096, 4096, 100, 2), (4096, 4100, 128, 1), (4000, 4096, 128, 1)])
def test_invalid_shapes_return_status_and_message(K, N, G, code):
    lib = _lib.lib()
    out = ctypes.c_int64(0)
    assert lib.awqb_blob_bytes(K, N, G, ctypes.byref(out)) == code
    assert len(lib.awqb_last_error()) > 0
    with pytest.raises(ValueError):
        _lib.check(code)


def test_gemm_rejects_bad_arguments_without_touching_the_gpu():
    lib = _lib.lib()
    # bad dtype
    assert lib.awqb_gemm(None, 1, 4096, 4096, 128, 7, None, None, None, None, 0, None) == 1
    # null pointers
    assert lib.awqb_gemm(None, 1, 4096, 4096, 128, 1, None, None, None, None, 0, None) == 1
    # misaligned activations
    assert lib.awqb_gemm(ctypes.c_void_p(8), 1, 4096, 4096, 128, 1, ctypes.c_void_p(256), None,
                         ctypes.c_void_p(256), ctypes.c_void_p(256), 1 << 30, None) == 1
    assert b"16-byte" in lib.awqb_last_error()
    # workspace too small (M > 32: the tcgen05 kernel, which needs one)
    assert lib.awqb_gemm(ctypes.c_void_p(256), 33, 4096, 4096, 128, 1, ctypes.c_void_p(256), None,
                         ctypes.c_void_p(256), ctypes.c_void_p(256), 64, None) == 1
    assert b"workspace too small" in lib.awqb_last_error()


def test_gemv_rejects_bad_arguments_without_touching_the_gpu():
    lib = _lib.lib()
    p = ctypes.c_void_p(256)
    # feature slice / warp count not built, ring depth out of range, too many rows
    assert lib.awqb_gemv_ex(p, 4, 4096, 4096, 128, 1, p, None, p, 24, 0, 0, 0, None) == 1
    assert b"feature slice" in lib.awqb_last_error()
    assert lib.awqb_gemv_ex(p, 4, 4096, 4096, 128, 1, p, None, p, 0, 12, 0, 0, None) == 1
    assert lib.awqb_gemv_ex(p, 4, 4096, 4096, 128, 1, p, None, p, 0, 0, 17, 0, None) == 1
    assert lib.awqb_gemv_ex(p, 33, 4096, 4096, 128, 1, p, None, p, 0, 0, 0, 0, None) == 1
    assert b"1..32 rows" in lib.awqb_last_error()
    assert lib.awqb_gemv_ex(p, 4, 4096, 4096, 128, 1, p, None, p, 64, 16, 0, 0, None) == 2
    # SiLU-and-mul needs N % 16 == 0; misaligned activations; bad group size
    assert lib.awqb_gemv_ex(p, 4, 4096, 4104, 128, 1, p, None, p, 0, 0, 0, 1, None) == 1
    assert lib.awqb_gemv_ex(ctypes.c_void_p(8), 4, 4096, 4096, 128, 1, p, None, p, 0, 0, 0, 0, None) == 1
    assert b"16-byte" in lib.awqb_last_error()
    assert lib.awqb_gemv_ex(p, 4, 4096, 4096, 96, 1, p, None, p, 0, 0, 0, 0, None) == 2


def test_norm_rejects_bad_arguments_without_touching_the_gpu():
    lib = _lib.lib()
    # N not a multiple of 8, N over the register-resident maximum
    assert lib.awqb_rmsnorm(None, None, None, 1, 12, 12, 12, 1e-6, 1, None) == 1
    assert lib.awqb_rmsnorm(None, None, None, 1, 16392, 16392, 16392, 1e-6, 1, None) == 1
    # row stride below N
    assert lib.awqb_fused_add_rmsnorm(None, None, None, 1, 4096, 2048, 4096, 1e-6, 1, None) == 1
    # null pointers, misaligned input
    assert lib.awqb_fused_add_rmsnorm(None, None, None, 1, 4096, 4096, 4096, 1e-6, 1, None) == 1
    assert lib.awqb_rmsnorm(ctypes.c_void_p(8), ctypes.c_void_p(256), ctypes.c_void_p(256), 1, 4096, 4096, 4096,
                            1e-6, 1, None) == 1
    assert b"16-byte" in lib.awqb_last_error()
    # no rows: nothing to do
    assert lib.awqb_rmsnorm(None, None, None, 0, 4096, 4096, 4096, 1e-6, 1, None) == 0


def test_moe_align_ex_checks_its_workspace_without_touching_the_gpu():
    lib = _lib.lib()
    need = lib.awqb_moe_align_workspace_bytes(32768, 128)
    assert need == 32 * 128 * 4  # one count per (1024-pair chunk, expert)
    p = ctypes.c_void_p(256)
    assert lib.awqb_moe_align_ex(p, 32768, 0, 128, 128, p, 32768 + 128 * 127, p, p, p, need - 4, None) == 1
    assert b"workspace too small" in lib.awqb_last_error()
    assert lib.awqb_moe_align_ex(p, 32768, 0, 128, 128, p, 100, p, p, p, need, None) == 1  # sorted_ids too small
    assert lib.awqb_moe_align_ex(p, 32768, 0, 1024, 128, p, 1 << 20, p, p, p, need, None) == 1  # too many experts


def test_norm_layers_mirror_reference_interface():
    from sglite_b200.norm import RMSNorm, RMSNormFused

    for cls in (RMSNorm, RMSNormFused):
        layer = cls(4096, 1e-6)
        assert layer.weight.shape == (4096,) and layer.eps == 1e-6
    assert hasattr(RMSNorm, "forward_inplace")


def test_config_matches_reference_semantics():
    cfg = AWQB200Config.from_config({"w_bit": 4, "q_group_size": 128, "zero_point": True})
    assert cfg.get_name() == "awq_b200" and cfg.pack_factor == 8
    assert torch.bfloat16 in cfg.get_supported_act_dtypes() and torch.half in cfg.get_supported_act_dtypes()
    assert cfg.get_min_capability() == 100
    assert cfg.get_config_filenames() == ["quant_config.json", "quantize_config.json"]
    with pytest.raises(ValueError):
        AWQB200Config(8, 128, True)       # only 4-bit (awq.py:19-23)
    with pytest.raises(ValueError):
        AWQB200Config(4, 48, True)
    with pytest.raises(ValueError):
        AWQB200Config.from_config({"bits": 4})  # missing keys (base_config.py:76-81)
    assert get_quantization_config("AWQ_B200") is AWQB200Config
    with pytest.raises(ValueError):
        get_quantization_config("gptq")
    assert AWQB200Config.is_awq_b200_compatible({"quant_method": "awq", "bits": 4, "group_size": 64, "zero_point": True})
    assert not AWQB200Config.is_awq_b200_compatible({"quant_method": "gptq", "bits": 4, "group_size": 64, "zero_point": True})
    assert isinstance(select_awq_config({"quant_method": "awq", "w_bit": 4, "q_group_size": 128, "zero_point": True}),
                      AWQB200Config)


def test_create_weights_mirrors_awq_tensors_and_attrs():
    m = AWQB200Config(4, 128, True).get_linear_method()
    assert isinstance(m, AWQB200LinearMethod)
    w = m.create_weights(4096, 6144)
    assert w["qweight"].shape == (4096, 768) and w["qweight"].dtype == torch.int32
    assert w["qzeros"].shape == (32, 768) and w["qzeros"].dtype == torch.int32
    assert w["scales"].shape == (32, 6144)
    for k in ("qweight", "qzeros"):
        assert (w[k].input_dim, w[k].output_dim, w[k].packed_dim, w[k].pack_factor) == (0, 1, 1, 8)
    assert (w["scales"].input_dim, w["scales"].output_dim) == (0, 1)
    assert w["_input_size"] == 4096 and w["_output_size"] == 6144 and w["_group_size"] == 128
    with pytest.raises(ValueError):
        m.create_weights(4000, 6144)   # K not a multiple of the group size
    with pytest.raises(ValueError):
        m.create_weights(4096, 6100)   # N not a multiple of the pack factor
    # channel-wise quantisation: group = input size
    mc = AWQB200Config(4, -1, True).get_linear_method()
    assert mc.create_weights(1024, 256)["_group_size"] == 1024


def test_process_weights_requires_cuda_and_apply_requires_processing():
    m = AWQB200Config(4, 128, True).get_linear_method()
    w = m.create_weights(256, 128)
    with pytest.raises(RuntimeError):
        m.process_weights_after_loading(w)
    with pytest.raises(RuntimeError):
        m.apply_weights(w, torch.zeros(1, 256))


def test_interleave_gate_up_is_a_column_permutation():
    """Interleaving moves nibbles, never changes them: column 2j of the result
    dequantises to gate column j, column 2j + 1 to up column j."""
    import torch
    from oracle.awq_ref import dequant_ref
    from sglite_b200 import ops
    from sglite_b200.synthetic import make_awq_weights

    K, I, G = 256, 192, 128
    w = make_awq_weights(K, 2 * I, G, torch.float16, seed=3)
    qw, qz, sc = ops.interleave_gate_up(w["qweight"], w["qzeros"], w["scales"])
    Wi = dequant_ref(qw, qz, sc, G)
    W = dequant_ref(w["qweight"], w["qzeros"], w["scales"], G)
    cols = [c for j in range(I) for c in (j, I + j)]
    assert torch.equal(Wi, W[:, cols])
