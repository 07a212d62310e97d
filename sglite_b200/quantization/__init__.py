"""Quantization registry for the B200 AWQ path.

``get_quantization_config`` mirrors the reference's registry
(``layers/quantization/__init__.py:15-29``) and adds ``"awq_b200"``;
``select_awq_config`` mirrors ``_create_awq_config``
(``model_executor/models/config.py:73-89``) with the B200 method first.
"""

from __future__ import annotations

from typing import Any, Dict

from .base_config import LinearMethodBase, QuantizationConfig, set_weight_attrs


def get_quantization_config(method_name: str) -> type:
    """Return the quantization config class for a method name."""
    name = method_name.lower()
    if name == "awq_b200":
        from .awq_b200 import AWQB200Config

        return AWQB200Config
    raise ValueError(f"Unknown quantization method: {method_name!r}. Supported methods: ['awq_b200']")


def select_awq_config(config_dict: Dict[str, Any]):
    """Pick the B200 AWQ config for compatible AWQ metadata, else raise.

    The reference falls back from Marlin to its Triton kernel; on B200 this
    package has a single backend, so an incompatible config is an error.
    """
    from .awq_b200 import AWQB200Config

    if not AWQB200Config.is_awq_b200_compatible(config_dict):
        raise ValueError(f"AWQ metadata {config_dict} is not supported by the B200 kernels")
    return AWQB200Config.from_config(config_dict)


def __getattr__(name: str):
    if name in ("AWQB200Config", "AWQB200LinearMethod"):
        from . import awq_b200

        return getattr(awq_b200, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


__all__ = [
    "AWQB200Config",
    "AWQB200LinearMethod",
    "LinearMethodBase",
    "QuantizationConfig",
    "get_quantization_config",
    "select_awq_config",
    "set_weight_attrs",
]
