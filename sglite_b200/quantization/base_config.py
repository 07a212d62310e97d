"""Linear-method / quantization-config interface.

When SGLite is importable, its own base classes are used, so the classes in
this package are drop-in subclasses of
``sglite.srt.model_executor.layers.quantization.base_config`` (reference
``layers/quantization/base_config.py:9-91``). Otherwise an equivalent
interface with the same names, signatures and error behaviour is defined here.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Any, Dict, List, Optional

import torch

try:  # pragma: no cover - depends on the host environment
    from sglite.srt.model_executor.layers.quantization.base_config import (  # type: ignore
        LinearMethodBase,
        QuantizationConfig,
        set_weight_attrs,
    )
except Exception:  # SGLite not installed: standalone interface

    def set_weight_attrs(weight: torch.Tensor, weight_attrs: Optional[Dict[str, Any]]) -> None:
        """Attach loader metadata to a weight tensor without overwriting fields."""
        if weight_attrs is None:
            return
        for key, value in weight_attrs.items():
            if hasattr(weight, key):
                raise RuntimeError(f"Overwriting existing attribute {key} on weight tensor.")
            setattr(weight, key, value)

    class LinearMethodBase(ABC):  # type: ignore[no-redef]
        """Base class for quantized linear-method implementations."""

        @abstractmethod
        def create_weights(self, input_size: int, output_size: int) -> Dict[str, Any]:
            raise NotImplementedError

        @abstractmethod
        def apply_weights(self, weights: Dict[str, Any], x: torch.Tensor,
                          bias: Optional[torch.Tensor] = None) -> torch.Tensor:
            raise NotImplementedError

        def process_weights_after_loading(self, weights: Dict[str, Any]) -> Dict[str, Any]:
            return weights

    class QuantizationConfig(ABC):  # type: ignore[no-redef]
        """Configuration container for a quantization scheme."""

        @abstractmethod
        def get_name(self) -> str:
            raise NotImplementedError

        @abstractmethod
        def get_supported_act_dtypes(self) -> List[torch.dtype]:
            raise NotImplementedError

        @abstractmethod
        def get_min_capability(self) -> int:
            raise NotImplementedError

        @staticmethod
        @abstractmethod
        def get_config_filenames() -> List[str]:
            raise NotImplementedError

        @classmethod
        @abstractmethod
        def from_config(cls, config: Dict[str, Any]) -> "QuantizationConfig":
            raise NotImplementedError

        @staticmethod
        def get_from_keys(config: Dict[str, Any], keys: List[str]) -> Any:
            for key in keys:
                if key in config:
                    return config[key]
            raise ValueError(f"Cannot find any of {keys} in the model's quantization config.")

        @abstractmethod
        def get_linear_method(self) -> LinearMethodBase:
            raise NotImplementedError

        @abstractmethod
        def get_scaled_act_names(self) -> List[str]:
            raise NotImplementedError


__all__ = ["LinearMethodBase", "QuantizationConfig", "set_weight_attrs"]
