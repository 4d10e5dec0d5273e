"""vLLM quantization config "espalier" over this library (the reference's vllm_espalier/config.py:54-133).

Which modules are trellis-coded is read from the checkpoint (checkpoint.Checkpoint: every `.esp_trellis` key) when
vLLM calls maybe_update_config with the model path. Coded dense layers and the LM head get EspLinearMethod (linear.py,
the fused dense kernel through espalier::dense), coded routed experts EspMoEMethod (moe.py, the grouped pipeline);
everything else stays unquantized. Importing this module needs vLLM; the rest of the package does not.
"""
from __future__ import annotations

from pathlib import Path
from typing import Any

import torch
from vllm.model_executor.layers.linear import LinearBase, UnquantizedLinearMethod
from vllm.model_executor.layers.quantization import register_quantization_config
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig

from .checkpoint import NAME, PACKED, Checkpoint, check_quant_config


def checkpoint_dir(model_name: str, revision: str | None = None) -> Path:
    """A local checkpoint directory as given, else the Hub snapshot of its JSON files (config.py:44-51)."""
    p = Path(model_name)
    if p.is_dir():
        return p
    from huggingface_hub import snapshot_download
    return Path(snapshot_download(model_name, revision=revision, allow_patterns=["*.json"]))


@register_quantization_config(NAME)
class EspalierConfig(QuantizationConfig):
    def __init__(self, raw: dict[str, Any] | None = None):
        super().__init__()
        self.raw = dict(raw or {})
        self.packed_modules_mapping = dict(PACKED)
        self.exl3: set[str] = set()          # text keys of the checkpoint's coded matrices
        self.checkpoint: Path | None = None
        self._ck: Checkpoint | None = None

    def get_name(self) -> str:
        return NAME

    def get_supported_act_dtypes(self) -> list[torch.dtype]:
        return [torch.bfloat16, torch.float16]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100                            # the kernels are built for sm_100a only

    @staticmethod
    def get_config_filenames() -> list[str]:
        return []

    @classmethod
    def from_config(cls, config: dict[str, Any]) -> "EspalierConfig":
        check_quant_config(config)
        return cls(config)

    @classmethod
    def override_quantization_method(cls, hf_quant_cfg, user_quant, hf_config=None):
        return NAME if str((hf_quant_cfg or {}).get("quant_method", "")).lower() == NAME else None

    def maybe_update_config(self, model_name: str, hf_config=None, revision: str | None = None):
        d = checkpoint_dir(model_name, revision)
        self._ck = Checkpoint(d)
        self.exl3 = self._ck.exl3
        self.checkpoint = d

    def is_exl3(self, prefix: str) -> bool:
        return self._ck is not None and self._ck.is_exl3(prefix)

    def experts_exl3(self, prefix: str) -> bool:
        return self._ck is not None and self._ck.experts_exl3(prefix)

    def get_quant_method(self, layer: torch.nn.Module, prefix: str):
        from vllm.model_executor.layers.vocab_parallel_embedding import ParallelLMHead
        from .linear import EspLinearMethod
        try:
            from vllm.model_executor.layers.fused_moe import RoutedExperts
        except ImportError:
            RoutedExperts = ()
        if RoutedExperts and isinstance(layer, RoutedExperts):
            if not self.experts_exl3(prefix):
                raise ValueError(f"{prefix}: routed experts without EXL3 tensors")
            from .moe import EspMoEMethod
            return EspMoEMethod(layer.moe_config)
        if isinstance(layer, ParallelLMHead):
            return EspLinearMethod(prefix) if self.is_exl3(prefix) else None
        if isinstance(layer, LinearBase):
            return EspLinearMethod(prefix) if self.is_exl3(prefix) else UnquantizedLinearMethod()
        return None
