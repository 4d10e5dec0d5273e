"""Espalier checkpoints: which modules are trellis-coded, and loading their tensors, without vLLM.

The reference splits this between its vLLM quantization config and its loaders:
  * key discovery (vllm_espalier/config.py:21-52, 90-121): every checkpoint key ending in `.esp_trellis` names a coded
    matrix; `text_key` maps checkpoint and vLLM module names to one namespace ('layers.N.<...>', 'mtp.layers.N.<...>'
    or 'lm_head'; vision modules are never coded); a vLLM layer that fuses several checkpoint matrices (PACKED) is
    coded if all of them are, and a partly coded fused layer is an error;
  * the tensors of one matrix (matrix.py:3-6, 19-37): esp_trellis, suh, svh, mcg, optionally mul1 or esp_grid, read
    from the shard the index names (tests/gpu_dense.py:40-59, tests/gpu_grouped.py:46-70);
  * a fused layer's matrices in vLLM's shard order (linear.py:28-36, 72-73) and an MoE layer's per-expert
    (gate, up, down) triples, every expert required (moe.py:50, 86-106).
This module does the same from a checkpoint directory (`model.safetensors.index.json` and its shards, or a single
`model.safetensors`), so a host that builds Dense / experts.prepare layers itself needs no vLLM.
"""
from __future__ import annotations

import json
import re
from pathlib import Path

import torch

from .matrix import SUFFIXES, EspMatrix

NAME = "espalier"
TRELLIS = ".esp_trellis"
INDEX = "model.safetensors.index.json"
SINGLE = "model.safetensors"
# vLLM fused layer -> the checkpoint matrices it holds, in output order
PACKED = {
    "qkv_proj": ["q_proj", "k_proj", "v_proj"],
    "gate_up_proj": ["gate_proj", "up_proj"],
    "in_proj_qkvz": ["in_proj_qkv", "in_proj_z"],
    "in_proj_ba": ["in_proj_b", "in_proj_a"],
}
PROJS = ("gate_proj", "up_proj", "down_proj")
_LAYER = re.compile(r"(?:^|\.)(mtp\.)?(layers\.\d+\..+)$")


def text_key(name: str) -> str | None:
    """Checkpoint or vLLM module name -> 'layers.N.<...>', 'mtp.layers.N.<...>' or 'lm_head' for the text model, else
    None (vision modules, and names outside the decoder layers). The MTP head's layers keep their own namespace, so
    they never alias the decoder's layer N."""
    if "visual" in name or "vision" in name:
        return None
    if name.endswith("lm_head") or ".lm_head." in name + ".":
        return "lm_head"
    m = _LAYER.search(name)
    return (m.group(1) or "") + m.group(2) if m else None


def check_quant_config(config: dict) -> None:
    """Raise unless a checkpoint's quantization_config names this method (config.py:78-82)."""
    method = str((config or {}).get("quant_method", "")).lower()
    if method != NAME:
        raise ValueError(f"not an {NAME} checkpoint: {config.get('quant_method') if config else None!r}")


def _weight_map(d: Path) -> dict[str, str]:
    """tensor key -> shard file name."""
    if (d / INDEX).exists():
        return dict(json.loads((d / INDEX).read_text())["weight_map"])
    if (d / SINGLE).exists():
        from safetensors import safe_open
        with safe_open(str(d / SINGLE), "pt") as f:
            return {k: SINGLE for k in f.keys()}
    raise FileNotFoundError(f"{d}: neither {INDEX} nor {SINGLE}")


class Checkpoint:
    """The coded matrices of one checkpoint directory and their tensors."""

    def __init__(self, path):
        self.dir = Path(path)
        self.weight_map = _weight_map(self.dir)
        self.bases: dict[str, str] = {}      # text_key -> checkpoint key without the suffix
        for k in self.weight_map:
            if k.endswith(TRELLIS):
                base = k[: -len(TRELLIS)]
                t = text_key(base)
                if t is not None:
                    self.bases[t] = base
        if not self.bases:
            raise ValueError(f"{self.dir}: no {TRELLIS} tensors found")
        self.exl3 = set(self.bases)           # the reference's name for the set of coded text keys
        self._handles: dict = {}

    # ---- which vLLM layers are coded (config.py:106-121) ----
    def parts(self, prefix: str) -> list[str] | None:
        """The text keys of the checkpoint matrices behind a vLLM layer prefix, in output order (None: not text)."""
        t = text_key(prefix)
        if t is None:
            return None
        if t == "lm_head":
            return ["lm_head"]
        head, _, leaf = t.rpartition(".")
        return [f"{head}.{c}" for c in PACKED.get(leaf, [leaf])]

    def is_exl3(self, prefix: str) -> bool:
        parts = self.parts(prefix)
        if parts is None:
            return False
        hit = [q in self.exl3 for q in parts]
        if any(hit) and not all(hit):
            raise ValueError(f"{prefix}: fused layer is only partly EXL3: {dict(zip(parts, hit))}")
        return all(hit)

    def experts_exl3(self, prefix: str) -> bool:
        t = text_key(prefix)
        return t is not None and any(k.startswith(t + ".") for k in self.exl3)

    # ---- tensors ----
    def _file(self, name: str, device):
        from safetensors import safe_open
        key = (name, str(device))
        if key not in self._handles:
            self._handles[key] = safe_open(str(self.dir / name), "pt", device=str(device))
        return self._handles[key]

    def tensors(self, base: str, device="cpu") -> dict[str, torch.Tensor]:
        """The tensors of one matrix (checkpoint key `base` + '.' + suffix), as the checkpoint stores them."""
        out = {}
        for s in SUFFIXES:
            k = f"{base}.{s}"
            if k in self.weight_map:
                out[s] = self._file(self.weight_map[k], device).get_tensor(k)
        return out

    def matrix(self, key: str, device="cpu") -> EspMatrix:
        """One coded matrix by its text key (or its checkpoint base name)."""
        base = self.bases.get(key, key)
        if base + TRELLIS not in self.weight_map:
            raise KeyError(f"{key}: no {TRELLIS} tensor in the checkpoint")
        return EspMatrix(self.tensors(base, device))

    def layer(self, prefix: str, device="cpu") -> list[EspMatrix]:
        """The matrices of a coded vLLM layer (e.g. '...layers.3.self_attn.qkv_proj' -> q, k, v), in vLLM's shard
        order: what dense.Dense takes."""
        if not self.is_exl3(prefix):
            raise ValueError(f"{prefix}: not an EXL3 layer of this checkpoint")
        return [self.matrix(q, device) for q in self.parts(prefix)]

    def experts(self, prefix: str, device="cpu") -> list[tuple[EspMatrix, EspMatrix, EspMatrix]]:
        """(gate, up, down) of every routed expert under an MoE prefix (e.g. '...layers.0.mlp.experts'), expert ids
        0..E-1 with E one more than the largest id seen; every expert needs all three: what experts.prepare takes."""
        t = text_key(prefix)
        if t is None:
            raise ValueError(f"{prefix}: not a text-model module")
        pat = re.compile(re.escape(t) + r"\.(\d+)\.(gate_proj|up_proj|down_proj)$")
        found = {}
        for k in self.exl3:
            m = pat.match(k)
            if m:
                found[(int(m.group(1)), m.group(2))] = k
        if not found:
            raise ValueError(f"{prefix}: no EXL3 experts")
        E = 1 + max(e for e, _ in found)
        missing = [(e, q) for e in range(E) for q in PROJS if (e, q) not in found]
        if missing:
            raise RuntimeError(f"{prefix}: {len(missing)} expert matrices missing, e.g. {missing[:3]}")
        return [tuple(self.matrix(found[(e, q)], device) for q in PROJS) for e in range(E)]
