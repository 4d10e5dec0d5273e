"""vLLM plugin entry (the reference's vllm_espalier/__init__.py:12-22 and register()).

register() is what a `vllm.general_plugins` entry point calls: it imports the quantization config (registering the
"espalier" method with vLLM) and the custom ops, and mixes the ESPALIER_* switches that change which custom ops a
compiled graph calls into VllmConfig.compute_hash, which keys vLLM's compile cache, so one setting's cached graph is
never handed to another. The reference's model-specific patches (its MTP drafter's embedding and head loading, the
inductor benchmark settings) belong to its serving stack and are not part of this package.
"""
from __future__ import annotations

import hashlib
import os

SWITCHES = ("ESPALIER_FUSED_DENSE", "ESPALIER_GROUPED_EXPERTS", "ESPALIER_FUSED_ROUTING", "ESPALIER_PREFILL_MODE")


def salted(compute_hash):
    """compute_hash with the switches' current values mixed in (same length as the original digest)."""
    def compute_hash_esp(self, *args, **kwargs):
        h = compute_hash(self, *args, **kwargs)
        salt = ",".join(f"{k}={os.environ.get(k, '')}" for k in SWITCHES)
        return hashlib.sha256(f"{h}|{salt}".encode()).hexdigest()[:len(h)]
    compute_hash_esp._esp = True
    return compute_hash_esp


def register():
    from . import config, ops  # noqa: F401  (register the quantization method and the custom ops)
    from vllm.config import VllmConfig
    if not getattr(VllmConfig.compute_hash, "_esp", False):
        VllmConfig.compute_hash = salted(VllmConfig.compute_hash)
