"""vllm_espalier_b200: the Espalier plugin's decode hot path, rebuilt for B200 (sm_100a).

Host modules keep the reference plugin's operator surface (the espalier::dense / espalier::matmul custom ops, Dense,
experts.prepare / route / routed2, EspMatrix, the ESPALIER_* switches, the vllm.general_plugins entry point); the
compute is libespalier_b200.so, hand-written sm_100a CUDA behind a C ABI (include/espalier_b200.h), loaded by _lib.py.
There is no CPU fallback: every op raises when the library or a GPU is missing.
"""
from ._lib import EspError, ext, lib  # noqa: F401

__version__ = "0.2.0"
