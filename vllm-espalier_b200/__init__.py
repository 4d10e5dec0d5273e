"""vllm_espalier_b200: B200-native (sm_100a) Espalier decode hot path.

The host side mirrors the reference plugin's operator surface (vllm_espalier: ops.py custom ops, dense.Dense,
experts.prepare / route / routed2, matrix.EspMatrix, the ESPALIER_* switches); the compute is the C-ABI library
libespalier_b200.so (csrc/, hand-written sm_100a CUDA), loaded through ctypes by _lib.py. There is no CPU fallback:
every op raises if the library or a GPU is missing.
"""
from ._lib import EspError, ext, lib  # noqa: F401

__version__ = "0.1.0"
