"""The package is importable by its name and declares the vLLM plugin entry point the reference declares
(vllm.general_plugins, pyproject.toml:13-14 of the reference), pointing at a register() that exists."""
from __future__ import annotations

import importlib
import tomllib
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_entry_point_resolves():
    meta = tomllib.loads((ROOT / "pyproject.toml").read_text())
    eps = meta["project"]["entry-points"]["vllm.general_plugins"]
    assert set(eps) == {"espalier"}
    module, _, attr = eps["espalier"].partition(":")
    assert callable(getattr(importlib.import_module(module), attr))
    assert meta["tool"]["setuptools"]["packages"] == ["vllm_espalier_b200"]


def test_package_imports_by_name():
    pkg = importlib.import_module("vllm_espalier_b200")
    assert Path(pkg.__file__).parent == ROOT / "vllm_espalier_b200"
    for name in ("codebooks", "matrix", "dense", "experts", "checkpoint", "ep", "plugin"):
        importlib.import_module(f"vllm_espalier_b200.{name}")
