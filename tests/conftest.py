"""Shared fixtures. The import paths (repository root, oracle/, tests/, tests/golden/) come from pyproject.toml."""
import pytest


@pytest.fixture(scope="session")
def dev():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
