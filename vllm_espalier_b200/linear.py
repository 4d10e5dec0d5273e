"""vLLM linear method for coded dense layers and the LM head.

A vLLM layer can fuse several checkpoint matrices (q/k/v, gate/up, in_proj_qkv/z) whose Hadamard signs and scales
differ, so the layer keeps one EspMatrix per checkpoint matrix and its output is theirs side by side in vLLM's shard
order, then the head's vocabulary padding. The shapes come from the checkpoint, not from vLLM, so create_weights
registers one empty placeholder per checkpoint suffix whose weight loader files each arriving tensor under its shard;
process_weights_after_loading turns them into matrices and, with ESPALIER_FUSED_DENSE (default), registers a
dense.Dense that espalier::dense runs in one or two launches. The vLLM interface is the reference's
(vllm_espalier/linear.py:45-117). Importing this module needs vLLM.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch.nn import Parameter
from vllm.model_executor.layers.linear import LinearMethodBase

from ._env import FUSED_DENSE
from .matrix import SUFFIXES, EspMatrix


def shard_order(shard) -> int:
    """Output position of a loader's shard id: no id (an unfused layer) first, 'q' / 'k' / 'v' in that order, an
    integer index as itself, a tuple of indices at its smallest."""
    if shard is None:
        return 0
    if isinstance(shard, str):
        return "qkv".index(shard)
    if isinstance(shard, (tuple, list)):
        return min(int(s) for s in shard)
    return int(shard)


def tensor_parallel_size() -> int:
    try:
        from vllm.distributed import get_tensor_model_parallel_world_size
        return get_tensor_model_parallel_world_size()
    except (AssertionError, ImportError):       # no tensor-parallel group yet: one process
        return 1


def single_process():
    """The coded layers are whole on every GPU: tensor parallelism is refused, as the reference does."""
    if tensor_parallel_size() != 1:
        raise NotImplementedError("espalier layers support tensor parallel size 1 only")


class ShardCollector:
    """The weight loader of a layer's placeholders: keeps a device copy of every tensor, by (shard id, suffix)."""

    def __init__(self):
        self.parts: dict = {}

    def __call__(self, param, tensor, shard_id=None, *args, **kwargs):
        shard = getattr(tensor, "shard_id", shard_id)
        shard = tuple(shard) if isinstance(shard, list) else shard
        self.parts.setdefault(shard, {})[param.esp_suffix] = tensor.to(param.device).clone()

    def matrices(self) -> list[EspMatrix]:
        return [EspMatrix(self.parts[s]) for s in sorted(self.parts, key=shard_order)]


@dataclass
class DenseState:
    """What a coded layer carries after loading (layer.espalier)."""

    mats: list            # EspMatrix per checkpoint matrix, in output order
    pad: int              # zero columns after them (the LM head's vocabulary padding)
    key: int | None       # espalier::dense registry key, None: matrix by matrix through espalier::matmul


def buffer_names(i: int) -> tuple[str, str, str]:
    return f"esp_trellis_{i}", f"esp_suh_{i}", f"esp_svh_{i}"


class EspLinearMethod(LinearMethodBase):
    def __init__(self, prefix: str):
        self.prefix = prefix

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **extra_weight_attrs):
        single_process()
        collector = ShardCollector()
        layer.esp_collector = collector
        layer.esp_shape = (input_size_per_partition, sum(output_partition_sizes))
        for suffix in SUFFIXES:
            p = Parameter(torch.empty(0), requires_grad=False)
            p.esp_suffix = suffix
            p.weight_loader = collector
            layer.register_parameter(suffix, p)

    def process_weights_after_loading(self, layer) -> None:
        collector = layer.__dict__.pop("esp_collector")
        if not collector.parts:
            if self.prefix.endswith("lm_head"):
                # a speculative drafter's own head that vLLM leaves unloaded on purpose (it shares the target's)
                layer.espalier = DenseState([], 0, None)
                return
            raise RuntimeError(f"{self.prefix}: no espalier tensors were loaded")
        mats = collector.matrices()
        k_in, n_out = layer.esp_shape
        widths = {m.in_features for m in mats}
        n = sum(m.out_features for m in mats)
        if widths != {k_in} or n > n_out:
            raise RuntimeError(f"{self.prefix}: coded matrices take {sorted(widths)} inputs and give {n} outputs, the "
                               f"layer has {k_in} inputs and {n_out} outputs")
        for i, m in enumerate(mats):     # module buffers: a compiled graph takes the packed tensors as inputs
            for name, t in zip(buffer_names(i), (m.trellis, m.suh, m.svh)):
                layer.register_buffer(name, t, persistent=False)
        key = None
        if FUSED_DENSE and all(m.in_features % 128 == 0 and m.out_features % 128 == 0 for m in mats):
            from . import dense, ops
            key = ops.register_dense(dense.Dense(mats, n_out), owner=layer)
        layer.espalier = DenseState(mats, n_out - n, key)

    @staticmethod
    def tensors(layer) -> tuple[list, list, list]:
        cols = [[getattr(layer, name) for name in buffer_names(i)] for i in range(len(layer.espalier.mats))]
        return tuple(list(c) for c in zip(*cols)) if cols else ([], [], [])

    def apply(self, layer, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        st = layer.espalier
        trellis, suh, svh = self.tensors(layer)
        if st.key is not None:
            from . import ops
            y = ops.dense(x.reshape(-1, x.shape[-1]), trellis, suh, svh, st.key)
            y = y.reshape(*x.shape[:-1], y.shape[-1])
        else:
            parts = [m.forward_with(x, t, s, v) for m, t, s, v in zip(st.mats, trellis, suh, svh)]
            y = parts[0] if len(parts) == 1 else torch.cat(parts, dim=-1)
            if st.pad:
                y = F.pad(y, (0, st.pad))
        return y if bias is None else y + bias
