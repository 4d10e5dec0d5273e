"""vLLM linear method for coded dense layers and the LM head (the reference's vllm_espalier/linear.py:45-117).

A vLLM layer may fuse several checkpoint matrices (q/k/v, gate/up, in_proj_qkv/z); each keeps its own suh / svh, so
the layer holds one EspMatrix per shard, in vLLM's shard order, and its output is their outputs side by side (plus
vocabulary padding for the head). Shapes are only known from the checkpoint, so create_weights registers empty
placeholders whose loader keeps each arriving tensor. With ESPALIER_FUSED_DENSE (default) the layer is one
espalier::dense call: the fused dense kernel for all its matrices, input and output in the model's dtype.
Importing this module needs vLLM.
"""
from __future__ import annotations

import weakref

import torch
import torch.nn.functional as F
from torch.nn import Parameter
from vllm.model_executor.layers.linear import LinearMethodBase

from ._env import FUSED_DENSE
from .matrix import SUFFIXES, EspMatrix

_QKV_ORDER = {"q": 0, "k": 1, "v": 2}


def shard_order(shard) -> int:
    """Position of a loader shard id among the layer's outputs: None (an unfused layer) 0, 'q'/'k'/'v', the smallest
    of a tuple of ids, or an integer index."""
    if shard is None:
        return 0
    if isinstance(shard, str):
        return _QKV_ORDER[shard]
    if isinstance(shard, (tuple, list)):
        return min(shard)
    return int(shard)


def single_process():
    """Tensor parallelism is not supported (the reference's milestone 1 holds too): every matrix is whole."""
    try:
        from vllm.distributed import get_tensor_model_parallel_world_size
        world = get_tensor_model_parallel_world_size()
    except (AssertionError, ImportError):   # no tensor-parallel group: a single process
        world = 1
    if world != 1:
        raise NotImplementedError("espalier layers support tensor parallel size 1 only")


class EspLinearMethod(LinearMethodBase):
    def __init__(self, prefix: str):
        self.prefix = prefix

    def create_weights(self, layer, input_size_per_partition, output_partition_sizes, input_size, output_size,
                       params_dtype, **extra_weight_attrs):
        single_process()
        layer._esp_parts = {}                  # shard id -> {suffix: tensor}
        layer._esp_in = input_size_per_partition
        layer._esp_out = sum(output_partition_sizes)

        def keep(param, loaded_weight, shard_id=None, *args, **kwargs):
            shard = getattr(loaded_weight, "shard_id", shard_id)
            if isinstance(shard, list):
                shard = tuple(shard)
            layer._esp_parts.setdefault(shard, {})[param._esp_suffix] = loaded_weight.to(param.device).clone()

        for suffix in SUFFIXES:
            p = Parameter(torch.empty(0), requires_grad=False)
            p._esp_suffix = suffix
            p.weight_loader = keep
            layer.register_parameter(suffix, p)

    def process_weights_after_loading(self, layer) -> None:
        if not layer._esp_parts:
            if self.prefix.endswith("lm_head"):
                # a speculative drafter's own head, left unloaded on purpose: vLLM gives it the target's
                layer._esp_mats, layer._esp_dense, layer._esp_pad = [], None, 0
                return
            raise RuntimeError(f"{self.prefix}: no EXL3 tensors were loaded")
        parts = sorted(layer._esp_parts.items(), key=lambda kv: shard_order(kv[0]))
        layer._esp_mats = [EspMatrix(t) for _, t in parts]
        del layer._esp_parts
        # module buffers, so a compiled graph takes the packed tensors as inputs
        for i, m in enumerate(layer._esp_mats):
            layer.register_buffer(f"_esp_t{i}", m.trellis, persistent=False)
            layer.register_buffer(f"_esp_s{i}", m.suh, persistent=False)
            layer.register_buffer(f"_esp_v{i}", m.svh, persistent=False)
        ins = {m.in_features for m in layer._esp_mats}
        out = sum(m.out_features for m in layer._esp_mats)
        if ins != {layer._esp_in} or out > layer._esp_out:
            raise RuntimeError(f"{self.prefix}: EXL3 shapes in {sorted(ins)} out {out} do not fit the layer "
                               f"(in {layer._esp_in}, out {layer._esp_out})")
        layer._esp_pad = layer._esp_out - out          # the LM head's vocabulary padding
        layer._esp_dense = None
        if FUSED_DENSE and all(m.in_features % 128 == 0 and m.out_features % 128 == 0 for m in layer._esp_mats):
            from . import dense, ops
            key = ops.register_dense(dense.Dense(layer._esp_mats, layer._esp_out))
            layer._esp_dense = key
            # a layer vLLM drops after loading must not stay alive through the registry
            weakref.finalize(layer, ops.DENSE_LAYERS.pop, key, None)

    def _tensors(self, layer, i: int):
        return getattr(layer, f"_esp_t{i}"), getattr(layer, f"_esp_s{i}"), getattr(layer, f"_esp_v{i}")

    def apply(self, layer, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        n = len(layer._esp_mats)
        if layer._esp_dense is not None:
            from . import ops  # noqa: F401  (registers espalier::dense)
            T, S, V = zip(*(self._tensors(layer, i) for i in range(n)))
            y = torch.ops.espalier.dense(x.reshape(-1, x.shape[-1]), list(T), list(S), list(V), layer._esp_dense)
            y = y.view(*x.shape[:-1], y.shape[-1])
        else:
            ys = [m.forward_with(x, *self._tensors(layer, i)) for i, m in enumerate(layer._esp_mats)]
            y = ys[0] if n == 1 else torch.cat(ys, dim=-1)
            if layer._esp_pad:
                y = F.pad(y, (0, layer._esp_pad))
        return y + bias if bias is not None else y
