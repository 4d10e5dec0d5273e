"""vLLM MoE method for coded routed experts (the reference's vllm_espalier/moe.py:64-236).

Every expert has its own gate / up / down EspMatrix (its own width and codebook), so nothing is stacked: the layer's
load_weights is replaced by one that files each checkpoint tensor under (expert, projection), because vLLM's expert
loader would take any 3-D tensor for a pre-fused all-experts tensor and a trellis is 3-D per expert.

Up to 32 tokens (and in 32-token windows above, ESPALIER_PREFILL_MODE=chunk) the layer runs the grouped pipeline of
experts.py with the shared expert folded in as one more slot when vLLM hands it to apply() (the method reports
mk_can_overlap_shared_experts), its gated output written where the runner reads it. With ESPALIER_FUSED_ROUTING
(default) the method is monolithic: the router GEMV, top-k, renormalisation and grouping are the fused routing launch,
the runner's gate replaced by a pass-through that keeps its weight. Otherwise (ESPALIER_GROUPED_EXPERTS=0, or gemm
prefill above 32 tokens) experts run one by one through espalier::matmul. Importing this module needs vLLM.
"""
from __future__ import annotations

import re
import types

import torch
import torch.nn.functional as F
from torch.nn import Parameter
from vllm.model_executor.layers.fused_moe.fused_moe_method_base import FusedMoEMethodBase
from vllm.model_executor.layers.fused_moe.runner.shared_experts import SharedExpertsOrder

from . import experts as grouped
from ._env import FUSED_ROUTING, GROUPED_EXPERTS, PREFILL
from .checkpoint import PROJS
from .linear import single_process
from .matrix import SUFFIXES, EspMatrix

ROWS = 32                                 # tokens a grouped window
ROUTE = GROUPED_EXPERTS and FUSED_ROUTING
_EXPERT_TENSOR = re.compile(r"(?:^|\.)(\d+)\.(gate_proj|up_proj|down_proj)\.(\w+)$")


class PassThroughGate(torch.nn.Module):
    """Takes the runner's router gate's place under fused routing: returns the hidden states as the "logits", so the
    monolithic apply computes the GEMV itself. Keeps the original module and its weight."""

    def __init__(self, gate):
        super().__init__()
        self.inner = gate
        self.weight = gate.weight

    def forward(self, x):
        return x, None


class EspMoEMethod(FusedMoEMethodBase):
    @property
    def topk_indices_dtype(self):
        return torch.int32

    @property
    def is_monolithic(self) -> bool:
        return ROUTE

    @property
    def mk_can_overlap_shared_experts(self) -> bool:
        return GROUPED_EXPERTS

    def create_weights(self, layer, num_experts, hidden_size, intermediate_size_per_partition, params_dtype,
                       **extra_weight_attrs):
        single_process()
        layer._esp_num_experts = num_experts
        layer._esp_parts = {}                  # (expert, projection) -> {suffix: tensor}
        for w in ("w13", "w2"):
            for s in SUFFIXES:
                layer.register_parameter(f"{w}_{s}", Parameter(torch.empty(0), requires_grad=False))
        dev = layer.w13_esp_trellis.device

        def load_weights(self_, weights):
            for name, t in weights:
                m = _EXPERT_TENSOR.search(name)
                if m is None:
                    raise ValueError(f"{getattr(self_, 'layer_name', '?')}: unexpected expert tensor {name!r}")
                e, proj, suffix = int(m.group(1)), m.group(2), m.group(3)
                if suffix not in SUFFIXES:
                    raise ValueError(f"{getattr(self_, 'layer_name', '?')}: unknown EXL3 suffix in {name!r}")
                self_._esp_parts.setdefault((e, proj), {})[suffix] = t.to(dev).clone()
                yield f"{'w2' if proj == 'down_proj' else 'w13'}_{suffix}"

        layer.load_weights = types.MethodType(load_weights, layer)

    def process_weights_after_loading(self, layer) -> None:
        E = layer._esp_num_experts
        mats = {key: EspMatrix(t) for key, t in layer._esp_parts.items()}
        missing = [(e, p) for e in range(E) for p in PROJS if (e, p) not in mats]
        if missing:
            raise RuntimeError(f"{getattr(layer, 'layer_name', '?')}: {len(missing)} expert matrices missing, "
                               f"e.g. {missing[:3]}")
        layer._esp_experts = [tuple(mats[(e, p)] for p in PROJS) for e in range(E)]
        del layer._esp_parts
        act = str(getattr(layer, "activation", "silu")).lower()
        if "silu" not in act:
            raise NotImplementedError(f"{getattr(layer, 'layer_name', '?')}: activation {act}")
        layer._esp_grouped = None              # built at the first apply(), once the shared expert is known

    def get_fused_moe_quant_config(self, layer):
        return None

    # ---- forward ----
    def _grouped(self, layer, shared_experts, internal: bool):
        """The layer's grouped tables, built once; the shared expert becomes its last entry when vLLM leaves it to
        apply() and the routed and shared inputs are the same value."""
        if layer._esp_grouped is None:
            layer._esp_same_input = self._runner_has_no_input_transform(layer)
            fold_in = shared_experts if internal and layer._esp_same_input else None
            layer._esp_grouped = self._prepare_grouped(layer, fold_in)
        return layer._esp_grouped

    def _run_grouped(self, layer, x, k, shared_experts, internal, pick=None, wts=None, gate=None):
        L = self._grouped(layer, shared_experts, internal)
        fold = internal and L.shared_id >= 0 and layer._esp_same_input
        s = grouped.scratch(L, ROWS, k + (L.shared_id >= 0), x.device)
        xc = x.contiguous()
        if x.shape[0] <= ROWS:
            if gate is not None:
                grouped.route(xc, gate, k, L, s)
            out, sh = grouped.routed2(xc, pick, wts, L, s, k=k)
        else:
            out, sh = grouped.windows(xc, pick, wts, L, s, k=k, gate=gate)
        return out, sh, fold

    def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None, shared_experts_input=None):
        T, k = topk_ids.shape
        internal = shared_experts is not None and shared_experts._determine_shared_experts_order(
            shared_experts_input) == SharedExpertsOrder.MK_INTERNAL_OVERLAPPED
        if GROUPED_EXPERTS and (T <= ROWS or PREFILL == "chunk"):
            out, sh, fold = self._run_grouped(layer, x, k, shared_experts, internal,
                                              pick=topk_ids.to(torch.int32).contiguous(),
                                              wts=topk_weights.float().contiguous())
            if fold:
                shared_experts._output[shared_experts._output_idx] = sh
            elif internal:
                shared_experts.forward(shared_experts_input, SharedExpertsOrder.MK_INTERNAL_OVERLAPPED)
            return out
        if internal:
            shared_experts.forward(shared_experts_input, SharedExpertsOrder.MK_INTERNAL_OVERLAPPED)
        return self._expert_by_expert(layer, x, topk_weights, topk_ids)

    @staticmethod
    def _expert_by_expert(layer, x, topk_weights, topk_ids):
        """Each picked expert on its tokens through espalier::matmul, weighted sums in fp32."""
        T, k = topk_ids.shape
        out = torch.zeros(x.shape, dtype=torch.float32, device=x.device)
        ids = topk_ids.reshape(-1)
        tok = torch.arange(T, device=x.device).repeat_interleave(k)
        w = topk_weights.reshape(-1).float()
        for e in ids.unique().tolist():
            sel = ids == e
            t = tok[sel]
            gate, up, down = layer._esp_experts[e]
            xs = x[t]
            h = F.silu(gate.forward(xs).float()) * up.forward(xs).float()
            out.index_add_(0, t, down.forward(h.to(x.dtype)).float() * w[sel, None])
        return out.to(x.dtype)

    def apply_monolithic(self, layer, x, router_logits, input_ids=None):
        """Fused routing: on the first call the runner's gate is swapped for a pass-through (its weight kept here), so
        router_logits is then the hidden states and the routing launch does the GEMV; a call that still gets real
        logits (E wide), or gemm prefill above 32 tokens, takes vLLM's router."""
        from vllm.forward_context import get_forward_context
        runner = get_forward_context().no_compile_layers[layer.layer_name]
        if getattr(layer, "_esp_gate_w", None) is None:
            r = runner.router
            if not (getattr(r, "renormalize", True) and getattr(r, "scoring_func", "softmax") == "softmax"):
                raise NotImplementedError("the fused routing implements softmax top-k with renormalisation only")
            layer._esp_gate_w = runner.gate.weight.detach()
            runner.gate = PassThroughGate(runner.gate)
        shared = runner._shared_experts
        logits_given = router_logits.shape[-1] == layer._esp_num_experts != x.shape[-1]
        T = x.shape[0]
        k = runner.router.top_k if hasattr(runner.router, "top_k") else layer.top_k
        internal = shared is not None and shared._determine_shared_experts_order(x) == \
            SharedExpertsOrder.MK_INTERNAL_OVERLAPPED
        if (T <= ROWS or PREFILL == "chunk") and not logits_given:
            out, sh, fold = self._run_grouped(layer, x, k, shared, internal, gate=layer._esp_gate_w)
            if fold:
                shared._output[shared._output_idx] = sh
            elif internal:
                shared.forward(x, SharedExpertsOrder.MK_INTERNAL_OVERLAPPED)
            return out
        logits = router_logits if logits_given else F.linear(x, layer._esp_gate_w)
        topk_weights, topk_ids = runner.router.select_experts(hidden_states=x, router_logits=logits,
                                                              topk_indices_dtype=self.topk_indices_dtype,
                                                              input_ids=input_ids)
        return self.apply(layer, x, topk_weights, topk_ids, shared, x)

    @staticmethod
    def _runner_has_no_input_transform(layer) -> bool:
        """True when the layer's MoE runner applies no routed-input transform, so the routed input and the shared
        experts' input are the same value."""
        try:
            from vllm.forward_context import get_forward_context
            runner = get_forward_context().no_compile_layers.get(layer.layer_name)
        except Exception:
            return False
        return runner is not None and getattr(runner, "routed_input_transform", "missing") is None

    @staticmethod
    def _prepare_grouped(layer, shared_experts):
        """Pointer / width / codebook tables of the layer's experts; a coded shared expert with a one-row sigmoid gate
        becomes the last entry."""
        shared = gate_w = None
        if shared_experts is not None:
            mlp = shared_experts._layer
            gu = getattr(mlp.gate_up_proj, "_esp_mats", None)
            dn = getattr(mlp.down_proj, "_esp_mats", None)
            gate = getattr(mlp, "expert_gate", None)
            if gu and dn and len(gu) == 2 and gate is not None and gate.weight.shape[0] == 1:
                shared, gate_w = (gu[0], gu[1], dn[0]), gate.weight.detach()
        return grouped.prepare(layer._esp_experts, shared, gate_w)
