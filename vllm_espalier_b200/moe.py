"""vLLM MoE method for coded routed experts.

Each expert's gate / up / down is its own EspMatrix (its own width and codebook), so nothing is stacked: the layer's
load_weights is replaced by an ExpertCollector, because vLLM's expert loader takes any 3-D tensor for a pre-fused
all-experts tensor and a trellis is 3-D per expert.

The forward is a GroupedRunner over experts.py's pipeline, up to 32 tokens a window (and in 32-token windows above,
ESPALIER_PREFILL_MODE=chunk). When vLLM hands the shared expert to apply() (the method reports
mk_can_overlap_shared_experts) and it is coded with a one-row sigmoid gate, it becomes one more slot of the grouped
launch and its gated output is written where vLLM's runner reads it. With ESPALIER_FUSED_ROUTING (default) the method
is monolithic: the fused routing launch does the router GEMV, top-k, renormalisation and grouping, and the runner's
gate is swapped for a pass-through that keeps its weight. Otherwise (ESPALIER_GROUPED_EXPERTS=0, or gemm prefill
above 32 tokens) the picked experts run one at a time through espalier::matmul. The vLLM hooks are the reference's
(vllm_espalier/moe.py:64-236). Importing this module needs vLLM.
"""
from __future__ import annotations

import re
import types
from dataclasses import dataclass

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

WINDOW = 32                                    # tokens a grouped call
ROUTE = GROUPED_EXPERTS and FUSED_ROUTING
_TENSOR_NAME = re.compile(r"(?:^|\.)(?P<expert>\d+)\.(?P<proj>gate_proj|up_proj|down_proj)\.(?P<suffix>\w+)$")


def parse_expert_tensor(name: str):
    """'...experts.<e>.<gate|up|down>_proj.<suffix>' -> (e, projection, suffix); None for any other name."""
    m = _TENSOR_NAME.search(name)
    return None if m is None else (int(m["expert"]), m["proj"], m["suffix"])


class ExpertCollector:
    """A layer's replacement load_weights: files each expert tensor under (expert, projection, suffix) and yields the
    name of the placeholder parameter that stands for it."""

    def __init__(self, device):
        self.device = device
        self.parts: dict = {}

    def load(self, layer, weights):
        for name, t in weights:
            key = parse_expert_tensor(name)
            if key is None:
                raise ValueError(f"{getattr(layer, 'layer_name', '?')}: unexpected expert tensor {name!r}")
            e, proj, suffix = key
            if suffix not in SUFFIXES:
                raise ValueError(f"{getattr(layer, 'layer_name', '?')}: unknown espalier suffix in {name!r}")
            self.parts.setdefault((e, proj), {})[suffix] = t.to(self.device).clone()
            yield f"{'w2' if proj == 'down_proj' else 'w13'}_{suffix}"

    def experts(self, E: int, where: str) -> list[tuple]:
        missing = [(e, p) for e in range(E) for p in PROJS if (e, p) not in self.parts]
        if missing:
            raise RuntimeError(f"{where}: {len(missing)} expert matrices missing, e.g. {missing[:3]}")
        return [tuple(EspMatrix(self.parts[(e, p)]) for p in PROJS) for e in range(E)]


class PassThroughGate(torch.nn.Module):
    """Replaces the runner's router gate under fused routing: the "logits" it returns are the hidden states, so the
    monolithic apply does the GEMV in the routing launch. Keeps the original module and its weight."""

    def __init__(self, gate):
        super().__init__()
        self.inner = gate
        self.weight = gate.weight

    def forward(self, x):
        return x, None


def _runner(layer):
    from vllm.forward_context import get_forward_context
    return get_forward_context().no_compile_layers.get(layer.layer_name)


class GroupedRunner:
    """One layer's grouped pipeline. Its tables are built at the first forward, once it is known whether vLLM hands
    the shared expert over (then the shared expert is the tables' last entry)."""

    def __init__(self, experts):
        self.experts = experts
        self.L = None
        self.same_input = False

    def tables(self, layer, shared_experts, internal: bool):
        if self.L is None:
            try:
                runner = _runner(layer)
            except Exception:   # outside a forward context (tests): no transform is known, so none is assumed
                runner = None
            # the shared slot reads the routed input: only valid when the runner applies no routed-input transform
            self.same_input = runner is not None and getattr(runner, "routed_input_transform", "missing") is None
            shared = gate_w = None
            if internal and self.same_input and shared_experts is not None:
                mlp = shared_experts._layer
                gu = getattr(getattr(mlp.gate_up_proj, "espalier", None), "mats", None)
                dn = getattr(getattr(mlp.down_proj, "espalier", None), "mats", None)
                g = getattr(mlp, "expert_gate", None)
                if gu and dn and len(gu) == 2 and g is not None and g.weight.shape[0] == 1:
                    shared, gate_w = (gu[0], gu[1], dn[0]), g.weight.detach()
            self.L = grouped.prepare(self.experts, shared, gate_w)
        return self.L

    def __call__(self, layer, x, k, shared_experts, internal, pick=None, wts=None, gate=None):
        """(routed sum, shared output or None, whether the shared output was computed here)."""
        L = self.tables(layer, shared_experts, internal)
        s = grouped.scratch(L, WINDOW, k + (L.shared_id >= 0), x.device)
        x = x.contiguous()
        if x.shape[0] > WINDOW:
            out, sh = grouped.windows(x, pick, wts, L, s, k=k, gate=gate)
        else:
            if gate is not None:
                grouped.route(x, gate, k, L, s)
            out, sh = grouped.routed2(x, pick, wts, L, s, k=k)
        return out, sh, internal and L.shared_id >= 0 and self.same_input


@dataclass
class MoEState:
    """What a coded MoE layer carries after loading (layer.espalier)."""

    experts: list                     # (gate, up, down) EspMatrix per expert
    runner: GroupedRunner
    gate_w: torch.Tensor | None = None


def _hand_over_shared(shared_experts, sh, folded: bool, internal: bool, x):
    if folded:
        shared_experts._output[shared_experts._output_idx] = sh
    elif internal:
        shared_experts.forward(x, SharedExpertsOrder.MK_INTERNAL_OVERLAPPED)


def _internal(shared_experts, x) -> bool:
    return shared_experts is not None and \
        shared_experts._determine_shared_experts_order(x) == SharedExpertsOrder.MK_INTERNAL_OVERLAPPED


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
        for w in ("w13", "w2"):
            for s in SUFFIXES:
                layer.register_parameter(f"{w}_{s}", Parameter(torch.empty(0), requires_grad=False))
        collector = ExpertCollector(layer.w13_esp_trellis.device)
        layer.esp_collector = collector
        layer.esp_num_experts = num_experts
        layer.load_weights = types.MethodType(collector.load, layer)

    def process_weights_after_loading(self, layer) -> None:
        where = getattr(layer, "layer_name", "?")
        collector = layer.__dict__.pop("esp_collector")
        experts = collector.experts(layer.esp_num_experts, where)
        act = str(getattr(layer, "activation", "silu")).lower()
        if "silu" not in act:
            raise NotImplementedError(f"{where}: activation {act}")
        layer.espalier = MoEState(experts, GroupedRunner(experts))

    def get_fused_moe_quant_config(self, layer):
        return None

    def apply(self, layer, x, topk_weights, topk_ids, shared_experts=None, shared_experts_input=None):
        T, k = topk_ids.shape
        internal = _internal(shared_experts, shared_experts_input)
        if GROUPED_EXPERTS and (T <= WINDOW or PREFILL == "chunk"):
            out, sh, folded = layer.espalier.runner(layer, x, k, shared_experts, internal,
                                                    pick=topk_ids.to(torch.int32).contiguous(),
                                                    wts=topk_weights.float().contiguous())
            _hand_over_shared(shared_experts, sh, folded, internal, shared_experts_input)
            return out
        _hand_over_shared(shared_experts, None, False, internal, shared_experts_input)
        return one_by_one(layer.espalier.experts, x, topk_weights, topk_ids)

    def apply_monolithic(self, layer, x, router_logits, input_ids=None):
        """Fused routing. The first call swaps the runner's gate for a pass-through (its weight kept), so from then on
        router_logits is the hidden states; a call that still gets E-wide logits, or gemm prefill above 32 tokens,
        routes through vLLM's router."""
        runner = _runner(layer)
        st = layer.espalier
        if st.gate_w is None:
            r = runner.router
            if not (getattr(r, "renormalize", True) and getattr(r, "scoring_func", "softmax") == "softmax"):
                raise NotImplementedError("the fused routing implements softmax top-k with renormalisation only")
            st.gate_w = runner.gate.weight.detach()
            runner.gate = PassThroughGate(runner.gate)
        shared = runner._shared_experts
        logits_given = router_logits.shape[-1] == layer.esp_num_experts != x.shape[-1]
        k = runner.router.top_k if hasattr(runner.router, "top_k") else layer.top_k
        if not logits_given and (x.shape[0] <= WINDOW or PREFILL == "chunk"):
            internal = _internal(shared, x)
            out, sh, folded = st.runner(layer, x, k, shared, internal, gate=st.gate_w)
            _hand_over_shared(shared, sh, folded, internal, x)
            return out
        logits = router_logits if logits_given else F.linear(x, st.gate_w)
        topk_weights, topk_ids = runner.router.select_experts(hidden_states=x, router_logits=logits,
                                                              topk_indices_dtype=self.topk_indices_dtype,
                                                              input_ids=input_ids)
        return self.apply(layer, x, topk_weights, topk_ids, shared, x)


def one_by_one(experts, x, topk_weights, topk_ids):
    """Each picked expert on its tokens through espalier::matmul; SwiGLU and the weighted sum in fp32."""
    T, k = topk_ids.shape
    acc = torch.zeros(x.shape, dtype=torch.float32, device=x.device)
    flat = topk_ids.reshape(-1)
    token = torch.arange(T, device=x.device).repeat_interleave(k)
    weight = topk_weights.reshape(-1).float()
    for e in flat.unique().tolist():
        sel = flat == e
        rows = token[sel]
        g, u, d = experts[e]
        xs = x[rows]
        h = F.silu(g.forward(xs).float()) * u.forward(xs).float()
        acc.index_add_(0, rows, d.forward(h.to(x.dtype)).float() * weight[sel, None])
    return acc.to(x.dtype)
