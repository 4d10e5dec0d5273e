"""Generate tests/golden/checkpoint_keys.json from the REFERENCE plugin's own key logic (vllm_espalier/config.py:
text_key, EspalierConfig.maybe_update_config / is_exl3 / experts_exl3; linear.py: shard_order; moe.py: the expert
tensor name pattern), imported from a reference checkout (it needs vLLM). tests/test_checkpoint.py and
tests/test_vllm_shell.py pin this package's checkpoint, linear and moe modules against these answers with no reference
present.

The names are synthetic module and checkpoint names of the kinds the reference handles (decoder layers, fused
projections, MTP layers, the head, vision modules, routed experts).

usage: python tests/golden/make_checkpoint_keys.py [--reference <checkout>]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent

LM = "model.language_model.layers"
CHECKPOINT_KEYS = (
    [f"{LM}.{i}.linear_attn.{m}.esp_trellis" for i in (0, 1) for m in ("in_proj_qkv", "in_proj_z", "out_proj")] +
    [f"{LM}.3.self_attn.{m}.esp_trellis" for m in ("q_proj", "k_proj", "v_proj", "o_proj")] +
    [f"{LM}.7.self_attn.{m}.esp_trellis" for m in ("q_proj", "k_proj")] +              # v_proj left out: partly coded
    [f"{LM}.0.mlp.shared_expert.{m}.esp_trellis" for m in ("gate_proj", "up_proj", "down_proj")] +
    [f"{LM}.0.mlp.experts.{e}.{m}.esp_trellis" for e in (0, 5) for m in ("gate_proj", "up_proj", "down_proj")] +
    ["lm_head.esp_trellis", "mtp.layers.0.mlp.experts.2.up_proj.esp_trellis", "mtp.layers.0.self_attn.o_proj.esp_trellis",
     f"{LM}.0.linear_attn.in_proj_a.weight", f"{LM}.0.mlp.gate.weight", "model.visual.blocks.0.attn.qkv.weight",
     "model.language_model.embed_tokens.weight"])
NAMES = [
    "language_model.model.layers.3.self_attn.qkv_proj", "language_model.model.layers.3.self_attn.o_proj",
    "language_model.model.layers.7.self_attn.qkv_proj", "language_model.model.layers.0.linear_attn.in_proj_qkvz",
    "language_model.model.layers.1.linear_attn.in_proj_qkvz", "language_model.model.layers.0.linear_attn.in_proj_ba",
    "language_model.model.layers.0.linear_attn.out_proj", "language_model.model.layers.0.mlp.shared_expert.gate_up_proj",
    "language_model.model.layers.0.mlp.shared_expert.down_proj", "language_model.model.layers.0.mlp.gate",
    "language_model.model.layers.0.mlp.experts", "language_model.model.layers.1.mlp.experts",
    "model.layers.3.self_attn.qkv_proj", "language_model.lm_head", "lm_head", "model.mtp.layers.0.self_attn.o_proj",
    "mtp.layers.0.mlp.experts", "model.layers.0.mlp.experts", "visual.blocks.0.attn.qkv",
    "model.vision_tower.layers.0.mlp.fc1", "language_model.model.embed_tokens", "language_model.model.norm",
]

SHARDS = [None, "q", "k", "v", [2, 1], [0, 1], 0, 3]
EXPERT_NAMES = [
    "model.language_model.layers.0.mlp.experts.7.down_proj.esp_trellis", "experts.0.gate_proj.suh",
    "layers.3.mlp.experts.12.up_proj.esp_grid", "model.layers.0.mlp.experts.gate_up_proj.weight",
    "model.layers.0.mlp.experts.3.w1.esp_trellis", "mtp.layers.0.mlp.experts.255.down_proj.svh",
    "layers.0.mlp.experts.1.down_proj.mul1", "layers.0.mlp.experts.x.up_proj.suh",
]


def main():
    ap = argparse.ArgumentParser()
    env = os.environ.get("ESPALIER_REFERENCE")
    ap.add_argument("--reference", type=Path, default=Path(env) if env else None, required=not env,
                    help="the reference checkout (default: $ESPALIER_REFERENCE)")
    a = ap.parse_args()
    sys.path.insert(0, str(a.reference))
    from vllm_espalier.config import EspalierConfig, text_key   # the reference's own module
    with tempfile.TemporaryDirectory() as d:
        (Path(d) / "model.safetensors.index.json").write_text(
            json.dumps({"weight_map": {k: "x.safetensors" for k in CHECKPOINT_KEYS}}))
        cfg = EspalierConfig.from_config({"quant_method": "espalier"})
        cfg.maybe_update_config(d)
    out = {"checkpoint_keys": CHECKPOINT_KEYS, "names": {}}
    for n in NAMES:
        try:
            exl3 = cfg.is_exl3(n)
        except ValueError:
            exl3 = "error"
        out["names"][n] = {"text_key": text_key(n), "is_exl3": exl3, "experts_exl3": cfg.experts_exl3(n)}
    # the loaders' own keying: vLLM shard ids -> output order (linear.py), expert tensor names -> (expert, projection,
    # suffix) (moe.py's name pattern)
    from vllm_espalier import linear as ref_linear
    from vllm_espalier import moe as ref_moe
    out["shard_order"] = [[sh, ref_linear.shard_order(tuple(sh) if isinstance(sh, list) else sh)] for sh in SHARDS]
    out["expert_names"] = {}
    for n in EXPERT_NAMES:
        m = ref_moe._NAME.search(n)
        out["expert_names"][n] = [int(m.group(1)), m.group(2), m.group(3)] if m else None
    (HERE / "checkpoint_keys.json").write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {len(NAMES)} names")


if __name__ == "__main__":
    main()
