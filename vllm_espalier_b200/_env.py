"""Environment switches (ESPALIER_*), the reference plugin's names and defaults (vllm_espalier/_env.py and the
switch reads in linear.py:26, moe.py:40-46, ops.py:20-21, dense.py:18,27, experts.py:44)."""
import os


def env(name: str, default: str | None = None) -> str | None:
    return os.environ.get(name, default)


def flag(name: str, default: str = "1") -> bool:
    return env(name, default) not in ("0", "", "false", "False")


FUSED_DENSE = flag("ESPALIER_FUSED_DENSE")            # one launch per vLLM layer
GROUPED_EXPERTS = flag("ESPALIER_GROUPED_EXPERTS")    # grouped MoE pipeline
FUSED_ROUTING = flag("ESPALIER_FUSED_ROUTING")        # fused router GEMV + top-k + grouping
MOE_ONE_LAUNCH = flag("ESPALIER_MOE_FUSED")          # gate/up and down of the experts in one launch (this library)
PREFILL = env("ESPALIER_PREFILL_MODE", "chunk")       # chunk | gemm
DEBUG_SHARED_FOLD = flag("ESPALIER_DEBUG_SHARED_FOLD", "0")
EP_EXCHANGE = env("ESPALIER_EP_EXCHANGE", "p2p")   # expert parallelism: p2p (peer stores) | nccl (all_to_all)
