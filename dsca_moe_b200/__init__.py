"""dsca_moe_b200 — B200-native (sm_100a) MoE-block forward for DSCA-MoE.

Public surface (mirrors the reference's plugin):
  QoSMoEConfig, QoSMoELayer, replace_qosmoe_layer, get_qosmoe_layers, RequestStateTable
  ShardedQwenMoE, patch                          (qwen_ep_adapter drop-in)
  MoEEngine, pack_swiglu, pack_relu, plan_harmony, plan_layout   (engine level)
  build_exec_plan, QoSInputs, ExpertCache        (expert cache / QoS planner path)
  write_run_outputs, TokenTrace                  (the reference's run output files)
The compute runs in libdsca_b200.so (include/dsca_b200.h); build it with
``python -m dsca_moe_b200.build``.
"""
from .config import QoSMoEConfig  # noqa: F401
from .runtime import QoSRuntimeContext, RequestStateTable  # noqa: F401


def __getattr__(name):
    # torch-dependent pieces load lazily so that `import dsca_moe_b200` stays cheap
    if name in ("QoSMoELayer", "ShardedQwenMoE", "patch", "placement_to_expert_to_gpu"):
        from . import layers
        return getattr(layers, name)
    if name in ("replace_qosmoe_layer", "get_qosmoe_layers", "get_tensor_by_path"):
        from . import plugin
        return getattr(plugin, name)
    if name in ("MoEEngine", "pack_swiglu", "pack_relu", "plan_harmony", "plan_layout", "PackedExperts",
                "default_expert_to_gpu", "exchange_chunks"):
        from . import engine
        return getattr(engine, name)
    if name in ("write_run_outputs", "TokenTrace"):
        from . import reporting
        return getattr(reporting, name)
    if name in ("QoSExecPlan", "QoSInputs", "ExpertCache", "build_exec_plan"):
        from . import qos
        return getattr(qos, name)
    raise AttributeError(name)
