"""QoSMoEConfig — same field names as the reference (src/qosmoe/config.py:4-54), plus the fields
the B200 block needs to cover the Qwen top-k + shared-expert block as well."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class QoSMoEConfig:
    rank: int
    world_size: int

    experts: list = None
    expert_example: object = None
    router_weights: object = None

    layer_idx: int = 0
    d_model: int = 768
    num_experts: int = 8
    model_name: str = ""

    cache_policy: str = "RAND"
    expert_cache_size: int = 2
    eq_tokens: int = 150
    expert_placement: str | list | None = None
    fetching_strategy: str = "async-cpu"

    enable_skew: bool = False
    enable_random: bool = False
    enable_uniform: bool = False
    skew: float = 0.0
    num_experts_skewed: int = 1

    qos_w1: float = 1.0
    qos_w2: float = 0.1
    qos_w3: float = 0.5

    qos_alpha: float = 1.0
    qos_beta: float = 0.1
    qos_delta: float = 0.5

    qos_epsilon: float = 1e-6
    qos_avg_token_cost: float = 0.005
    qos_default_deadline_s: float = 2.0

    qos_phase_prefill: float = 0.5
    qos_phase_decode: float = 1.0

    qos_target_batch: int = 64
    qos_attention_mode: str = "router_var"
    qos_budget_tokens_per_gpu: int = 0

    qos_enable_prefetch: bool = False
    qos_enable_async: bool = True
    qos_enable_load_balance: bool = True
    qos_prefetch_topk: int = 2
    qos_prefetch_budget_experts: int = 1
    qos_prefetch_score_power: float = 1.0

    # --- added for the B200 block
    top_k: int = 1                 # 1 = Switch argmax routing; >1 = softmax top-k (Qwen)
    norm_topk_prob: bool = False
    shared_expert: object = None   # module with gate_proj / up_proj / down_proj, or None
    shared_expert_gate: object = None  # Linear(d, 1) or None
    process_group: object = None   # torch.distributed group for world_size > 1
    collect_stats: bool = False    # per-forward latency / token statistics (host syncs)
    # forward returns (h, (router_logits, expert_index)) — the reference contract, which
    # transformers-4.x SwitchTransformersLayerFF unpacks — or h alone (transformers-5.x callers);
    # replace_qosmoe_layer sets it from the installed transformers
    return_router_tuple: bool = True
