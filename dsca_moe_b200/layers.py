"""Drop-in MoE blocks backed by libdsca_b200.

QoSMoELayer      — constructor and forward contract of src/qosmoe/moe_layer.py:58-459:
                   QoSMoELayer(QoSMoEConfig); set_runtime_context() required before forward
                   (RuntimeError otherwise); forward(h[B,S,d]) -> (h, (router_logits[T,E],
                   expert_index[T] int64)); set_next_layer(); get_statistics().
                   Top-1 Switch routing by default; config.top_k > 1 plus shared_expert /
                   shared_expert_gate give the Qwen block behind the same plugin.
ShardedQwenMoE   — constructor and forward contract of qwen_ep_adapter/qwen_ep.py:25-97:
                   ShardedQwenMoE(old_block, rank, world, policy); forward(h) -> (h, logits).
"""
from __future__ import annotations

import dataclasses
import json

import numpy as np
import torch
import torch.nn as nn

from . import _lib as L
from .engine import MoEEngine, default_expert_to_gpu, pack_relu, pack_swiglu
from .qos import QoSInputs
from .reporting import TRACE


def hf_callers_unpack_tuples() -> bool:
    """Whether the installed transformers' decoder layers accept a tuple from their MoE child.
    transformers 4.x (the reference's pins, 4.39 / 4.45) unpacks `(h, router_tuple)` in
    SwitchTransformersLayerFF and `(h, router_logits)` in Qwen2MoeDecoderLayer; from 5.0 the
    callers add the child's output to the residual directly, so a swapped block must return
    the tensor alone.  No transformers installed: True (the reference contract)."""
    try:
        import transformers
    except ImportError:
        return True
    return int(transformers.__version__.split(".")[0]) < 5


def _sd(expert) -> dict:
    if isinstance(expert, dict):
        return expert
    return {k: v for k, v in expert.state_dict().items()}


def experts_from_list(experts: list):
    """Per-expert state dicts (or modules) -> ('relu', wi, wo) or ('swiglu', gate, up, down),
    each stacked [E, ...] on the CPU.  Switch DenseActDense has wi / wo; Qwen2MoeMLP has
    gate_proj / up_proj / down_proj."""
    sds = [_sd(e) for e in experts]
    k0 = sds[0]
    if "wi.weight" in k0 and "wo.weight" in k0:
        return ("relu", torch.stack([s["wi.weight"] for s in sds]), torch.stack([s["wo.weight"] for s in sds]))
    if "gate_proj.weight" in k0:
        return ("swiglu", torch.stack([s["gate_proj.weight"] for s in sds]),
                torch.stack([s["up_proj.weight"] for s in sds]), torch.stack([s["down_proj.weight"] for s in sds]))
    raise ValueError(f"unrecognised expert parameters: {sorted(k0)}")


def experts_from_fused(mod):
    """transformers >= 5 fused experts: gate_up_proj [E, 2I, d] (gate rows first), down_proj [E, d, I]."""
    gu = mod.gate_up_proj.detach()
    I = gu.shape[1] // 2
    return ("swiglu", gu[:, :I], gu[:, I:], mod.down_proj.detach())


def placement_to_expert_to_gpu(placement, layer_idx: int, E: int, G: int) -> np.ndarray:
    """exflow placement ([layer][gpu] -> experts, a JSON path or the list itself;
    src/harmonymoe/scheduler.py:51-64) -> expert_to_gpu[E].  Layers past the end of the file fall
    back to the contiguous split, as the reference falls back to its naive placement."""
    if placement is None:
        return default_expert_to_gpu(E, G)
    if isinstance(placement, str):
        with open(placement) as f:
            placement = json.load(f)
    if len(placement) <= layer_idx:
        return default_expert_to_gpu(E, G)
    e2g = np.full(E, -1, np.int32)
    for gpu, lst in enumerate(placement[layer_idx]):
        for e in lst:
            e2g[int(e)] = gpu
    if (e2g < 0).any() or len(placement[layer_idx]) != G:
        raise ValueError("placement must list every expert exactly once over world_size GPUs")
    return e2g


class QoSMoELayer(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.rank, self.num_gpus = config.rank, config.world_size
        self.layer_idx = config.layer_idx
        self.num_experts, self.d_model = config.num_experts, config.d_model
        self.next_layer = None
        self.runtime_context = None
        dev = torch.device("cuda", torch.cuda.current_device())
        experts = config.experts
        spec = experts_from_fused(experts) if hasattr(experts, "gate_up_proj") else experts_from_list(list(experts))
        dtype = spec[1].dtype
        if dtype not in (torch.bfloat16, torch.float32):
            raise ValueError(f"expert dtype {dtype} not supported")
        # expert_cache_size below the expert count: the reference's non-resident path (pinned host
        # weights, cache slots, QoS-planned loads; src/qosmoe/moe_layer.py:129-131,296-330).
        # Expert parallel keeps every local expert resident.
        n_exp = int(spec[1].shape[0])
        cache_slots = None
        if int(config.expert_cache_size) < n_exp:
            cache_slots = max(1, int(config.expert_cache_size))
        pack_dev = "cpu" if cache_slots is not None else dev
        shared = None
        sg_w = None
        if spec[0] == "relu":
            packed = pack_relu(spec[1], spec[2], dtype=dtype, device=pack_dev)
        else:
            if config.shared_expert is not None:
                s = _sd(config.shared_expert)
                shared = (s["gate_proj.weight"], s["up_proj.weight"], s["down_proj.weight"])
                sg_w = _sd(config.shared_expert_gate)["weight"]
            packed = pack_swiglu(spec[1], spec[2], spec[3], shared=shared, dtype=dtype, device=pack_dev)
        router_w = config.router_weights.detach()
        top_k = int(getattr(config, "top_k", 1) or 1)
        mode = L.ROUTE_SWITCH_TOP1 if top_k == 1 else L.ROUTE_SOFTMAX_TOPK
        e2g = placement_to_expert_to_gpu(config.expert_placement, config.layer_idx, config.num_experts,
                                         config.world_size)
        self.engine = MoEEngine(router_w, packed, top_k=top_k, route_mode=mode,
                                norm_topk=bool(getattr(config, "norm_topk_prob", False)),
                                shared_gate_weight=sg_w, rank=config.rank, world=config.world_size,
                                group=getattr(config, "process_group", None), expert_to_gpu=e2g,
                                eq_tokens=config.eq_tokens, cache_slots=cache_slots, device=dev)
        for k in ("alpha", "beta", "delta", "target_batch", "epsilon"):
            self.engine.qos_params[k] = float(getattr(config, "qos_" + k, self.engine.qos_params[k]))
        self.engine.qos_params["attention_mode"] = 0 if getattr(config, "qos_attention_mode", "router_var") == "router_var" else 1
        # the experts now live packed in the engine: drop this layer's references to the caller's
        # expert modules / state dicts so that a swapped model does not hold both copies
        if dataclasses.is_dataclass(config):
            self.config = dataclasses.replace(config, experts=None, expert_example=None)
        self.tot_num_toks_send, self.tot_num_toks_recv = [], []
        self.latencies, self.expert_freqs, self.num_prefetch_launched = [], [], []
        self.expert_swaps = []

    def set_runtime_context(self, ctx):
        self.runtime_context = ctx

    def set_next_layer(self, next_layer):
        self.next_layer = next_layer

    def get_statistics(self):
        """Same keys as src/qosmoe/moe_layer.py:147-162 (filled when config.collect_stats)."""
        prefetched = getattr(self, "num_prefetch_launched", [])
        return [{"latency (ms)": self.latencies[i],
                 "total number of tokens sent": self.tot_num_toks_send[i],
                 "total number of tokens recv": self.tot_num_toks_recv[i],
                 "expert distribution": self.expert_freqs[i],
                 "num expert swaps": self.expert_swaps[i],
                 "num prefetch launched": prefetched[i] if i < len(prefetched) else 0}
                for i in range(len(self.latencies))]

    def _maybe_prefetch_next_layer(self, priority):
        """src/qosmoe/moe_layer.py:164-194: with qos_enable_prefetch and a next layer, the top
        qos_prefetch_topk (at most qos_prefetch_budget_experts) experts by this layer's priority
        (clamped at 0, raised to qos_prefetch_score_power) are copied into the next layer's expert
        cache ahead of its forward.  A next layer whose experts are all resident has no cache and
        loads nothing, as in the reference, where every candidate is already cached."""
        cfg = self.config
        if not getattr(cfg, "qos_enable_prefetch", False) or self.next_layer is None or priority is None:
            self.num_prefetch_launched.append(0)
            return []
        budget = int(getattr(cfg, "qos_prefetch_budget_experts", 0))
        scores = torch.as_tensor(np.asarray(priority, np.float32)).clamp_min(0)
        if budget <= 0 or scores.numel() == 0 or bool((scores <= 0).all()):
            self.num_prefetch_launched.append(0)
            return []
        power = float(getattr(cfg, "qos_prefetch_score_power", 1.0))
        if power != 1.0:
            scores = scores.pow(power)
        k = min(int(getattr(cfg, "qos_prefetch_topk", budget)), budget, scores.numel())
        ids = torch.topk(scores, k=k).indices.tolist()
        nxt = getattr(self.next_layer, "engine", None)
        cache = getattr(nxt, "cache", None)
        launched = cache.prefetch(ids) if cache is not None else []
        self.num_prefetch_launched.append(len(launched))
        return launched

    @torch.no_grad()
    def forward(self, hidden_states):
        if self.runtime_context is None:
            raise RuntimeError("QoSMoELayer requires runtime_context before forward")
        stats = bool(getattr(self.config, "collect_stats", False))
        if stats:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        shape = hidden_states.shape
        qos = None
        if self.engine._uses_qos:
            ctx = self.runtime_context
            qos = QoSInputs(x_prev=getattr(ctx, "last_hidden_states", None),
                            seq_priority=getattr(ctx, "flat_seq_priority", None),
                            remaining=getattr(ctx, "flat_remaining_tokens", None),
                            valid=getattr(ctx, "flat_valid_mask", None))
        trace = TRACE.enabled()
        if trace:  # the reference's token trace: host times around the block, device synchronised
            torch.cuda.synchronize()
            t0 = TRACE.now_ms()
        r = self.engine.forward(hidden_states.reshape(-1, self.d_model), qos=qos)
        if trace:
            torch.cuda.synchronize()
            TRACE.record_block(self.layer_idx, r["topk_ids"].cpu().numpy(), t0, t0, TRACE.now_ms())
        out = r["out"].view(shape)
        self.runtime_context.last_hidden_states = r["out"]
        if getattr(self.config, "qos_enable_prefetch", False):
            self._maybe_prefetch_next_layer(self.engine.last_priority_host())
        tuple_out = getattr(self.config, "return_router_tuple", True)
        if stats:
            ev1.record()
            ev1.synchronize()
            self.latencies.append(ev0.elapsed_time(ev1))
            self.expert_freqs.append(r["counts"].tolist())
            self.expert_swaps.append(self.engine.last_loads)
            lay = self.engine.last_layout
            T = r["out"].shape[0] * self.engine.top_k
            self.tot_num_toks_send.append(int(lay.send_splits.sum()) if lay is not None else T)
            self.tot_num_toks_recv.append(int(lay.recv_splits.sum()) if lay is not None else T)
        if not tuple_out:
            return out
        return out, (r["logits"], r["expert_index"])


class ShardedQwenMoE(nn.Module):
    """Qwen top-k + shared-expert block, expert parallel over `world` ranks of the default
    process group (or `group`).  Accepts a transformers-4.x block (experts ModuleList of
    Qwen2MoeMLP, gate Linear) or a transformers-5.x block (fused experts, Qwen2MoeTopKRouter).
    Placement: contiguous blocks (E % world need not be 0) or `expert_to_gpu`; `eq_tokens` >= 0
    turns on harmony rebalancing (the reference block uses fixed ownership: eq_tokens = -1).
    forward returns `(h, router_logits)` (the reference contract) or, with
    `return_logits=False`, `h` alone for transformers-5.x decoder layers."""

    def __init__(self, old, rank, world, policy="fifo", group=None, expert_to_gpu=None, eq_tokens=-1,
                 return_logits=True):
        super().__init__()
        self.rank, self.world, self.policy = rank, world, policy
        # transformers 4.x keeps num_experts / top_k / norm_topk_prob on the block, 5.x on its router
        src = old if hasattr(old, "top_k") else old.gate
        self.num_experts, self.top_k = int(src.num_experts), int(src.top_k)
        self.norm_topk_prob = bool(src.norm_topk_prob)
        self.return_logits = bool(return_logits)
        dev = torch.device("cuda", torch.cuda.current_device())
        experts = old.experts
        spec = experts_from_fused(experts) if hasattr(experts, "gate_up_proj") else experts_from_list(list(experts))
        dtype = spec[1].dtype
        s = _sd(old.shared_expert)
        packed = pack_swiglu(spec[1], spec[2], spec[3],
                             shared=(s["gate_proj.weight"], s["up_proj.weight"], s["down_proj.weight"]),
                             dtype=dtype, device=dev)
        self.engine = MoEEngine(old.gate.weight.detach(), packed, top_k=self.top_k,
                                route_mode=L.ROUTE_SOFTMAX_TOPK, norm_topk=self.norm_topk_prob,
                                shared_gate_weight=old.shared_expert_gate.weight.detach(), rank=rank,
                                world=world, group=group, expert_to_gpu=expert_to_gpu, eq_tokens=eq_tokens)
        self.route_calls = 0

    @torch.no_grad()
    def forward(self, hidden_states):
        b, s, d = hidden_states.shape
        r = self.engine.forward(hidden_states.reshape(-1, d))
        self.route_calls += 1
        if not self.return_logits:
            return r["out"].view(b, s, d)
        return r["out"].view(b, s, d), r["logits"]


def patch(model, rank, world, policy="fifo"):
    """qwen_ep_adapter/qwen_ep.py:100-109: swap every Qwen2MoeSparseMoeBlock of model.model.layers.
    The swapped blocks return what the installed transformers' Qwen2MoeDecoderLayer expects."""
    changed = 0
    tuple_out = hf_callers_unpack_tuples()
    for layer in model.model.layers:
        if layer.mlp.__class__.__name__ == "Qwen2MoeSparseMoeBlock":
            layer.mlp = ShardedQwenMoE(layer.mlp, rank, world, policy, return_logits=tuple_out)
            changed += 1
    if not changed:
        raise RuntimeError("No Qwen2MoeSparseMoeBlock found: wrong checkpoint/model version")
    return changed
