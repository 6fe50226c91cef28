"""Model surgery — the reference's plugin entry (src/qosmoe/utils.py:8-97).

replace_qosmoe_layer(model, moe_parent_type, moe_type, name_experts, router_tensor_path, config,
                     placement=None)
walks the module tree; inside every module whose class name is `moe_parent_type` it replaces
each child whose class name is `moe_type` by a QoSMoELayer built from the child's experts (at the
dotted path `name_experts`: ModuleDict -> values, ModuleList -> list, or transformers-5.x fused
experts) and router weight (`router_tensor_path` + ".weight").  layer_idx counts replacements
in traversal order.  Qwen blocks also carry shared_expert / shared_expert_gate / top_k /
norm_topk_prob, which are picked up so the swapped block keeps top-k routing and the shared
expert (the reference's QoSMoELayer drops both).  `placement` overrides
config.expert_placement (exflow JSON path or [layer][gpu] -> experts list).  d_model and
num_experts are taken from the router weight's shape; the swapped layers return the
`(h, (logits, idx))` tuple when the installed transformers' callers unpack it (4.x) and `h`
alone otherwise (5.x).
"""
from __future__ import annotations

import dataclasses

import torch.nn as nn

from .layers import QoSMoELayer, hf_callers_unpack_tuples


def get_tensor_by_path(module, path):
    cur = module
    for part in path.split("."):
        cur = getattr(cur, part)
    return cur


def replace_qosmoe_layer(model, moe_parent_type, moe_type, name_experts, router_tensor_path, config,
                         placement=None):
    _replace(model, moe_parent_type, moe_type, [0], name_experts, router_tensor_path, config, placement,
             hf_callers_unpack_tuples())


def _replace(model, parent_t, moe_t, layer_idx, name_experts, router_path, config, placement, tuple_out):
    if type(model).__name__ == parent_t:
        for child_name, child in model.named_children():
            if type(child).__name__ != moe_t:
                continue
            experts = get_tensor_by_path(child, name_experts)
            if isinstance(experts, nn.ModuleDict):
                experts = list(experts.values())
            elif isinstance(experts, nn.ModuleList):
                experts = list(experts)
            cfg = dataclasses.replace(config)
            cfg.layer_idx = layer_idx[0]
            cfg.experts = experts
            cfg.expert_example = experts[0] if isinstance(experts, list) else experts
            cfg.router_weights = get_tensor_by_path(child, router_path).weight
            cfg.num_experts, cfg.d_model = (int(v) for v in cfg.router_weights.shape)
            cfg.return_router_tuple = tuple_out
            if placement is not None:
                cfg.expert_placement = placement
            if getattr(child, "shared_expert", None) is not None and cfg.shared_expert is None:
                cfg.shared_expert = child.shared_expert
                cfg.shared_expert_gate = child.shared_expert_gate
            if hasattr(child, "top_k") and cfg.top_k == 1:
                cfg.top_k = int(child.top_k)
                cfg.norm_topk_prob = bool(getattr(child, "norm_topk_prob", False))
            elif hasattr(getattr(child, "gate", None), "top_k") and cfg.top_k == 1:
                cfg.top_k = int(child.gate.top_k)
                cfg.norm_topk_prob = bool(getattr(child.gate, "norm_topk_prob", False))
            new_layer = QoSMoELayer(cfg)
            layer_idx[0] += 1
            setattr(model, child_name, new_layer)
    else:
        for child in model.children():
            _replace(child, parent_t, moe_t, layer_idx, name_experts, router_path, config, placement, tuple_out)


def get_qosmoe_layers(model):
    acc = []
    for module in model.children():
        if isinstance(module, QoSMoELayer):
            acc.append(module)
        else:
            acc.extend(get_qosmoe_layers(module))
    return acc
