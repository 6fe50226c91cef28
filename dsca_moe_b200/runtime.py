"""Runtime context accepted by the block (interface of src/qosmoe/runtime.py:86-152).

QoSMoELayer.forward refuses to run without a context (src/qosmoe/moe_layer.py:273-274).  The
reference uses it only to derive token priorities that reorder expert execution
(src/qosmoe/planner.py:63-151) — numerically inert — so this module keeps the interface and the
per-token fields, and the B200 block does not read them on the hot path.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch


@dataclass
class QoSRuntimeContext:
    seq_ids: torch.Tensor
    seq_priority: torch.Tensor
    remaining_tokens: torch.Tensor
    phase_tensor: torch.Tensor
    flat_seq_priority: torch.Tensor
    flat_remaining_tokens: torch.Tensor
    flat_valid_mask: torch.Tensor
    last_hidden_states: torch.Tensor | None = None
    created_at: float = field(default_factory=time.time)


class RequestStateTable:
    """build_context(batch) -> QoSRuntimeContext with the reference's fields
    (src/qosmoe/runtime.py:86-152: deadline slack, waiting time and phase -> sequence priority)."""

    def __init__(self, args):
        self.args = args
        self.table: dict[int, dict] = {}
        self.next_seq_id = 0

    def build_context(self, batch: dict, phase: str = "prefill") -> QoSRuntimeContext:
        now = time.time()
        attn = batch["attention_mask"]
        attn = attn if torch.is_tensor(attn) else torch.tensor(attn)
        B, Ls = attn.shape
        remaining = attn.sum(dim=1).float()
        ph = self.args.qos_phase_decode if phase == "decode" else self.args.qos_phase_prefill
        if "_qos_seq_ids" in batch:
            ids = [int(v) for v in torch.as_tensor(batch["_qos_seq_ids"]).reshape(-1).tolist()]
        else:
            ids = list(range(self.next_seq_id, self.next_seq_id + B))
            self.next_seq_id += B
        waiting, deadlines = [], []
        for i, sid in enumerate(ids):
            rem = float(remaining[i])
            st = self.table.get(sid)
            if st is None:
                st = {"start": now, "deadline": now + self.args.qos_default_deadline_s
                      + rem * self.args.qos_avg_token_cost}
                self.table[sid] = st
            waiting.append(max(now - st["start"], 0.0))
            deadlines.append(st["deadline"])
        dev = attn.device
        waiting_t = torch.tensor(waiting, device=dev)
        deadlines_t = torch.tensor(deadlines, device=dev)
        phase_t = torch.full((B,), ph, device=dev)
        slack = torch.clamp(deadlines_t - now - remaining.to(dev) * self.args.qos_avg_token_cost,
                            min=self.args.qos_epsilon)
        prio = self.args.qos_w1 / slack + self.args.qos_w2 * waiting_t + self.args.qos_w3 * phase_t
        return QoSRuntimeContext(
            seq_ids=torch.tensor(ids, device=dev), seq_priority=prio, remaining_tokens=remaining,
            phase_tensor=phase_t, flat_seq_priority=prio.repeat_interleave(Ls),
            flat_remaining_tokens=remaining.repeat_interleave(Ls),
            flat_valid_mask=attn.reshape(-1).bool())

    def mark_finished(self, seq_ids):
        for sid in torch.as_tensor(seq_ids).reshape(-1).tolist():
            self.table.pop(int(sid), None)
