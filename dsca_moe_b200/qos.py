"""Expert cache and QoS execution plan — the reference's non-resident expert path.

When a GPU may hold only `cache_size` routed experts (QoSMoEConfig.expert_cache_size <
num_experts, src/qosmoe/config.py:19), the reference keeps every expert's weights in pinned host
memory, computes the QoS planner's expert priorities (src/qosmoe/planner.py:63-170, here the
dsca_qos_priority kernel), orders the active experts with build_exec_plan (:172-237) and runs
them one by one, copying the ones that are not resident into cache slots on a load stream while
the compute stream waits on per-slot events (src/qosmoe/async_cpu.py:98-256,
src/qosmoe/expert_manager.py:8-128).

Here each expert of the plan is one launch of the grouped expert GEMM over that expert's rows of
the expert-major buffer, with its weights read from the slot the plan gave it (group_weight = the
slot index).  Every expert is loaded into its planned slot before it is computed, and a slot is
overwritten only after the GEMM that last read it has finished, so the output equals the
all-resident result bit for bit; the plan changes only the order and what crosses PCIe.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class QoSExecPlan:
    """src/qosmoe/planner.py:7-11."""
    expert_order: list
    slot_idxs: list
    need_loading: list


def build_exec_plan(active, priority, local_cache: list, cache_size: int) -> QoSExecPlan:
    """QoSPlanner.build_exec_plan (src/qosmoe/planner.py:172-237).  `active`: experts with at
    least one routed row; `priority`: expert priorities (indexable by expert id).  Resident
    experts first, then the others, each by priority descending (ties: expert id ascending, the
    order of a stable sort); the experts to load take the free slots, then the resident
    experts' slots from the lowest priority up, cyclically."""
    local_cache = list(local_cache or [])
    act = sorted(set(int(e) for e in active))
    pr = [float(p) for p in priority]
    loaded = sorted([e for e in act if e in local_cache], key=lambda e: -pr[e])
    unloaded = sorted([e for e in act if e not in local_cache], key=lambda e: -pr[e])
    if not unloaded:
        return QoSExecPlan(loaded, [local_cache.index(e) for e in loaded], [])
    low_to_high = [local_cache.index(e) for e in sorted(loaded, key=lambda e: pr[e])]
    used = set(low_to_high)
    cand = [s for s in range(cache_size) if s not in used] + low_to_high
    cand = cand or [0]
    order, slots, need = loaded + unloaded, [], []
    c = 0
    for e in order:
        if e in local_cache:
            slots.append(local_cache.index(e))
        else:
            slots.append(cand[c % len(cand)])
            c += 1
            need.append(e)
    return QoSExecPlan(order, slots, need)


@dataclass
class QoSInputs:
    """Per-token inputs of the planner (src/qosmoe/runtime.py: flat_seq_priority,
    flat_remaining_tokens, flat_valid_mask) and the previous layer's hidden states; each may be
    None (priority 1, remaining 0, valid, no previous states)."""
    x_prev: torch.Tensor | None = None
    seq_priority: torch.Tensor | None = None
    remaining: torch.Tensor | None = None
    valid: torch.Tensor | None = None


def match_token_length(v: torch.Tensor | None, n: int) -> torch.Tensor | None:
    """QoSPlanner._match_token_length (src/qosmoe/planner.py:29-50): a per-sequence or
    per-token vector stretched to n tokens (repeat each entry when n is a multiple, truncate when
    longer, pad with the last value when shorter)."""
    if v is None:
        return None
    v = v.reshape(-1)
    if v.numel() == n:
        return v
    if v.numel() == 0:
        return torch.zeros(n, dtype=torch.float32, device=v.device)
    if n % v.numel() == 0:
        return v.repeat_interleave(n // v.numel())
    if v.numel() > n:
        return v[:n]
    return torch.cat([v, v[-1:].expand(n - v.numel())])


@dataclass
class ExpertCache:
    """`slots` device slots for the routed experts of one block; the packed weights of all
    experts stay in pinned host memory.  `resident[s]` is the expert in slot s (-1: empty)."""
    host_w1: torch.Tensor            # [E, n1p, d] pinned
    host_w2: torch.Tensor            # [E, dp, ip] pinned
    w1: torch.Tensor                 # [slots, n1p, d] device
    w2: torch.Tensor                 # [slots, dp, ip] device
    slot_ids: torch.Tensor           # [slots] int32 device: group_weight views
    resident: list
    load_stream: torch.cuda.Stream
    loaded: list = field(default_factory=list)   # per slot: copy of its current expert done
    free: list = field(default_factory=list)     # per slot: last GEMM that read it done
    loads: int = 0                   # experts copied in since creation
    bytes_loaded: int = 0
    prefetch_cursor: int = 0         # next slot a prefetch overwrites (round robin)

    @property
    def slots(self) -> int:
        return self.w1.shape[0]

    @staticmethod
    def create(host_w1: torch.Tensor, host_w2: torch.Tensor, slots: int, device, initial=None) -> "ExpertCache":
        if slots <= 0:
            raise ValueError("an expert cache needs at least one slot")
        hw1 = host_w1 if host_w1.is_pinned() else host_w1.cpu().pin_memory()
        hw2 = host_w2 if host_w2.is_pinned() else host_w2.cpu().pin_memory()
        c = ExpertCache(host_w1=hw1, host_w2=hw2,
                        w1=torch.empty((slots,) + tuple(hw1.shape[1:]), dtype=hw1.dtype, device=device),
                        w2=torch.empty((slots,) + tuple(hw2.shape[1:]), dtype=hw2.dtype, device=device),
                        slot_ids=torch.arange(slots, dtype=torch.int32, device=device),
                        resident=[-1] * slots, load_stream=torch.cuda.Stream(device))
        c.loaded = [torch.cuda.Event() for _ in range(slots)]
        c.free = [torch.cuda.Event() for _ in range(slots)]
        # the reference fills the slots with the GPU's first cached experts at construction
        # (src/qosmoe/expert_manager.py:37-45)
        for s, e in enumerate(list(initial if initial is not None else range(min(slots, hw1.shape[0])))[:slots]):
            c.load(int(e), s)
        return c

    def load(self, expert: int, slot: int):
        """Copy `expert` into `slot` on the load stream, after the last GEMM that read the slot."""
        with torch.cuda.stream(self.load_stream):
            self.load_stream.wait_event(self.free[slot])
            self.w1[slot].copy_(self.host_w1[expert], non_blocking=True)
            self.w2[slot].copy_(self.host_w2[expert], non_blocking=True)
            self.loaded[slot].record(self.load_stream)
        self.resident[slot] = int(expert)
        self.loads += 1
        self.bytes_loaded += (self.host_w1[expert].numel() * self.host_w1.element_size()
                              + self.host_w2[expert].numel() * self.host_w2.element_size())

    def prefetch(self, expert_ids) -> list:
        """ExpertManager.prefetch_experts (src/qosmoe/expert_manager.py:94-128): every listed expert
        that is not cached yet is copied into the next slot of a round-robin cursor (on the load
        stream, after the last GEMM that read that slot); returns the (expert, slot) pairs."""
        launched = []
        cached = {e for e in self.resident if e >= 0}
        for e in expert_ids:
            e = int(e)
            if e < 0 or e >= self.host_w1.shape[0] or e in cached:
                continue
            slot = self.prefetch_cursor % self.slots
            self.prefetch_cursor = (self.prefetch_cursor + 1) % self.slots
            self.load(e, slot)
            launched.append((e, slot))
            cached.add(e)
        return launched
