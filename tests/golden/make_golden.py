#!/usr/bin/env python3
"""Generate the golden fixtures in this directory by running the reference's own code on CPU.

The reference (acbling/DSCA-MoE) is pure Python/PyTorch and hard-codes CUDA streams, events and
``device="cuda"`` literals.  This script imports it from the directory named by the environment
variable REFERENCE_ROOT (required: the root of an acbling/DSCA-MoE checkout) behind a small shim
that
  * replaces torch.cuda.Event / Stream / stream / default_stream with host no-ops,
  * makes nn.Module.cuda, Tensor.cuda and Tensor.pin_memory identities,
  * rewrites ``device="cuda"`` keyword arguments to the CPU (TorchFunctionMode),
  * turns the reference's CSV tracers off (QOSMOE_REAL_TOKEN_TRACE=0, QOSMOE_TRACE_SYNC_CUDA=0),
and then calls, unmodified:
  * ``QoSMoELayer.forward`` at world_size=1 with every expert resident
    (src/qosmoe/moe_layer.py:271-296 -> :196-269) — the Switch top-1 block;
  * ``ShardedQwenMoE.forward`` (qwen_ep_adapter/qwen_ep.py:44-97) on gloo CPU ranks,
    world 1 and 4 — the Qwen top-4 + shared-expert block;
  * ``Scheduler.schedule_harmony`` / ``schedule_fixed`` (src/harmonymoe/scheduler.py:268-372),
    ``distribute_tokens`` (:101-124) and ``generate_expert_mask`` (:185-213).

The fixtures are small; inputs that are not stored are regenerated from the seeds recorded in
each file by ``dsca_moe_b200.synthetic``.  Run from the repository root:

    REFERENCE_ROOT=<path to the DSCA-MoE checkout> python tests/golden/make_golden.py
"""
from __future__ import annotations

import contextlib
import json
import os
import socket
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REFERENCE_ROOT = os.environ.get("REFERENCE_ROOT", "")
if not REFERENCE_ROOT or not os.path.isdir(REFERENCE_ROOT):
    raise SystemExit("set REFERENCE_ROOT to the root of the DSCA-MoE checkout")
sys.path.insert(0, REPO)

os.environ["QOSMOE_REAL_TOKEN_TRACE"] = "0"
os.environ["QOSMOE_TRACE_SYNC_CUDA"] = "0"
os.environ["QOSMOE_TRACE_ENABLE"] = "0"

import torch  # noqa: E402
import torch.nn as nn  # noqa: E402
from torch.overrides import TorchFunctionMode  # noqa: E402

from dsca_moe_b200 import synthetic as syn  # noqa: E402


# ----------------------------------------------------------------------------- shim
class _Event:
    def __init__(self, *a, **k):
        self.t = time.perf_counter()

    def record(self, *a, **k):
        self.t = time.perf_counter()

    def synchronize(self):
        pass

    def wait(self, *a, **k):
        pass

    def query(self):
        return True

    def elapsed_time(self, other):
        return (other.t - self.t) * 1e3


class _Stream:
    def __init__(self, *a, **k):
        pass

    def wait_event(self, *a, **k):
        pass

    def wait_stream(self, *a, **k):
        pass

    def synchronize(self):
        pass

    def record_event(self, *a, **k):
        return _Event()


class _CudaToCpu(TorchFunctionMode):
    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = dict(kwargs or {})
        dev = kwargs.get("device")
        if dev is not None and str(dev).startswith("cuda"):
            kwargs["device"] = "cpu"
        return func(*args, **kwargs)


def install_shim():
    torch.cuda.Event = _Event
    torch.cuda.Stream = _Stream
    torch.cuda.default_stream = lambda *a, **k: _Stream()
    torch.cuda.current_stream = lambda *a, **k: _Stream()
    torch.cuda.stream = lambda *a, **k: contextlib.nullcontext()
    nn.Module.cuda = lambda self, *a, **k: self
    torch.Tensor.cuda = lambda self, *a, **k: self
    torch.Tensor.pin_memory = lambda self, *a, **k: self
    for p in (os.path.join(REFERENCE_ROOT, "src"), os.path.join(REFERENCE_ROOT, "qwen_ep_adapter")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _t(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype)


def _np(t):
    return t.detach().to(torch.float32).cpu().numpy()


# ----------------------------------------------------------------------------- Switch
class _DenseActDense(nn.Module):
    """Same parameter names and math as transformers' SwitchTransformersDenseActDense
    (wi -> ReLU -> wo, no bias); dropout is identity in eval."""

    def __init__(self, d, F, dtype):
        super().__init__()
        self.wi = nn.Linear(d, F, bias=False, dtype=dtype)
        self.wo = nn.Linear(F, d, bias=False, dtype=dtype)
        self.act = nn.ReLU()

    def forward(self, x):
        h = self.act(self.wi(x))
        if h.dtype != self.wo.weight.dtype:
            h = h.to(self.wo.weight.dtype)
        return self.wo(h)


def run_switch_reference(x, Wr, wi, wo, dtype, B, S):
    """QoSMoELayer world=1, all experts resident -> (y[T,d], logits[T,E], expert_index[T])."""
    from qosmoe.config import QoSMoEConfig
    from qosmoe.moe_layer import QoSMoELayer
    from qosmoe.runtime import RequestStateTable

    E, F, d = wi.shape
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    experts = []
    for e in range(E):
        m = _DenseActDense(d, F, tdt)
        with torch.no_grad():
            m.wi.weight.copy_(_t(wi[e], tdt))
            m.wo.weight.copy_(_t(wo[e], tdt))
        experts.append(m)
    sds = [{k: v.detach().clone() for k, v in m.state_dict().items()} for m in experts]
    cfg = QoSMoEConfig(rank=0, world_size=1, experts=sds, expert_example=experts[0],
                       router_weights=_t(Wr, tdt), d_model=d, num_experts=E,
                       expert_cache_size=E)
    with _CudaToCpu():
        layer = QoSMoELayer(cfg)
        ctx = RequestStateTable(cfg).build_context({"attention_mask": torch.ones(B, S, dtype=torch.long)})
        layer.set_runtime_context(ctx)
        y, (logits, idx) = layer(_t(x, tdt).view(B, S, d))
    return _np(y).reshape(-1, d), _np(logits), idx.numpy().astype(np.int64)


def switch_fixture(name, T, d, E, F, seed, dtype, zipf_s=1.0, B=None, tie_rows=None,
                   store_weights=True):
    B = B or 1
    S = T // B
    x = syn.hidden_states(T, d, seed, dtype)
    Wr, info = syn.router_weight(E, d, seed + 1, zipf_s=zipf_s, dtype=dtype)
    if tie_rows is not None:
        a, b = tie_rows
        Wr[b] = Wr[a]
    wi, wo = syn.switch_expert_weights(E, d, F, seed + 2, dtype=dtype)
    y, logits, idx = run_switch_reference(x, Wr, wi, wo, dtype, B, S)
    arrays = dict(x=x, Wr=Wr, y=y, logits=logits, expert_index=idx)
    if store_weights:
        arrays.update(wi=wi, wo=wo)
    np.savez_compressed(os.path.join(HERE, name), **arrays, meta=json.dumps({"T": T, "d": d, "E": E, "F": F,
                                                           "seed": seed, "dtype": dtype,
                                                           "zipf_s": zipf_s, "B": B, "S": S,
                                                           "tie_rows": tie_rows,
                                                           "weights_regen": "synthetic.switch_expert_weights(E,d,F,seed+2,dtype)"}))
    print(f"{name}: counts={np.bincount(idx, minlength=E).tolist()}")


def switch_routing_fixture(name, T, d, E, seed, dtype, zipf_s=1.0):
    """Router-only golden at a production shape: Router.standard_forward
    (src/harmonymoe/router.py:52-63) -> logits, argmax, max prob.  x is regenerated from seed."""
    from harmonymoe.router import Router, RouterConfig

    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    x = syn.hidden_states(T, d, seed, dtype)
    Wr, info = syn.router_weight(E, d, seed + 1, zipf_s=zipf_s, dtype=dtype)
    r = Router(RouterConfig(d_model=d, num_experts=E, weights=_t(Wr, tdt)))
    with torch.no_grad():
        mask, probs, logits = r(_t(x, tdt))
    idx = torch.argmax(mask, dim=-1).numpy().astype(np.int64)
    np.savez_compressed(os.path.join(HERE, name), Wr=Wr, logits=_np(logits), probs_max=_np(probs)[:, 0],
                        expert_index=idx, meta=json.dumps({"T": T, "d": d, "E": E, "seed": seed,
                                                           "dtype": dtype, "zipf_s": zipf_s,
                                                           "x_regen": "synthetic.hidden_states(T,d,seed,dtype)"}))
    print(f"{name}: top1 hist max share={np.bincount(idx, minlength=E).max() / T:.3f}")


# ----------------------------------------------------------------------------- Qwen
class _QwenMLP(nn.Module):
    """Same names and math as transformers 4.x Qwen2MoeMLP: down(SiLU(gate x) * up x)."""

    def __init__(self, d, I, dtype):
        super().__init__()
        self.gate_proj = nn.Linear(d, I, bias=False, dtype=dtype)
        self.up_proj = nn.Linear(d, I, bias=False, dtype=dtype)
        self.down_proj = nn.Linear(I, d, bias=False, dtype=dtype)
        self.act_fn = nn.SiLU()

    def forward(self, x):
        return self.down_proj(self.act_fn(self.gate_proj(x)) * self.up_proj(x))


class _QwenBlockStub(nn.Module):
    """The transformers-4.x Qwen2MoeSparseMoeBlock attributes ShardedQwenMoE reads
    (qwen_ep_adapter/qwen_ep.py:26-40)."""

    def __init__(self, Wg, p, top_k, norm_topk_prob, dtype):
        super().__init__()
        E, d = Wg.shape
        I = p["gate"].shape[1]
        Is = p["s_gate"].shape[0]
        self.num_experts, self.top_k, self.norm_topk_prob = E, top_k, norm_topk_prob
        self.gate = nn.Linear(d, E, bias=False, dtype=dtype)
        self.experts = nn.ModuleList([_QwenMLP(d, I, dtype) for _ in range(E)])
        self.shared_expert = _QwenMLP(d, Is, dtype)
        self.shared_expert_gate = nn.Linear(d, 1, bias=False, dtype=dtype)
        with torch.no_grad():
            self.gate.weight.copy_(_t(Wg, dtype))
            for e, m in enumerate(self.experts):
                m.gate_proj.weight.copy_(_t(p["gate"][e], dtype))
                m.up_proj.weight.copy_(_t(p["up"][e], dtype))
                m.down_proj.weight.copy_(_t(p["down"][e], dtype))
            self.shared_expert.gate_proj.weight.copy_(_t(p["s_gate"], dtype))
            self.shared_expert.up_proj.weight.copy_(_t(p["s_up"], dtype))
            self.shared_expert.down_proj.weight.copy_(_t(p["s_down"], dtype))
            self.shared_expert_gate.weight.copy_(_t(p["s_gate_w"], dtype))


def _qwen_rank_main(rank, world, port, args, out_q):
    install_shim()
    import torch.distributed as dist
    from qwen_ep import ShardedQwenMoE

    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    xs, Wg, p, top_k, norm, dtype = args
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    block = ShardedQwenMoE(_QwenBlockStub(Wg, p, top_k, norm, tdt), rank, world, "fifo")
    x = _t(xs[rank], tdt)
    with torch.no_grad():
        y, logits = block(x.view(1, -1, x.shape[-1]))
    out_q.put((rank, _np(y).reshape(x.shape), _np(logits)))
    dist.barrier()
    dist.destroy_process_group()


def run_qwen_reference(xs, Wg, p, top_k, norm, dtype):
    """ShardedQwenMoE on len(xs) gloo CPU ranks; rank r serves tokens xs[r]."""
    import torch.multiprocessing as mp

    world = len(xs)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_qwen_rank_main, args=(r, world, port, (xs, Wg, p, top_k, norm, dtype), q))
             for r in range(world)]
    for pr in procs:
        pr.start()
    res = {}
    for _ in range(world):
        r, y, lg = q.get(timeout=600)
        res[r] = (y, lg)
    for pr in procs:
        pr.join(timeout=120)
        if pr.exitcode != 0:
            raise RuntimeError(f"reference rank exited with {pr.exitcode}")
    return [res[r][0] for r in range(world)], [res[r][1] for r in range(world)]


def qwen_fixture(name, T, d, E, I, Is, top_k, seed, dtype, world=1, zipf_s=None, norm=False,
                 store_weights=True, tie_rows=None):
    xs = [syn.hidden_states(T, d, seed + 100 * r, dtype) for r in range(world)]
    Wg, info = syn.router_weight(E, d, seed + 1, zipf_s=zipf_s, dtype=dtype)
    if tie_rows is not None:
        Wg[tie_rows[1]] = Wg[tie_rows[0]]
    p = syn.qwen_expert_weights(E, d, I, Is, seed + 2, dtype=dtype)
    ys, logits = run_qwen_reference(xs, Wg, p, top_k, norm, dtype)
    arrays = dict(x=np.stack(xs), y=np.stack(ys), logits=np.stack(logits), Wg=Wg)
    if store_weights:
        arrays.update({k: v for k, v in p.items()})
    np.savez_compressed(os.path.join(HERE, name), **arrays,
                        meta=json.dumps({"T": T, "d": d, "E": E, "I": I, "Is": Is, "top_k": top_k,
                                         "seed": seed, "dtype": dtype, "world": world,
                                         "zipf_s": zipf_s, "norm_topk_prob": norm, "tie_rows": tie_rows,
                                         "weights_regen": "synthetic.qwen_expert_weights(E,d,I,Is,seed+2,dtype)"}))
    print(f"{name}: world={world} y[0] absmax={np.abs(ys[0]).max():.4f}")


# ----------------------------------------------------------------------------- scheduler
def _reference_scheduler(policy, E, G, eq_tokens, rank=0, expert_to_gpu=None, placement_path=None):
    from harmonymoe.scheduler import Scheduler

    with _CudaToCpu():
        s = Scheduler(rank=rank, scheduling_policy=policy, num_experts=E, eq_tokens=eq_tokens,
                      num_gpus=G, d_model=8, expert_placement=placement_path, layer_idx=0)
    if expert_to_gpu is not None:
        s.expert_to_gpu = torch.tensor(expert_to_gpu, dtype=torch.long)
    return s


def scheduler_fixture(name):
    """Plans S[src, e, dst] from the reference's schedule_harmony / schedule_fixed."""
    cases = []
    g = syn.rng(4242)
    specs = [
        # (E, G, eq_tokens, count model, placement)
        (8, 2, 150, "uniform", "naive"),
        (8, 4, 150, "zipf1.5", "naive"),
        (64, 4, 150, "zipf1.0", "naive"),
        (64, 8, 150, "zipf1.5", "naive"),
        (60, 4, 150, "zipf1.5", "naive"),
        (60, 4, 0, "zipf1.5", "naive"),
        (60, 8, 150, "zipf1.5", "exflow"),
        (60, 8, 150, "uniform", "exflow"),
        (60, 8, 150, "zero_rank", "exflow"),
        (64, 8, 150, "hot_one", "naive"),
        (64, 2, 1000000, "zipf1.5", "naive"),
        (60, 2, 150, "zipf1.5", "exflow"),
    ]
    for E, G, eq, model, plc in specs:
        T = 4096
        meta = np.zeros((G, E), dtype=np.int64)
        for r in range(G):
            if model == "uniform":
                pr = np.full(E, 1.0 / E)
            elif model.startswith("zipf"):
                pr = syn.zipf_targets(E, float(model[4:]))
            elif model == "hot_one":
                pr = np.full(E, 0.3 / (E - 1))
                pr[5] = 0.7
            else:  # zero_rank: rank 3 has no tokens at all
                pr = syn.zipf_targets(E, 1.0)
            n = 0 if (model == "zero_rank" and r == 3) else T
            meta[r] = g.multinomial(n, pr / pr.sum())
        if plc == "naive":
            e2g = (np.arange(E) // (E // G)).tolist()
        else:
            lay = syn.exflow_uneven_placement(E, G)[0]
            e2g = [0] * E
            for gpu, lst in enumerate(lay):
                for e in lst:
                    e2g[e] = gpu
        s = _reference_scheduler("harmony", E, G, eq, expert_to_gpu=e2g)
        with _CudaToCpu():
            harm = s(torch.tensor(meta, dtype=torch.int32)).numpy().astype(np.int64)
            fixed = s.schedule_fixed(torch.tensor(meta, dtype=torch.int32)).numpy().astype(np.int64)
        cases.append({"E": E, "G": G, "eq_tokens": eq, "counts": model, "placement": plc,
                      "expert_to_gpu": e2g, "meta": meta.tolist(), "harmony": harm.tolist(),
                      "fixed": fixed.tolist()})
    # the exflow JSON path proper: Scheduler('exflow') reads [layer][gpu] -> experts from a file
    tmp = os.path.join(HERE, "_exflow_tmp.json")
    with open(tmp, "w") as f:
        json.dump(syn.exflow_uneven_placement(60, 8, num_layers=2), f)
    try:
        s = _reference_scheduler("exflow", 60, 8, 150, placement_path=tmp)
        exflow_e2g = s.expert_to_gpu.numpy().tolist()
        exflow_cache = [list(map(int, x)) for x in s.get_cache()]
    finally:
        os.remove(tmp)
    with open(os.path.join(HERE, name), "w") as f:
        json.dump({"cases": cases, "exflow_60_on_8": {"expert_to_gpu": exflow_e2g,
                                                      "gpu_to_experts": exflow_cache}}, f)
    print(f"{name}: {len(cases)} plans")


def dispatch_fixture(name):
    """Send-buffer order (distribute_tokens) and receive-side expert lists (generate_expert_mask)
    for small plans.  hidden_states[t] = t, so the send buffer spells out token ids."""
    out = []
    g = syn.rng(777)
    for (E, G, T, eq) in [(8, 2, 64, 4), (8, 4, 96, 3), (12, 4, 128, 5), (6, 3, 40, 1)]:
        ranks_ids = [g.integers(0, E, size=T) for _ in range(G)]
        ranks_ids[0][: T // 2] = 0  # a hot expert to force migration
        meta = np.stack([np.bincount(ids, minlength=E) for ids in ranks_ids])
        e2g = (np.arange(E) // (E // G)).tolist()
        s0 = _reference_scheduler("harmony", E, G, eq, expert_to_gpu=e2g)
        with _CudaToCpu():
            sched = s0(torch.tensor(meta, dtype=torch.int32))
        sched_list = sched.tolist()
        per_rank = []
        for r in range(G):
            s = _reference_scheduler("harmony", E, G, eq, rank=r, expert_to_gpu=e2g)
            hid = torch.arange(T, dtype=torch.float32)[:, None].repeat(1, 8)
            expert_indices = [torch.nonzero(torch.tensor(ranks_ids[r] == e)).flatten() for e in range(E)]
            n_send = int(sched[r].sum())
            with _CudaToCpu():
                tokens, splits = s.distribute_tokens(sched_list, hid, expert_indices, n_send)
                recv_total = int(sched[:, :, r].sum())
                masks = s.generate_expert_mask(sched, recv_total)
                _, recv_splits = s.allocate_recv_tensors(sched)
            per_rank.append({"send_tokens": tokens[:, 0].long().tolist(), "send_splits": list(map(int, splits)),
                             "recv_splits": list(map(int, recv_splits)),
                             "expert_mask": [m.tolist() for m in masks]})
        out.append({"E": E, "G": G, "T": T, "eq_tokens": eq, "expert_ids": [x.tolist() for x in ranks_ids],
                    "schedule": sched_list, "ranks": per_rank})
    with open(os.path.join(HERE, name), "w") as f:
        json.dump(out, f)
    print(f"{name}: {len(out)} cases")


# ----------------------------------------------------------------------------- QoS planner
def planner_fixture(name):
    """Token scores, expert priorities and execution plans from the reference's QoSPlanner
    (src/qosmoe/planner.py:63-237) on seeded inputs; the runtime context carries fixed
    per-token vectors (the reference derives them from wall-clock deadlines)."""
    from types import SimpleNamespace

    from qosmoe.planner import QoSPlanner

    g = syn.rng(5150)
    out = {}
    meta = []
    score_cases = [
        # (T, d, E, prev, mode, invalid fraction)
        (96, 64, 8, "same", "router_var", 0.1),
        (64, 32, 8, None, "router_var", 0.0),
        (80, 48, 16, "other", "router_var", 0.25),
        (50, 64, 8, "same", "none", 0.0),
    ]
    for ci, (T, d, E, prev, mode, inv) in enumerate(score_cases):
        args = SimpleNamespace(qos_attention_mode=mode, qos_target_batch=64, qos_epsilon=1e-6,
                               qos_alpha=1.0, qos_beta=0.1, qos_delta=0.5)
        x = g.standard_normal((T, d)).astype(np.float32)
        xp = None
        if prev == "same":
            xp = (x + 0.3 * g.standard_normal((T, d))).astype(np.float32)
        elif prev == "other":
            xp = g.standard_normal((T + 7, d)).astype(np.float32)
        logits = (2.0 * g.standard_normal((T, E))).astype(np.float32)
        eidx = np.argmax(logits, axis=1).astype(np.int64)
        seq_pri = g.uniform(0.5, 2.0, T).astype(np.float32)
        rem = g.integers(1, 300, T).astype(np.float32)
        valid = (g.uniform(0, 1, T) >= inv).astype(np.float32)
        ctx = SimpleNamespace(flat_remaining_tokens=torch.from_numpy(rem),
                              flat_seq_priority=torch.from_numpy(seq_pri),
                              flat_valid_mask=torch.from_numpy(valid))
        pl = QoSPlanner(args, rank=0, num_experts=E, num_gpus=1, d_model=d)
        with _CudaToCpu():
            sc = pl.compute_token_scores(torch.from_numpy(x), None if xp is None else torch.from_numpy(xp),
                                         torch.from_numpy(logits), torch.from_numpy(eidx), ctx)
            lists = [torch.nonzero(torch.from_numpy(eidx) == e).flatten() for e in range(E)]
            pri = pl.aggregate_expert_priority(lists, sc)
        key = f"s{ci}"
        out.update({key + "_x": x, key + "_logits": logits, key + "_eidx": eidx, key + "_seq": seq_pri,
                    key + "_rem": rem, key + "_valid": valid, key + "_score": _np(sc), key + "_prio": _np(pri)})
        if xp is not None:
            out[key + "_xprev"] = xp
        meta.append(dict(key=key, T=T, d=d, E=E, prev=prev, mode=mode))
    plans = []
    plan_cases = [
        # (E, active experts, cache contents, cache_size)
        (8, [0, 1, 2, 3, 4, 5, 6, 7], [], 2),
        (8, [1, 3, 4, 6], [3, 6], 2),
        (8, [0, 2, 5, 7], [2, 9, 5, 1], 4),
        (16, list(range(16)), [4, 8, 12], 3),
        (8, [2, 4], [2, 4, 6], 3),
        (8, [1, 2, 3], [], 8),
    ]
    for E, active, cache, cs in plan_cases:
        pr = g.standard_normal(E).astype(np.float32)
        pr[2] = pr[3]  # a tie: the stable sort keeps expert id order
        mask = [torch.zeros(3 if e in active else 0, dtype=torch.long) for e in range(E)]
        pl = QoSPlanner(SimpleNamespace(), rank=0, num_experts=E, num_gpus=1, d_model=8)
        plan = pl.build_exec_plan(mask, torch.from_numpy(pr), list(cache), cs)
        plans.append(dict(E=E, active=active, cache=cache, cache_size=cs, priority=pr.tolist(),
                          expert_order=[int(v) for v in plan.expert_order],
                          slot_idxs=[int(v) for v in plan.slot_idxs],
                          need_loading=[int(v) for v in plan.need_loading]))
    out["meta"] = np.array(json.dumps(dict(score_cases=meta, plans=plans)))
    np.savez_compressed(os.path.join(HERE, name), **out)
    print("wrote", name)


def main():
    install_shim()
    torch.manual_seed(0)
    # Switch top-1 block, world=1 (QoSMoELayer resident-all path)
    switch_fixture("switch_f32_small.npz", T=96, d=64, E=8, F=128, seed=11, dtype="f32", B=3)
    switch_fixture("switch_bf16_small.npz", T=96, d=64, E=8, F=128, seed=12, dtype="bf16", B=3)
    switch_fixture("switch_f32_ties.npz", T=64, d=32, E=8, F=64, seed=13, dtype="f32", B=2,
                   zipf_s=None, tie_rows=(2, 5))
    switch_fixture("switch_f32_mid.npz", T=256, d=128, E=16, F=256, seed=14, dtype="f32", B=1,
                   store_weights=False)
    # Router-only at the Switch-base-64 shape (C1 f32 and C2 bf16)
    switch_routing_fixture("switch_routing_c1_f32.npz", T=1024, d=768, E=64, seed=21, dtype="f32")
    switch_routing_fixture("switch_routing_c2_bf16.npz", T=1024, d=768, E=64, seed=22, dtype="bf16")
    # Qwen top-4 + shared expert (ShardedQwenMoE on gloo ranks)
    qwen_fixture("qwen_tiny_f32.npz", T=16, d=64, E=8, I=32, Is=64, top_k=4, seed=20261016, dtype="f32")
    qwen_fixture("qwen_tiny_bf16.npz", T=16, d=64, E=8, I=32, Is=64, top_k=4, seed=20261016, dtype="bf16")
    qwen_fixture("qwen_small_bf16.npz", T=128, d=128, E=60, I=64, Is=256, top_k=4, seed=31,
                 dtype="bf16", zipf_s=1.5, store_weights=False)
    qwen_fixture("qwen_small_f32_w4.npz", T=64, d=128, E=60, I=64, Is=256, top_k=4, seed=32,
                 dtype="f32", world=4, zipf_s=1.5, store_weights=False)
    qwen_fixture("qwen_ties_bf16.npz", T=32, d=64, E=8, I=32, Is=64, top_k=4, seed=34,
                 dtype="bf16", tie_rows=(1, 6))
    qwen_fixture("qwen_norm_f32.npz", T=32, d=64, E=8, I=32, Is=64, top_k=4, seed=33, dtype="f32",
                 norm=True)
    # Scheduler plans and dispatch order
    scheduler_fixture("harmony_plans.json")
    dispatch_fixture("dispatch_order.json")
    # QoS planner: token scores, expert priorities, execution plans
    planner_fixture("qos_planner.npz")


if __name__ == "__main__":
    main()
