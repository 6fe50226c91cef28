"""Expert cache + QoS planner on the GPU.

* dsca_qos_priority: token scores and expert priorities against the oracle's restatement of
  QoSPlanner.compute_token_scores / aggregate_expert_priority (src/qosmoe/planner.py:63-170),
  itself pinned to the reference by tests/test_qos.py (float32 device arithmetic: 1e-5 relative).
* the expert-cache path (pinned host weights, device slots, QoS-planned loads) gives the
  all-resident output bit for bit, over repeated calls and with fewer slots than active experts;
  its plan is build_exec_plan's on the device priorities and the cache state before the call.
* QoSMoELayer with the reference's default expert_cache_size (2) runs the cache path.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from dsca_moe_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _t(a, dtype, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=dev, dtype=dtype)


def _engines(kind, dtype, dev, slots, T=300, d=128, E=16, seed=7):
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_relu, pack_swiglu

    tau = "bf16" if dtype == torch.bfloat16 else "f32"
    x = syn.hidden_states(T, d, seed, tau)
    if kind == "switch":
        Wr, _ = syn.router_weight(E, d, seed + 1, zipf_s=1.0, dtype=tau)
        wi, wo = syn.switch_expert_weights(E, d, 256, seed + 2, dtype=tau)

        def make(cache):
            pe = pack_relu(_t(wi, dtype, "cpu"), _t(wo, dtype, "cpu"), dtype=dtype,
                           device="cpu" if cache else dev)
            return MoEEngine(_t(Wr, dtype, dev), pe, top_k=1, route_mode=L.ROUTE_SWITCH_TOP1,
                             cache_slots=cache, device=dev)
    else:
        Wr, _ = syn.router_weight(E, d, seed + 1, zipf_s=1.5, dtype=tau)
        p = syn.qwen_expert_weights(E, d, 64, 192, seed + 2, dtype=tau)

        def make(cache):
            loc = "cpu" if cache else dev
            pe = pack_swiglu(_t(p["gate"], dtype, loc), _t(p["up"], dtype, loc), _t(p["down"], dtype, loc),
                             shared=(_t(p["s_gate"], dtype, loc), _t(p["s_up"], dtype, loc),
                                     _t(p["s_down"], dtype, loc)), dtype=dtype, device=loc)
            return MoEEngine(_t(Wr, dtype, dev), pe, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK,
                             shared_gate_weight=_t(p["s_gate_w"], dtype, dev), cache_slots=cache, device=dev)
    return x, make(None), make(slots)


@pytest.mark.parametrize("kind,dtype,slots", [("switch", torch.bfloat16, 4), ("qwen", torch.bfloat16, 3),
                                              ("qwen", torch.float32, 1), ("switch", torch.float32, 16)])
def test_cache_path_equals_resident(cuda, kind, dtype, slots):
    from dsca_moe_b200.qos import QoSInputs

    x, res, cached = _engines(kind, dtype, cuda, slots)
    xd = _t(x, dtype, cuda)
    want = res.forward(xd)["out"].clone()
    prev = None
    for it in range(3):
        before = list(cached.cache.resident)
        q = QoSInputs(x_prev=prev, seq_priority=torch.linspace(0.5, 2.0, xd.shape[0]),
                      remaining=torch.arange(xd.shape[0], dtype=torch.float32) % 50,
                      valid=(torch.arange(xd.shape[0]) % 11 != 3).float())
        r = cached.forward(xd, qos=q)
        torch.cuda.synchronize()
        cached.check()
        assert torch.equal(r["out"], want), f"iteration {it}"
        # the plan is build_exec_plan on the device priorities and the cache state before the call
        counts = r["counts"].cpu().numpy()
        prio = r["expert_priority"].cpu().numpy()
        order, slot_idxs, need = O.qos_exec_plan(list(np.nonzero(counts)[0]), prio, before, slots)
        plan = cached.last_exec_plan
        assert (plan.expert_order, plan.slot_idxs, plan.need_loading) == (order, slot_idxs, need)
        assert cached.last_loads == len(need)
        prev = r["out"].clone()
    if slots >= 16:  # every expert fits: nothing is loaded after the first call
        assert cached.last_loads == 0


@pytest.mark.parametrize("dtype,with_prev,mode", [(torch.bfloat16, True, 0), (torch.float32, False, 0),
                                                  (torch.bfloat16, False, 1)])
def test_qos_scores_match_oracle(cuda, dtype, with_prev, mode):
    from dsca_moe_b200.qos import QoSInputs

    x, _, cached = _engines("qwen", dtype, cuda, 2, T=257, seed=21)
    cached.qos_params["attention_mode"] = mode
    T = x.shape[0]
    xd = _t(x, dtype, cuda)
    g = np.random.default_rng(3)
    xp = (x + 0.5 * g.standard_normal(x.shape)).astype(np.float32) if with_prev else None
    seq = g.uniform(0.5, 2.0, T).astype(np.float32)
    rem = g.integers(1, 300, T).astype(np.float32)
    valid = (g.uniform(0, 1, T) > 0.1).astype(np.float32)
    q = QoSInputs(x_prev=None if xp is None else _t(xp, dtype, cuda), seq_priority=torch.from_numpy(seq),
                  remaining=torch.from_numpy(rem), valid=torch.from_numpy(valid))
    r = cached.forward(xd, qos=q)
    torch.cuda.synchronize()
    cached.check()
    lg = r["logits"].float().cpu().numpy()
    ids = r["topk_ids"].cpu().numpy()
    xq = xd.float().cpu().numpy()
    xpq = None if xp is None else q.x_prev.float().cpu().numpy()
    want = O.qos_token_scores(xq, xpq, lg, ids[:, 0], seq, rem, valid, x.shape[1],
                              mode="router_var" if mode == 0 else "none")
    got = r["token_score"].cpu().numpy()
    ok = valid != 0
    assert np.array_equal(got[~ok], np.full((~ok).sum(), -1e9, np.float32))
    assert np.abs(got[ok] - want[ok]).max() <= 1e-5 * np.abs(want[ok]).max()
    pr = O.qos_expert_priority(got.astype(np.float64), ids, cached.E)
    gp = r["expert_priority"].cpu().numpy()
    assert np.abs(gp - pr).max() <= 1e-5 * np.abs(pr).max()


def test_plugin_layer_default_cache_size_runs_cache_path(cuda):
    from dsca_moe_b200 import QoSMoEConfig, QoSMoELayer, RequestStateTable

    T, d, E, F = 128, 64, 8, 128
    x = syn.hidden_states(T, d, 5, "f32")
    Wr, _ = syn.router_weight(E, d, 6, zipf_s=1.0, dtype="f32")
    wi, wo = syn.switch_expert_weights(E, d, F, 7, dtype="f32")
    sds = [{"wi.weight": torch.from_numpy(wi[e]), "wo.weight": torch.from_numpy(wo[e])} for e in range(E)]
    outs = []
    for cache_size in (2, E):  # 2 = the reference's default (src/qosmoe/config.py:19)
        cfg = QoSMoEConfig(rank=0, world_size=1, experts=sds, router_weights=torch.from_numpy(Wr), d_model=d,
                           num_experts=E, expert_cache_size=cache_size, collect_stats=True)
        layer = QoSMoELayer(cfg)
        assert (layer.engine.cache is not None) == (cache_size < E)
        layer.set_runtime_context(RequestStateTable(cfg).build_context({"attention_mask": torch.ones(2, 64)}))
        y, (logits, idx) = layer(_t(x, torch.float32, cuda).view(2, 64, d))
        torch.cuda.synchronize()
        outs.append(y.clone())
        st = layer.get_statistics()[0]
        assert st["num expert swaps"] == (layer.engine.last_loads if cache_size < E else 0)
    assert torch.equal(outs[0], outs[1])
    y_ref, *_ = O.switch_forward(x, Wr, wi, wo, "f32")
    assert O.max_rel_err(outs[0].reshape(T, d).cpu().numpy(), y_ref) < 1e-4


def test_next_layer_prefetch_loads_top_priority_experts(cuda):
    """qos_enable_prefetch (src/qosmoe/moe_layer.py:164-194): after a layer's forward, the top
    qos_prefetch_topk experts by its priority (at most qos_prefetch_budget_experts) are copied
    into the next layer's expert cache, round robin over its slots, skipping cached ones; the
    next layer's output is unchanged by what was prefetched."""
    from dsca_moe_b200 import QoSMoEConfig, QoSMoELayer, RequestStateTable

    T, d, E, F = 128, 64, 8, 128
    x = syn.hidden_states(T, d, 15, "f32")
    Wr, _ = syn.router_weight(E, d, 16, zipf_s=1.0, dtype="f32")
    wi, wo = syn.switch_expert_weights(E, d, F, 17, dtype="f32")
    sds = [{"wi.weight": torch.from_numpy(wi[e]), "wo.weight": torch.from_numpy(wo[e])} for e in range(E)]

    def layer(idx, prefetch):
        cfg = QoSMoEConfig(rank=0, world_size=1, experts=sds, router_weights=torch.from_numpy(Wr), d_model=d,
                           num_experts=E, expert_cache_size=3, layer_idx=idx, collect_stats=True,
                           qos_enable_prefetch=prefetch, qos_prefetch_topk=2, qos_prefetch_budget_experts=2)
        lay = QoSMoELayer(cfg)
        lay.set_runtime_context(RequestStateTable(cfg).build_context({"attention_mask": torch.ones(2, 64)}))
        return lay

    a, b = layer(0, True), layer(1, False)
    a.set_next_layer(b)
    before = list(b.engine.cache.resident)
    xd = _t(x, torch.float32, cuda).view(2, 64, d)
    ya, _ = a(xd)
    torch.cuda.synchronize()
    prio = a.engine.last_priority
    top = [int(e) for e in torch.topk(torch.as_tensor(prio).clamp_min(0), k=2).indices]
    want = [e for e in top if e not in before]
    assert a.get_statistics()[0]["num prefetch launched"] == len(want)
    for e in top:
        assert e in b.engine.cache.resident
    yb, _ = b(ya)
    ref = layer(2, False)
    yr, _ = ref(ya)
    torch.cuda.synchronize()
    assert torch.equal(yb, yr)
