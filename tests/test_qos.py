"""QoS planner and expert-cache plan (CPU): the oracle and the product's host plan against
fixtures made by the reference's own QoSPlanner (src/qosmoe/planner.py:63-237,
tests/golden/make_golden.py:planner_fixture)."""
import numpy as np
import pytest
import torch

from golden_io import load
from oracle import oracle as O
from dsca_moe_b200.qos import build_exec_plan, match_token_length


def _case(z, c):
    k = c["key"]
    xp = z[k + "_xprev"] if k + "_xprev" in z else None
    return k, xp


def test_token_scores_and_expert_priority_match_reference():
    z, m = load("qos_planner.npz")
    for c in m["score_cases"]:
        k, xp = _case(z, c)
        sc = O.qos_token_scores(z[k + "_x"], xp, z[k + "_logits"], z[k + "_eidx"], z[k + "_seq"],
                                z[k + "_rem"], z[k + "_valid"], c["d"], mode=c["mode"])
        ok = z[k + "_valid"] != 0
        assert np.array_equal(sc[~ok], np.full((~ok).sum(), -1e9))
        assert np.abs(sc[ok] - z[k + "_score"][ok]).max() <= 1e-6 * np.abs(z[k + "_score"][ok]).max()
        pr = O.qos_expert_priority(sc, z[k + "_eidx"], c["E"])
        assert np.abs(pr - z[k + "_prio"]).max() <= 1e-6 * np.abs(z[k + "_prio"]).max()


@pytest.mark.parametrize("impl", ["oracle", "product"])
def test_exec_plans_match_reference(impl):
    _, m = load("qos_planner.npz")
    for p in m["plans"]:
        if impl == "oracle":
            got = O.qos_exec_plan(p["active"], p["priority"], p["cache"], p["cache_size"])
        else:
            r = build_exec_plan(p["active"], p["priority"], p["cache"], p["cache_size"])
            got = (r.expert_order, r.slot_idxs, r.need_loading)
        assert got == (p["expert_order"], p["slot_idxs"], p["need_loading"]), p


def test_exec_plan_product_matches_oracle_on_random_states():
    g = np.random.default_rng(7)
    for _ in range(300):
        E = int(g.integers(1, 40))
        cs = int(g.integers(1, 10))
        active = sorted(set(g.integers(0, E, int(g.integers(0, E + 1))).tolist()))
        cache = [int(v) for v in g.choice(np.arange(-1, E), size=min(cs, E + 1), replace=False)]
        pr = np.round(g.standard_normal(E), 1).tolist()  # rounded: many ties
        r = build_exec_plan(active, pr, cache, cs)
        assert (r.expert_order, r.slot_idxs, r.need_loading) == O.qos_exec_plan(active, pr, cache, cs)


def test_match_token_length_follows_reference_rules():
    v = torch.tensor([1.0, 2.0, 3.0])
    assert torch.equal(match_token_length(v, 3), v)
    assert torch.equal(match_token_length(v, 6), torch.tensor([1.0, 1.0, 2.0, 2.0, 3.0, 3.0]))
    assert torch.equal(match_token_length(v, 2), torch.tensor([1.0, 2.0]))
    assert torch.equal(match_token_length(v, 5), torch.tensor([1.0, 2.0, 3.0, 3.0, 3.0]))
    assert torch.equal(match_token_length(torch.zeros(0), 4), torch.zeros(4))
    assert match_token_length(None, 4) is None
