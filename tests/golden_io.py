"""Loading helpers for the fixtures in tests/golden (made by tests/golden/make_golden.py)."""
import json
import os

import numpy as np

from dsca_moe_b200 import synthetic as syn

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    z = np.load(os.path.join(GOLDEN, name))
    d = {k: z[k] for k in z.files if k != "meta"}
    return d, json.loads(str(z["meta"]))


def switch_weights(z, m):
    if "wi" in z:
        return z["wi"], z["wo"]
    return syn.switch_expert_weights(m["E"], m["d"], m["F"], m["seed"] + 2, dtype=m["dtype"])


def qwen_weights(z, m):
    keys = ["gate", "up", "down", "s_gate", "s_up", "s_down", "s_gate_w"]
    if "gate" in z:
        return {k: z[k] for k in keys}
    return syn.qwen_expert_weights(m["E"], m["d"], m["I"], m["Is"], m["seed"] + 2, dtype=m["dtype"])


def json_fixture(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def assert_logits_close(ours, ref, tau):
    """Logits from the fixed chunked order vs the reference's own accumulation order: f32 within
    a few ulps; bf16 equal or one bf16 ulp apart on under 1 % of the entries."""
    ours = np.asarray(ours, np.float32)
    ref = np.asarray(ref, np.float32)
    if tau == "f32":
        assert np.all(np.abs(ours - ref) <= 4e-6 * np.maximum(np.abs(ref), 1.0))
    else:
        a = ours.view(np.int32).astype(np.int64)
        b = ref.view(np.int32).astype(np.int64)
        diff = np.abs(a - b) >> 16
        assert diff.max() <= 1
        assert (diff > 0).mean() < 0.01


def routing_near_ties(logits, k, tau="bf16"):
    """Tokens whose k-th and (k+1)-th probabilities are within 2^-7 (bf16 logits: one logit ulp)
    or 1e-5 (f32 logits: a few ulps) of each other: another valid summation order can swap them."""
    from oracle import oracle as O

    return O.near_tie_tokens(logits, k, tau, rel=2.0 ** -7 if tau == "bf16" else 1e-5)
