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
