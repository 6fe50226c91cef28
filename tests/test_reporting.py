"""Run outputs in the reference's formats (src/start_qosmoe.py:297-333,
src/real_token_gantt_trace.py:18-131), on the CPU with layers that carry statistics only."""
import csv
import json

import numpy as np
import torch.nn as nn

from dsca_moe_b200 import reporting
from dsca_moe_b200.layers import QoSMoELayer


def _stat_layer(idx, n):
    layer = QoSMoELayer.__new__(QoSMoELayer)
    nn.Module.__init__(layer)
    layer.layer_idx = idx
    layer.latencies = [0.5 + i for i in range(n)]
    layer.tot_num_toks_send = [100 + i for i in range(n)]
    layer.tot_num_toks_recv = [200 + i for i in range(n)]
    layer.expert_freqs = [[i, 1, 2] for i in range(n)]
    layer.expert_swaps = [i % 2 for i in range(n)]
    return layer


def test_run_outputs_have_the_reference_layout(tmp_path):
    model = nn.Sequential(nn.Linear(2, 2), _stat_layer(1, 4), nn.Sequential(_stat_layer(3, 4)))
    reporting.write_run_outputs(str(tmp_path), 0, [0.25, 0.5, 0.75], model, warmup_rounds=1,
                                run_info={"batch_size": 16, "path": str(tmp_path)}, run_start=1.0, run_end=2.0)
    with open(tmp_path / "0" / "e2e.csv") as f:
        rows = list(csv.DictReader(f))
    assert list(rows[0].keys()) == ["iteration", "latency (s)"] and len(rows) == 3
    assert float(rows[2]["latency (s)"]) == 0.75
    for idx in (1, 3):
        with open(tmp_path / "0" / f"moe_layer-{idx}.csv") as f:
            rows = list(csv.DictReader(f))
        assert list(rows[0].keys()) == ["iteration", "latency (ms)", "total number of tokens sent",
                                        "total number of tokens recv", "expert distribution", "num expert swaps",
                                        "num prefetch launched"]
        assert len(rows) == 3 and rows[0]["iteration"] == "0" and float(rows[0]["latency (ms)"]) == 1.5
    info = json.load(open(tmp_path / "data.json"))
    assert info["start"] == 1.0 and info["end"] == 2.0 and info["system_name"] == "qosmoe"
    assert info["batch_size"] == 16


def test_token_trace_rows(tmp_path, monkeypatch):
    monkeypatch.setenv("QOSMOE_REAL_TOKEN_TRACE_DIR", str(tmp_path))
    monkeypatch.setenv("QOSMOE_TRACE_RANK", "3")
    monkeypatch.setenv("QOSMOE_TRACE_MAX_TOKENS", "2")
    tr = reporting.TokenTrace()
    ids = np.array([[0, 2], [2, 1], [0, 1], [2, 0]])
    tr.record_block(5, ids, 10.0, 12.0, 15.0)
    tr.flush()
    with open(tmp_path / "real_token_trace_qosmoe_rank3.csv") as f:
        rows = list(csv.DictReader(f))
    assert list(rows[0].keys()) == reporting.TRACE_HEADER
    got = [(int(r["expert_id"]), int(r["token_id"])) for r in rows]
    assert got == [(0, 0), (0, 2), (1, 1), (1, 2), (2, 0), (2, 1)]  # first two tokens per expert
    assert all(r["layer"] == "5" and r["rank"] == "3" and float(r["wait_ms"]) == 2.0 and float(r["expert_ms"]) == 3.0
               for r in rows)
