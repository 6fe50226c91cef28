"""Run outputs in the reference's formats, so that its analysis scripts read runs of this block.

write_run_outputs — the files src/start_qosmoe.py:297-333 writes after a run:
    {path}/{rank}/e2e.csv                 iteration, latency (s)
    {path}/{rank}/moe_layer-{idx}.csv     iteration + the keys of QoSMoELayer.get_statistics()
    {path}/data.json                      (rank 0) start, end, the run arguments, system_name
TokenTrace    — the per-(token, expert) CSV of src/real_token_gantt_trace.py:18-131
    ({dir}/real_token_trace_{system}_rank{rank}.csv, same columns and environment variables).
    The reference turns it on unless QOSMOE_REAL_TOKEN_TRACE is "0" and synchronises the device
    per expert; here it is off unless QOSMOE_REAL_TOKEN_TRACE is "1".  The block runs all experts
    in one grouped launch, so every expert of a forward gets the block's start and end times.
"""
from __future__ import annotations

import atexit
import csv
import json
import os
import time
from pathlib import Path

TRACE_HEADER = ["system", "rank", "iteration", "layer", "job_id", "token_id", "expert_id", "ready_ms",
                "expert_start_ms", "expert_end_ms", "wait_ms", "expert_ms", "note"]


def write_run_outputs(path: str, rank: int, latencies, model=None, warmup_rounds: int = 0, run_info=None,
                      run_start: float | None = None, run_end: float | None = None):
    """The reference's per-run files (src/start_qosmoe.py:297-333).  `latencies`: seconds per
    iteration; `model`: the swapped model (its QoSMoELayer statistics become moe_layer-*.csv);
    `run_info`: the run's arguments (a dict or an argparse namespace) for data.json."""
    from .plugin import get_qosmoe_layers

    out = os.path.join(path, str(rank))
    os.makedirs(out, exist_ok=True)
    with open(os.path.join(out, "e2e.csv"), "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=["iteration", "latency (s)"])
        w.writeheader()
        for i, lat in enumerate(latencies):
            w.writerow({"iteration": i, "latency (s)": lat})
    if model is not None:
        for layer in get_qosmoe_layers(model):
            stats = layer.get_statistics()[warmup_rounds:]
            if not stats:
                continue
            with open(os.path.join(out, f"moe_layer-{layer.layer_idx}.csv"), "w", newline="") as f:
                w = csv.DictWriter(f, fieldnames=["iteration"] + list(stats[0].keys()))
                w.writeheader()
                for i, row in enumerate(stats):
                    w.writerow({"iteration": i, **row})
    if rank == 0:
        info = dict(vars(run_info)) if run_info is not None and not isinstance(run_info, dict) else dict(run_info or {})
        info["system_name"] = "qosmoe"
        with open(os.path.join(path, "data.json"), "w") as f:
            json.dump({"start": run_start, "end": run_end, **info}, f, indent=4, default=str)


class TokenTrace:
    """Buffered writer of the reference's token trace rows (src/real_token_gantt_trace.py)."""

    def __init__(self):
        self.rows = []
        self.job_id = 0
        atexit.register(self.flush)

    @staticmethod
    def enabled() -> bool:
        return os.environ.get("QOSMOE_REAL_TOKEN_TRACE", "0") == "1"

    @staticmethod
    def now_ms() -> float:
        return time.perf_counter_ns() / 1e6

    def record_block(self, layer_idx: int, topk_ids, ready_ms: float, start_ms: float, end_ms: float,
                     note: str = "dsca grouped expert GEMM (block start / end)"):
        """One job: for every expert, its first QOSMOE_TRACE_MAX_TOKENS tokens (token order)."""
        import numpy as np

        self.job_id += 1
        system = os.environ.get("QOSMOE_TRACE_SYSTEM", "qosmoe")
        rank = int(os.environ.get("QOSMOE_TRACE_RANK", "0"))
        iteration = int(os.environ.get("QOSMOE_TRACE_ITER", "-1"))
        max_tokens = int(os.environ.get("QOSMOE_TRACE_MAX_TOKENS", "64"))
        ids = np.asarray(topk_ids).reshape(len(topk_ids), -1)
        for e in np.unique(ids[ids >= 0]):
            toks = np.nonzero((ids == e).any(axis=1))[0]
            if max_tokens > 0:
                toks = toks[:max_tokens]
            for t in toks:
                self.rows.append({"system": system, "rank": rank, "iteration": iteration, "layer": int(layer_idx),
                                  "job_id": self.job_id, "token_id": int(t), "expert_id": int(e),
                                  "ready_ms": ready_ms, "expert_start_ms": start_ms, "expert_end_ms": end_ms,
                                  "wait_ms": start_ms - ready_ms, "expert_ms": end_ms - start_ms, "note": note})
        if len(self.rows) >= 2048:
            self.flush()

    def flush(self):
        if not self.rows:
            return
        out_dir = Path(os.environ.get("QOSMOE_REAL_TOKEN_TRACE_DIR", os.environ.get("QOSMOE_TRACE_DIR", ".")))
        out_dir.mkdir(parents=True, exist_ok=True)
        system = os.environ.get("QOSMOE_TRACE_SYSTEM", "qosmoe")
        rank = int(os.environ.get("QOSMOE_TRACE_RANK", "0"))
        path = out_dir / f"real_token_trace_{system}_rank{rank}.csv"
        exists = path.exists()
        with open(path, "a", newline="") as f:
            w = csv.DictWriter(f, fieldnames=TRACE_HEADER)
            if not exists:
                w.writeheader()
            w.writerows(self.rows)
        self.rows.clear()


TRACE = TokenTrace()
