"""C-ABI library: loads, exports every symbol include/dsca_b200.h declares, and its host-side
planner (no GPU needed) matches the oracle and the reference's plans."""
import ctypes
import os
import re

import numpy as np

from golden_io import json_fixture
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "dsca_b200.h")).read()
    return sorted(set(re.findall(r"\b(dsca_[a-z0-9_]+)\s*\(", src)))


def test_header_symbols_exported(lib):
    from dsca_moe_b200 import _lib

    declared = _declared_symbols()
    assert set(declared) == set(_lib.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name
    assert b"sm_100a" in lib.dsca_version()
    assert lib.dsca_status_string(3) == b"device wait timed out"


# C struct name -> ctypes mirror in dsca_moe_b200._lib
_STRUCTS = {"dsca_router_args": "RouterArgs", "dsca_scan_args": "ScanArgs", "dsca_permute_args": "PermuteArgs",
            "dsca_ffn_args": "FfnArgs", "dsca_combine_args": "CombineArgs", "dsca_qos_args": "QosArgs",
            "dsca_ep_setup": "EpSetup", "dsca_ep_dispatch_args": "EpDispatchArgs", "dsca_split_args": "SplitArgs"}


def test_struct_layouts_match_c_compiler(tmp_path):
    """Every ctypes mirror has the size and field offsets that the C compiler gives the header's
    declarations: a small C program prints sizeof / offsetof of every field of every argument
    struct, compiled with gcc against include/dsca_b200.h."""
    import json
    import shutil
    import subprocess

    import pytest

    from dsca_moe_b200 import _lib

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "dsca_b200.h"', "int main(void) {",
             '  printf("{");']
    first = True
    for cname, pyname in _STRUCTS.items():
        cls = getattr(_lib, pyname)
        sep = "" if first else ","
        first = False
        lines.append(f'  printf("{sep}\\"{cname}\\": {{\\"size\\": %zu", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'  printf(", \\"{fname}\\": %zu", offsetof({cname}, {fname}));')
        lines.append('  printf("}");')
    lines += ['  printf("}\\n");', "  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src), "-o",
                    str(exe)], check=True)
    got = json.loads(subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout)
    for cname, pyname in _STRUCTS.items():
        cls = getattr(_lib, pyname)
        assert got[cname]["size"] == ctypes.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert got[cname][fname] == getattr(cls, fname).offset, (cname, fname)


def _header_struct_members():
    """{struct name: [member names in declaration order]} parsed from include/dsca_b200.h."""
    src = open(os.path.join(ROOT, "include", "dsca_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", " ", src, flags=re.S)
    out = {}
    for body, name in re.findall(r"typedef struct \{(.*?)\}\s*(dsca_[a-z0-9_]+)\s*;", src, flags=re.S):
        members = []
        for stmt in body.split(";"):
            stmt = " ".join(stmt.split())
            if not stmt:
                continue
            # "type a, b[8], *c" -> a, b, c (the first word(s) are the type)
            decl = re.sub(r"^(const\s+)?(unsigned\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**", "", stmt)
            for part in decl.split(","):
                m = re.match(r"\s*\**\s*([A-Za-z_][A-Za-z0-9_]*)", part)
                members.append(m.group(1))
        out[name] = members
    return out


def test_every_argument_struct_is_mirrored():
    """The header declares no argument struct without a ctypes mirror, and every mirror lists the
    C members in the C order (their offsets are checked above)."""
    from dsca_moe_b200 import _lib

    members = _header_struct_members()
    assert set(members) == set(_STRUCTS), set(members) ^ set(_STRUCTS)
    for cname, pyname in _STRUCTS.items():
        assert [f for f, _ in getattr(_lib, pyname)._fields_] == members[cname], cname


def test_qos_bad_args_rejected_without_gpu(lib):
    from dsca_moe_b200 import _lib

    assert lib.dsca_qos_priority(None, None) == _lib.ERR_BAD_ARG
    q = _lib.QosArgs()
    q.x = q.logits = q.topk_ids = q.token_score = q.expert_priority = 4096
    q.T, q.d, q.E, q.top_k, q.dtype = 16, 64, 8, 2, _lib.BF16
    q.attention_mode = 2
    assert lib.dsca_qos_priority(ctypes.byref(q), None) == _lib.ERR_BAD_ARG
    q.attention_mode, q.top_k = 0, 9
    assert lib.dsca_qos_priority(ctypes.byref(q), None) == _lib.ERR_BAD_ARG
    q.top_k, q.E = 2, 257
    assert lib.dsca_qos_priority(ctypes.byref(q), None) == _lib.ERR_CAPACITY


def test_bad_args_rejected_without_gpu(lib):
    from dsca_moe_b200 import _lib

    assert lib.dsca_router_topk(None, None) == _lib.ERR_BAD_ARG
    a = _lib.RouterArgs()
    assert lib.dsca_router_topk(ctypes.byref(a), None) == _lib.ERR_BAD_ARG
    # the fused scan needs all four of counts / offsets / block_base / done_counter (checked
    # before any device call; the pointers are never dereferenced)
    a.x = a.w_router = a.logits = a.topk_ids = a.topk_w = a.block_hist = a.local_rank = 4096
    a.T, a.d, a.E, a.top_k, a.dtype, a.mode = 32, 64, 8, 2, _lib.BF16, _lib.ROUTE_SOFTMAX_TOPK
    a.counts = a.offsets = 4096
    assert lib.dsca_router_topk(ctypes.byref(a), None) == _lib.ERR_BAD_ARG
    a.T = 0  # a valid empty call with all four set returns OK without launching
    a.block_base = a.done_counter = 4096
    assert lib.dsca_router_topk(ctypes.byref(a), None) == _lib.OK
    # tensor-core logits (checked before any device call): w_slices and w_exp together, bf16
    # only, and above d = 2048 the three scratch buffers as well
    a.T = 32
    a.w_slices = 4096
    assert lib.dsca_router_topk(ctypes.byref(a), None) == _lib.ERR_BAD_ARG
    a.w_exp = 4096
    a.d = 2304
    a.x_slices = a.x_exp = 4096
    assert lib.dsca_router_topk(ctypes.byref(a), None) == _lib.ERR_BAD_ARG
    a.d = 64
    a.logits_f32 = 4096
    a.dtype = _lib.F32
    assert lib.dsca_router_topk(ctypes.byref(a), None) == _lib.ERR_BAD_ARG
    assert lib.dsca_router_pack_i8(None, 8, 64, None, None, None) == _lib.ERR_BAD_ARG
    assert lib.dsca_router_pack_i8(ctypes.c_void_p(4096), 65, 64, ctypes.c_void_p(4096), ctypes.c_void_p(4096),
                                   None) == _lib.ERR_BAD_ARG  # more than 64 router rows
    assert lib.dsca_router_pack_i8(ctypes.c_void_p(4096), 8, 60, ctypes.c_void_p(4096), ctypes.c_void_p(4096),
                                   None) == _lib.ERR_BAD_ARG  # width not a multiple of 8
    assert lib.dsca_grouped_ffn(None, None) == _lib.ERR_BAD_ARG
    assert lib.dsca_plan_harmony(None, 2, 8, None, 150, None) == _lib.ERR_BAD_ARG


def test_plan_harmony_matches_reference_plans(lib):
    from dsca_moe_b200.engine import plan_harmony

    for c in json_fixture("harmony_plans.json")["cases"]:
        meta = np.array(c["meta"], np.int32)
        S = plan_harmony(meta, c["expert_to_gpu"], c["eq_tokens"])
        assert np.array_equal(S, np.array(c["harmony"])), (c["E"], c["G"], c["counts"])
        F = plan_harmony(meta, c["expert_to_gpu"], -1)
        assert np.array_equal(F, np.array(c["fixed"]))


def test_plan_harmony_random_vs_oracle(lib):
    from dsca_moe_b200.engine import default_expert_to_gpu, plan_harmony

    g = np.random.default_rng(5)
    for trial in range(300):
        G = int(g.choice([2, 3, 4, 8]))
        E = int(g.choice([6, 8, 16, 60, 64]))
        eq = int(g.choice([0, 1, 50, 150, 10**6]))
        meta = g.integers(0, int(g.choice([1, 5, 300])), size=(G, E)).astype(np.int32)
        if trial % 3 == 0:
            meta[:, 0] += g.integers(0, 3000, size=G).astype(np.int32)
        e2g = default_expert_to_gpu(E, G)
        assert np.array_equal(plan_harmony(meta, e2g, eq), O.harmony_schedule(meta, e2g, eq))


def test_plan_layout_matches_reference_order(lib):
    """Sender rows (dst, expert, token) and receiver groups (expert, src) as in
    distribute_tokens / generate_expert_mask."""
    from dsca_moe_b200.engine import plan_layout

    for c in json_fixture("dispatch_order.json"):
        S = np.array(c["schedule"], np.int32)
        G, E = c["G"], c["E"]
        for r in range(G):
            lay = plan_layout(S, r)
            assert lay.send_splits.tolist() == c["ranks"][r]["send_splits"]
            assert lay.recv_splits.tolist() == c["ranks"][r]["recv_splits"]
            # sender: row of the q-th token of expert e is send_base[e, dst] + q - cum_before
            lists = O.expert_token_lists(np.array(c["expert_ids"][r]), E)
            send_rows = np.full(int(S[r].sum()), -1)
            for e in range(E):
                for q, tok in enumerate(lists[e]):
                    dst = int(np.searchsorted(lay.cum_split[e], q, side="right"))
                    before = lay.cum_split[e, dst - 1] if dst > 0 else 0
                    send_rows[lay.send_base[e, dst] + q - before] = tok
            assert send_rows.tolist() == c["ranks"][r]["send_tokens"]
            # receiver: expert-major groups; group g rows = recv positions of expert_mask[e]
            recv = O.recv_expert_lists(S, r)
            src_start = np.concatenate([[0], np.cumsum(lay.recv_splits)])
            for gi, e in enumerate(lay.group_expert):
                rows = []
                for src in range(G):
                    n = int(S[src, e, r])
                    if n:
                        # position in the reference's src-major receive buffer of chunk (src, e)
                        pos0 = src_start[src] + int(S[src, :e, r].sum())
                        rows.extend(range(pos0, pos0 + n))
                        assert lay.recv_off[src, e] == lay.group_offsets[gi] + len(rows) - n
                assert rows == recv[e].tolist()
                assert lay.group_offsets[gi + 1] - lay.group_offsets[gi] == len(rows)
