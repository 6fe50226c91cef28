"""The fused expert-parallel kernels on one GPU:
  * the device harmony plan (one warp) equals the oracle's restatement of
    Scheduler.schedule_harmony bit for bit;
  * the whole fused path (counts -> plan -> dispatch -> grouped GEMM with the return epilogue ->
    combine) in loopback — the rank is its own only peer — equals the local path;
  * a device wait on a flag that nothing sets gives up after its limit, reports
    DSCA_ERR_WAIT_TIMEOUT through the error word, and leaves the context usable.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from dsca_moe_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _st():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_device_plan_matches_oracle(lib, cuda):
    from dsca_moe_b200.engine import default_expert_to_gpu

    g = np.random.default_rng(11)
    for trial in range(120):
        G = int(g.choice([1, 2, 3, 4, 8]))
        E = int(g.choice([8, 16, 60, 64]))
        eq = int(g.choice([-1, 0, 1, 150, 10 ** 6]))
        meta = g.integers(0, int(g.choice([2, 50, 500])), size=(G, E)).astype(np.int32)
        if trial % 2 == 0:
            meta[:, int(g.integers(0, E))] += g.integers(0, 4000, size=G).astype(np.int32)
        e2g = default_expert_to_gpu(E, G) if trial % 3 else g.integers(0, G, size=E).astype(np.int32)
        md = torch.from_numpy(meta).to(cuda)
        ed = torch.from_numpy(np.ascontiguousarray(e2g, np.int32)).to(cuda)
        Sd = torch.zeros(G * E * G, dtype=torch.int32, device=cuda)
        assert lib.dsca_ep_plan_eval(_p(md), G, E, _p(ed), eq, _p(Sd), _st()) == 0
        S = Sd.cpu().numpy().reshape(G, E, G)
        want = O.schedule_fixed(meta, e2g) if eq < 0 else O.harmony_schedule(meta, e2g, eq)
        assert np.array_equal(S, want), (G, E, eq)


def _qwen_pair(dev, T=384, d=512, E=60, I=128, Is=256):
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_swiglu

    Wg, _ = syn.router_weight(E, d, 51, zipf_s=1.5, dtype="bf16")
    g = torch.Generator(device=dev)
    g.manual_seed(52)

    def n(*s):
        return (torch.randn(*s, generator=g, device=dev) * 0.03).to(torch.bfloat16)

    pe = pack_swiglu(n(E, I, d), n(E, I, d), n(E, d, I), shared=(n(Is, d), n(Is, d), n(d, Is)), device=dev)
    sgw = n(d)
    Wt = torch.from_numpy(Wg).to(dev, torch.bfloat16)
    loop = MoEEngine(Wt, pe, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK, shared_gate_weight=sgw, exchange="p2p")
    loop.ep_loopback = True
    local = MoEEngine(Wt, pe, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK, shared_gate_weight=sgw)
    x = torch.from_numpy(syn.hidden_states(T, d, 53, "bf16")).to(dev, torch.bfloat16)
    return loop, local, x


@pytest.mark.parametrize("ret_mode", ["overlap", "fused"])
def test_p2p_loopback_equals_local_path(lib, cuda, ret_mode):
    loop, local, x = _qwen_pair(cuda)
    loop.ep_return = ret_mode
    try:
        for it in range(3):  # successive epochs reuse the region
            a = loop.forward(x)
            b = local.forward(x)
            torch.cuda.synchronize()
            loop.check()
            local.check()
            assert torch.equal(a["topk_ids"], b["topk_ids"])
            assert torch.equal(a["out"], b["out"]), f"iteration {it}"
        S, rows = loop.read_plan()
        assert rows == x.shape[0] * 4
        assert np.array_equal(S[0, :, 0], np.bincount(a["topk_ids"].cpu().numpy().reshape(-1), minlength=60))
        # QoS execution order: experts by the planner's priority (summed over the ranks: here one),
        # descending, lowest id on ties — a permutation, and the output above is unchanged by it
        order, prio = loop.read_qos_order()
        mine = loop._workspace(x.shape[0])["expert_priority"].cpu().numpy()
        assert np.array_equal(prio.view(np.uint32), mine.view(np.uint32))
        want = sorted(range(60), key=lambda e: (-float(mine[e]), e))
        assert order.tolist() == want
    finally:
        loop.close()


def test_qos_order_changes_no_result(lib, cuda):
    """The routed GEMM tiles in any execution order (here reversed) give the same output bit for
    bit: the QoS order only decides which experts run first."""
    loop, local, x = _qwen_pair(cuda)
    try:
        a = loop.forward(x)["out"].clone()
        ws = loop._workspace(x.shape[0])
        rev = torch.arange(59, -1, -1, dtype=torch.int32, device=cuda)
        b = local.forward(x)
        torch.cuda.synchronize()
        lws = local._workspace(x.shape[0])
        y_ref = lws["y"].clone()
        cap = lws["a"].shape[0]
        local._ffn_call(x, lws, lws["a"], lws["h"], lws["y"], cap, local.E, lws["offsets"], None, 3,
                        group_order=rev)
        torch.cuda.synchronize()
        local.check()
        assert torch.equal(lws["y"], y_ref)
        assert torch.equal(a, b["out"])
        del ws
    finally:
        loop.close()


def test_p2p_loopback_switch_top1(lib, cuda):
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_relu

    T, d, E, F = 300, 256, 64, 512
    Wr, _ = syn.router_weight(E, d, 61, zipf_s=1.0, dtype="bf16")
    g = torch.Generator(device=cuda)
    g.manual_seed(62)
    wi = (torch.randn(E, F, d, generator=g, device=cuda) * 0.03).to(torch.bfloat16)
    wo = (torch.randn(E, d, F, generator=g, device=cuda) * 0.03).to(torch.bfloat16)
    pe = pack_relu(wi, wo, device=cuda)
    Wt = torch.from_numpy(Wr).to(cuda, torch.bfloat16)
    loop = MoEEngine(Wt, pe, top_k=1, route_mode=L.ROUTE_SWITCH_TOP1)
    loop.ep_loopback = True
    local = MoEEngine(Wt, pe, top_k=1, route_mode=L.ROUTE_SWITCH_TOP1)
    x = torch.from_numpy(syn.hidden_states(T, d, 63, "bf16")).to(cuda, torch.bfloat16)
    try:
        a = loop.forward(x)
        b = local.forward(x)
        torch.cuda.synchronize()
        loop.check()
        assert torch.equal(a["expert_index"], b["expert_index"])
        assert torch.equal(a["out"], b["out"])
    finally:
        loop.close()


def test_wait_timeout_reports_and_context_survives(lib, cuda):
    from dsca_moe_b200 import _lib as L

    region = ctypes.c_void_p()
    assert lib.dsca_ep_region_alloc(ctypes.c_size_t(1 << 20), ctypes.byref(region)) == 0
    try:
        s = L.EpSetup()
        s.G, s.E, s.me, s.d, s.elem_bytes = 1, 8, 0, 64, 2
        s.recv_capacity, s.ret_capacity, s.eq_tokens = 16, 16, 0
        s.start_epoch = 7  # waits for flags >= 7; nothing ever sets them
        e2g = np.zeros(8, np.int32)
        s.expert_to_gpu = e2g.ctypes.data
        s.flags[0] = region.value
        s.meta[0] = region.value + 256
        s.recv[0] = region.value + 8192
        s.ret[0] = region.value + 65536
        ctx = torch.empty(int(lib.dsca_ep_ctx_bytes()), dtype=torch.uint8, device=cuda)
        assert lib.dsca_ep_init(_p(ctx), ctypes.byref(s), _st()) == 0
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        assert lib.dsca_ep_wait(_p(ctx), 1, ctypes.c_uint64(20_000_000), _p(err), _st()) == 0
        assert lib.dsca_check_error(_p(err), _st()) == L.ERR_WAIT_TIMEOUT
        # the error word was cleared and the context still runs kernels
        assert lib.dsca_check_error(_p(err), _st()) == L.OK
        xs = torch.linspace(-5, 0, 1000, device=cuda)
        ys = torch.empty_like(xs)
        assert lib.dsca_exp_neg_eval(_p(xs), _p(ys), 1000, _st()) == 0
        torch.cuda.synchronize()
        assert torch.allclose(ys, torch.exp(xs), rtol=1e-6)
    finally:
        torch.cuda.synchronize()
        lib.dsca_ep_region_free(region)


def test_p2p_loopback_fp8_weights(lib, cuda):
    """fp8-e4m3 expert weights through the fused exchange in loopback: the dispatch writes the
    rows as f16 (and the f16 copy of x for the shared expert), the rows go back by the return
    kernel; the output equals the one-GPU fp8 path bit for bit."""
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, quantize_fp8

    loop, local, x = _qwen_pair(cuda, d=512, I=256, Is=512)
    pe8 = quantize_fp8(local.experts)
    loop8 = MoEEngine(local.router_weight, pe8, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK,
                      shared_gate_weight=local.shared_gate_weight, exchange="p2p")
    loop8.ep_loopback = True
    local8 = MoEEngine(local.router_weight, pe8, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK,
                       shared_gate_weight=local.shared_gate_weight)
    try:
        for mode in ("overlap", "fused"):  # "fused" falls back to the return kernel for fp8
            loop8.ep_return = mode
            a = loop8.forward(x)
            b = local8.forward(x)
            torch.cuda.synchronize()
            loop8.check()
            local8.check()
            assert torch.equal(a["out"], b["out"]), mode
    finally:
        loop8.close()
        loop.close()
