"""GPU parity: the CUDA path (through the C-ABI) against the oracle and the golden fixtures.

Bars: routing (logits, expert ids, per-expert counts, permutation) bit-exact against the oracle,
which follows the kernels' fixed arithmetic order; outputs within 1e-4 (fp32) / 2e-2 (bf16)
max|d| / max|ref| of the fp32 oracle; against the reference's own fixtures, routing exact except
on near-ties and boundary ties (see tests/test_oracle_golden.py).
"""
import ctypes

import numpy as np
import pytest
import torch

import torch_ref
from golden_io import assert_logits_close, load, qwen_weights, routing_near_ties, switch_weights
from oracle import oracle as O
from dsca_moe_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
F32_TOL = 1e-4


def _t(a, dtype, dev):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device=dev, dtype=dtype)


def _np(t):
    return t.detach().float().cpu().numpy()


def switch_engine(Wr, wi, wo, dtype, dev):
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_relu

    pe = pack_relu(_t(wi, dtype, dev), _t(wo, dtype, dev), dtype=dtype, device=dev)
    return MoEEngine(_t(Wr, dtype, dev), pe, top_k=1, route_mode=L.ROUTE_SWITCH_TOP1)


def qwen_engine(Wg, p, top_k, norm, dtype, dev):
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_swiglu

    pe = pack_swiglu(_t(p["gate"], dtype, dev), _t(p["up"], dtype, dev), _t(p["down"], dtype, dev),
                     shared=(_t(p["s_gate"], dtype, dev), _t(p["s_up"], dtype, dev), _t(p["s_down"], dtype, dev)),
                     dtype=dtype, device=dev)
    return MoEEngine(_t(Wg, dtype, dev), pe, top_k=top_k, route_mode=L.ROUTE_SOFTMAX_TOPK, norm_topk=norm,
                     shared_gate_weight=_t(p["s_gate_w"], dtype, dev))


def test_device_is_b200(lib, cuda):
    n, ok = ctypes.c_int(0), ctypes.c_int(0)
    assert lib.dsca_device_info(ctypes.byref(n), ctypes.byref(ok)) == 0
    assert ok.value == 1 and n.value >= 100


def test_exp_neg_bit_exact_vs_oracle(lib, cuda):
    x = np.concatenate([np.linspace(-88.0, 0.0, 1 << 20, dtype=np.float32),
                        -np.logspace(-10, 1.95, 1 << 16).astype(np.float32),
                        np.array([0.0, -0.0, -87.0, -86.99999, 1.0], np.float32)])
    xd = torch.from_numpy(x).to(cuda)
    yd = torch.empty_like(xd)
    assert lib.dsca_exp_neg_eval(ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(yd.data_ptr()), x.size,
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    got = yd.cpu().numpy()
    ref = O.exp_neg(x)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    # accuracy against CUDA's expf on the same device: within 2 ulp
    tex = torch.exp(xd).cpu().numpy()
    m = (x > -87.0) & (x <= 0.0)  # the routing exp is defined on x <= 0 (larger x clamps to 0)
    ulp = np.abs(got[m].view(np.int32).astype(np.int64) - tex[m].view(np.int32).astype(np.int64))
    assert ulp.max() <= 2


@pytest.mark.parametrize("dtype,T,d,E", [("bf16", 1000, 768, 64), ("f32", 1000, 768, 64),
                                         ("bf16", 33, 256, 8), ("bf16", 1, 64, 3)])
def test_router_switch_bit_exact(cuda, dtype, T, d, E):
    x = syn.hidden_states(T, d, 101, dtype)
    Wr, _ = syn.router_weight(E, d, 102, zipf_s=1.0 if E > 8 else None, dtype=dtype)
    wi, wo = syn.switch_expert_weights(E, d, 256, 103, dtype=dtype)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    eng = switch_engine(Wr, wi, wo, tdt, cuda)
    r = eng.forward(_t(x, tdt, cuda))
    torch.cuda.synchronize()
    eng.check()
    lg = O.router_logits_for(x, Wr, dtype, eng.router_tensor_cores)
    idx, gate = O.route_top1(lg, dtype)
    assert np.array_equal(_np(r["logits"]).view(np.uint32), lg.view(np.uint32))
    assert np.array_equal(r["expert_index"].cpu().numpy(), idx)
    assert np.array_equal(r["topk_ids"].cpu().numpy()[:, 0], idx)
    assert np.array_equal(r["topk_w"].cpu().numpy()[:, 0].view(np.uint32), gate.view(np.uint32))
    assert np.array_equal(r["counts"].cpu().numpy(), np.bincount(idx, minlength=E))


@pytest.mark.parametrize("T,d,E,k,norm", [(515, 2048, 60, 4, False), (64, 128, 8, 4, True),
                                          (100, 256, 16, 2, False), (7, 64, 63, 8, False)])
def test_router_topk_bit_exact(cuda, T, d, E, k, norm):
    x = syn.hidden_states(T, d, 201, "bf16")
    Wg, _ = syn.router_weight(E, d, 202, zipf_s=1.5 if E > 8 else None, dtype="bf16")
    p = syn.qwen_expert_weights(E, d, 64, 128, 203, dtype="bf16")
    eng = qwen_engine(Wg, p, k, norm, torch.bfloat16, cuda)
    r = eng.forward(_t(x, torch.bfloat16, cuda))
    torch.cuda.synchronize()
    eng.check()
    lg = O.router_logits_for(x, Wg, "bf16", eng.router_tensor_cores)
    ids, w = O.route_topk(lg, k, norm, "bf16")
    assert np.array_equal(_np(r["logits"]).view(np.uint32), lg.view(np.uint32))
    assert np.array_equal(r["topk_ids"].cpu().numpy(), ids)
    assert np.array_equal(r["topk_w"].cpu().numpy().view(np.uint32), w.view(np.uint32))
    # shared-expert gate: sigmoid of the bf16-rounded gate logit
    z = O.router_logits_for(x, p["s_gate_w"], "bf16", eng.router_tensor_cores)[:, 0].astype(np.float64)
    sg = 1.0 / (1.0 + np.exp(-z))
    assert np.abs(r["shared_gate"].cpu().numpy() - sg).max() < 1e-6


@pytest.mark.parametrize("T,k,E", [(4096, 4, 60), (1000, 1, 64), (31, 4, 60), (1, 1, 8)])
def test_permutation_bit_exact(cuda, T, k, E):
    """Rows expert-major, tokens ascending inside each expert; the row contents equal x."""
    d = 128
    x = syn.hidden_states(T, d, 301, "bf16")
    Wg, _ = syn.router_weight(E, d, 302, zipf_s=1.5, dtype="bf16")
    if k == 1:
        wi, wo = syn.switch_expert_weights(E, d, 256, 303, dtype="bf16")
        eng = switch_engine(Wg, wi, wo, torch.bfloat16, cuda)
    else:
        eng = qwen_engine(Wg, syn.qwen_expert_weights(E, d, 64, 128, 303, dtype="bf16"), k, False,
                          torch.bfloat16, cuda)
    xd = _t(x, torch.bfloat16, cuda)
    r = eng.forward(xd)
    torch.cuda.synchronize()
    eng.check()
    ids = r["topk_ids"].cpu().numpy()
    rows, slots, offs = O.permutation_world1(ids, E)
    assert np.array_equal(r["offsets"].cpu().numpy(), offs)
    tr = r["token_row"].cpu().numpy()
    assert np.array_equal(np.sort(tr.reshape(-1)), np.arange(T * k))
    want = np.empty(T * k, np.int64)
    want[np.arange(T * k)] = 0
    got_tok = np.empty(T * k, np.int64)
    got_slot = np.empty(T * k, np.int64)
    t_idx, j_idx = np.meshgrid(np.arange(T), np.arange(k), indexing="ij")
    got_tok[tr.reshape(-1)] = t_idx.reshape(-1)
    got_slot[tr.reshape(-1)] = j_idx.reshape(-1)
    assert np.array_equal(got_tok, rows) and np.array_equal(got_slot, slots)
    a = eng._workspace(T)["a"][: T * k]
    assert torch.equal(a, xd[torch.from_numpy(rows).to(cuda)])


@pytest.mark.parametrize("T,d,E,I,Is,k", [(77, 128, 60, 64, 256, 4), (256, 256, 8, 128, 384, 2),
                                          (300, 64, 16, 32, 64, 4), (1, 128, 8, 64, 128, 4)])
def test_qwen_block_bf16_vs_oracle(cuda, T, d, E, I, Is, k):
    x = syn.hidden_states(T, d, 401, "bf16")
    Wg, _ = syn.router_weight(E, d, 402, zipf_s=1.5, dtype="bf16")
    p = syn.qwen_expert_weights(E, d, I, Is, 403, dtype="bf16")
    eng = qwen_engine(Wg, p, k, False, torch.bfloat16, cuda)
    r = eng.forward(_t(x, torch.bfloat16, cuda))
    torch.cuda.synchronize()
    eng.check()
    y, *_ = O.qwen_forward(x, Wg, p, k, False, "bf16")
    assert O.max_rel_err(_np(r["out"]), y) < BF16_TOL


@pytest.mark.parametrize("T,d,E,F", [(200, 128, 8, 256), (129, 256, 16, 512), (1000, 768, 64, 3072)])
def test_switch_block_bf16_vs_oracle(cuda, T, d, E, F):
    x = syn.hidden_states(T, d, 501, "bf16")
    Wr, _ = syn.router_weight(E, d, 502, zipf_s=1.0, dtype="bf16")
    wi, wo = syn.switch_expert_weights(E, d, F, 503, dtype="bf16")
    eng = switch_engine(Wr, wi, wo, torch.bfloat16, cuda)
    r = eng.forward(_t(x, torch.bfloat16, cuda))
    torch.cuda.synchronize()
    eng.check()
    y, *_ = O.switch_forward(x, Wr, wi, wo, "bf16")
    assert O.max_rel_err(_np(r["out"]), y) < BF16_TOL


@pytest.mark.parametrize("T,d,E,F", [(96, 64, 8, 128), (300, 128, 16, 256)])
def test_switch_block_f32_parity_mode(cuda, T, d, E, F):
    x = syn.hidden_states(T, d, 601, "f32")
    Wr, _ = syn.router_weight(E, d, 602, zipf_s=1.0, dtype="f32")
    wi, wo = syn.switch_expert_weights(E, d, F, 603, dtype="f32")
    eng = switch_engine(Wr, wi, wo, torch.float32, cuda)
    r = eng.forward(_t(x, torch.float32, cuda))
    torch.cuda.synchronize()
    eng.check()
    y, lg, idx, g = O.switch_forward(x, Wr, wi, wo, "f32")
    assert np.array_equal(r["expert_index"].cpu().numpy(), idx)
    assert O.max_rel_err(_np(r["out"]), y) < F32_TOL


def test_qwen_block_f32_parity_mode(cuda):
    T, d, E, I, Is = 64, 128, 16, 64, 128
    x = syn.hidden_states(T, d, 701, "f32")
    Wg, _ = syn.router_weight(E, d, 702, zipf_s=1.5, dtype="f32")
    p = syn.qwen_expert_weights(E, d, I, Is, 703, dtype="f32")
    eng = qwen_engine(Wg, p, 4, False, torch.float32, cuda)
    r = eng.forward(_t(x, torch.float32, cuda))
    torch.cuda.synchronize()
    eng.check()
    y, *_ = O.qwen_forward(x, Wg, p, 4, False, "f32")
    assert O.max_rel_err(_np(r["out"]), y) < F32_TOL


# ------------------------------------------------------------------ reference fixtures
@pytest.mark.parametrize("name", ["switch_f32_small.npz", "switch_bf16_small.npz", "switch_f32_ties.npz",
                                  "switch_f32_mid.npz"])
def test_switch_golden_through_plugin_layer(cuda, name):
    """The drop-in QoSMoELayer on the reference's own fixture."""
    from dsca_moe_b200 import QoSMoEConfig, QoSMoELayer, RequestStateTable

    z, m = load(name)
    wi, wo = switch_weights(z, m)
    tdt = torch.bfloat16 if m["dtype"] == "bf16" else torch.float32
    sds = [{"wi.weight": torch.from_numpy(wi[e]).to(tdt), "wo.weight": torch.from_numpy(wo[e]).to(tdt)}
           for e in range(m["E"])]
    cfg = QoSMoEConfig(rank=0, world_size=1, experts=sds, router_weights=torch.from_numpy(z["Wr"]).to(tdt),
                       d_model=m["d"], num_experts=m["E"], expert_cache_size=m["E"])
    layer = QoSMoELayer(cfg)
    with pytest.raises(RuntimeError):
        layer(_t(z["x"], tdt, cuda).view(m["B"], m["S"], m["d"]))
    layer.set_runtime_context(RequestStateTable(cfg).build_context(
        {"attention_mask": torch.ones(m["B"], m["S"], dtype=torch.long)}))
    y, (logits, idx) = layer(_t(z["x"], tdt, cuda).view(m["B"], m["S"], m["d"]))
    torch.cuda.synchronize()
    assert y.shape == (m["B"], m["S"], m["d"]) and idx.dtype == torch.int64
    lg = _np(logits)
    assert_logits_close(lg, z["logits"], m["dtype"])
    near = routing_near_ties(lg, 1, m["dtype"])
    got = idx.cpu().numpy()
    assert np.array_equal(got[~near], z["expert_index"][~near])
    # exact against the oracle on every token
    tc = layer.engine.router_tensor_cores
    assert np.array_equal(got, O.route_top1(O.router_logits_for(z["x"], z["Wr"], m["dtype"], tc), m["dtype"])[0])
    tol = F32_TOL if m["dtype"] == "f32" else BF16_TOL
    same = got == z["expert_index"]
    assert O.max_rel_err(_np(y).reshape(-1, m["d"])[same], z["y"][same]) < tol


@pytest.mark.parametrize("name", ["qwen_tiny_f32.npz", "qwen_tiny_bf16.npz", "qwen_small_bf16.npz",
                                  "qwen_small_f32_w4.npz", "qwen_norm_f32.npz", "qwen_ties_bf16.npz"])
def test_qwen_golden(cuda, name):
    z, m = load(name)
    p = qwen_weights(z, m)
    tdt = torch.bfloat16 if m["dtype"] == "bf16" else torch.float32
    eng = qwen_engine(z["Wg"], p, m["top_k"], m["norm_topk_prob"], tdt, cuda)
    tol = F32_TOL if m["dtype"] == "f32" else BF16_TOL
    for r in range(m["world"]):
        res = eng.forward(_t(z["x"][r], tdt, cuda))
        torch.cuda.synchronize()
        eng.check()
        lg = _np(res["logits"])
        assert_logits_close(lg, z["logits"][r], m["dtype"])
        assert np.array_equal(lg.view(np.uint32), O.router_logits_for(z["x"][r], z["Wg"], m["dtype"],
                                                                       eng.router_tensor_cores).view(np.uint32))
        pr = O.softmax(lg)
        s = -np.sort(-pr, axis=1)
        keep = (s[:, m["top_k"] - 1] != s[:, m["top_k"]]) & ~routing_near_ties(lg, m["top_k"], m["dtype"])
        assert O.max_rel_err(_np(res["out"])[keep], z["y"][r][keep]) < tol


def test_switch_routing_golden_production_shape(cuda):
    z, m = load("switch_routing_c2_bf16.npz")
    x = syn.hidden_states(m["T"], m["d"], m["seed"], "bf16")
    wi, wo = syn.switch_expert_weights(m["E"], m["d"], 256, 9, dtype="bf16")
    eng = switch_engine(z["Wr"], wi, wo, torch.bfloat16, cuda)
    r = eng.forward(_t(x, torch.bfloat16, cuda))
    torch.cuda.synchronize()
    lg = _np(r["logits"])
    near = O.near_tie_tokens(lg, 1, "bf16")
    bad = r["expert_index"].cpu().numpy() != z["expert_index"]
    assert not (bad & ~near).any()


# ------------------------------------------------------------------ full size
def _device_qwen_weights(E, d, I, Is, seed, dev):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def n(*shape):
        return (torch.randn(*shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)

    return {"gate": n(E, I, d), "up": n(E, I, d), "down": n(E, d, I), "s_gate": n(Is, d), "s_up": n(Is, d),
            "s_down": n(d, Is)}


def test_qwen_full_size_bf16(cuda):
    """Qwen1.5-MoE-A2.7B block, 4096 tokens: routing bit-exact on every token, permutation a
    bijection, output within 2e-2 of the fp32 oracle on a token sample and of the fp32 torch
    restatement on every token."""
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_swiglu

    T, d, E, I, Is, k = 4096, 2048, 60, 1408, 5632, 4
    x = syn.hidden_states(T, d, 801, "bf16")
    Wg, info = syn.router_weight(E, d, 802, zipf_s=1.5, dtype="bf16")
    sgw = syn.bf16_round(syn.rng(804).standard_normal((1, d)).astype(np.float32) / np.sqrt(d))
    w = _device_qwen_weights(E, d, I, Is, 803, cuda)
    pe = pack_swiglu(w["gate"], w["up"], w["down"], shared=(w["s_gate"], w["s_up"], w["s_down"]),
                     dtype=torch.bfloat16, device=cuda)
    eng = MoEEngine(_t(Wg, torch.bfloat16, cuda), pe, top_k=k, route_mode=L.ROUTE_SOFTMAX_TOPK,
                    shared_gate_weight=_t(sgw, torch.bfloat16, cuda))
    r = eng.forward(_t(x, torch.bfloat16, cuda))
    torch.cuda.synchronize()
    eng.check()
    lg = O.router_logits_for(x, Wg, "bf16", eng.router_tensor_cores)
    ids, wts = O.route_topk(lg, k, False, "bf16")
    assert np.array_equal(_np(r["logits"]).view(np.uint32), lg.view(np.uint32))
    assert np.array_equal(r["topk_ids"].cpu().numpy(), ids)
    assert np.array_equal(r["counts"].cpu().numpy(), np.bincount(ids.reshape(-1), minlength=E))
    tr = r["token_row"].cpu().numpy().reshape(-1)
    assert np.array_equal(np.sort(tr), np.arange(T * k))
    # output on a token sample against the fp32 oracle (weights copied back for those experts)
    sample = syn.rng(805).choice(T, 48, replace=False)
    p = {key: v.float().cpu().numpy() for key, v in w.items() if key.startswith("s_")}
    used = np.unique(ids[sample])
    p["gate"] = np.zeros((E, I, d), np.float32)
    p["up"] = np.zeros((E, I, d), np.float32)
    p["down"] = np.zeros((E, d, I), np.float32)
    for e in used:
        p["gate"][e] = w["gate"][e].float().cpu().numpy()
        p["up"][e] = w["up"][e].float().cpu().numpy()
        p["down"][e] = w["down"][e].float().cpu().numpy()
    p["s_gate_w"] = sgw
    y, *_ = O.qwen_forward(x[sample], Wg, p, k, False, "bf16")
    assert O.max_rel_err(_np(r["out"])[sample], y) < BF16_TOL
    # every token against the fp32 torch restatement (routing from the kernel, checked above)
    ref = torch_ref.qwen_block_fp32(_t(x, torch.bfloat16, cuda), r["topk_ids"], r["topk_w"], w,
                                    _t(sgw, torch.bfloat16, cuda))
    assert torch_ref.max_rel_err(r["out"], ref) < BF16_TOL
    # per-row diagnostic: no token's output norm is off by more than 2 %
    rn = (r["out"].float() - ref).norm(dim=1) / ref.norm(dim=1).clamp_min(1e-30)
    assert float(rn.max()) < BF16_TOL
    # Zipf s=1.5: the hottest expert takes about 42 % of the top-1 choices
    assert 0.35 < np.mean(ids[:, 0] == 0) < 0.5


def test_switch_full_size_bf16(cuda):
    T, d, E, F = 4096, 768, 64, 3072
    x = syn.hidden_states(T, d, 901, "bf16")
    Wr, _ = syn.router_weight(E, d, 902, zipf_s=1.0, dtype="bf16")
    g = torch.Generator(device=cuda)
    g.manual_seed(903)
    wi = (torch.randn(E, F, d, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    wo = (torch.randn(E, d, F, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_relu

    eng = MoEEngine(_t(Wr, torch.bfloat16, cuda), pack_relu(wi, wo, device=cuda), top_k=1,
                    route_mode=L.ROUTE_SWITCH_TOP1)
    r = eng.forward(_t(x, torch.bfloat16, cuda))
    torch.cuda.synchronize()
    eng.check()
    lg = O.router_logits_for(x, Wr, "bf16", eng.router_tensor_cores)
    idx, gate = O.route_top1(lg, "bf16")
    assert np.array_equal(r["expert_index"].cpu().numpy(), idx)
    sample = syn.rng(904).choice(T, 64, replace=False)
    wi_h, wo_h = wi.float().cpu().numpy(), wo.float().cpu().numpy()
    y, *_ = O.switch_forward(x[sample], Wr, wi_h, wo_h, "bf16")
    assert O.max_rel_err(_np(r["out"])[sample], y) < BF16_TOL
    # every token against the fp32 torch restatement (routing from the kernel, checked above)
    ref = torch_ref.switch_block_fp32(_t(x, torch.bfloat16, cuda), r["expert_index"], r["topk_w"], wi, wo)
    assert torch_ref.max_rel_err(r["out"], ref) < BF16_TOL


def test_repeat_calls_are_deterministic(cuda):
    T, d, E, I, Is = 512, 256, 60, 128, 256
    x = _t(syn.hidden_states(T, d, 1001, "bf16"), torch.bfloat16, cuda)
    Wg, _ = syn.router_weight(E, d, 1002, zipf_s=1.5, dtype="bf16")
    eng = qwen_engine(Wg, syn.qwen_expert_weights(E, d, I, Is, 1003, dtype="bf16"), 4, False, torch.bfloat16, cuda)
    a = eng.forward(x)["out"].clone()
    b = eng.forward(x)["out"].clone()
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("T,k,E", [(4096, 4, 60), (33, 1, 8), (20000, 8, 63)])
def test_fused_scan_matches_separate_scan(cuda, T, k, E):
    """The router's last-CTA scan gives the same counts, offsets and block bases as the separate
    scan launch, and leaves its completion counter at zero (two fused calls in a row agree)."""
    d = 128
    x = _t(syn.hidden_states(T, d, 1101, "bf16"), torch.bfloat16, cuda)
    Wg, _ = syn.router_weight(E, d, 1102, zipf_s=1.2, dtype="bf16")
    eng = qwen_engine(Wg, syn.qwen_expert_weights(E, d, 64, 128, 1103, dtype="bf16"), k, False,
                      torch.bfloat16, cuda)
    keys = ("counts", "offsets", "block_base", "token_row", "out")
    ws = eng._workspace(T)
    got = []
    for fused in (True, True, False):
        eng.fuse_scan = fused
        r = eng.forward(x)
        torch.cuda.synchronize()
        eng.check()
        got.append({kk: (ws[kk] if kk in ws else r[kk]).clone() for kk in keys})
        assert int(eng._done_counter.item()) == 0
    for kk in keys:
        assert torch.equal(got[0][kk], got[2][kk]), kk
        assert torch.equal(got[1][kk], got[2][kk]), kk


@pytest.mark.parametrize("T,d,E,I,Is,k", [(600, 256, 60, 128, 512, 4), (257, 128, 8, 64, 256, 2),
                                           (1100, 512, 8, 384, 640, 2)])
def test_single_cta_and_pair_tiles_agree(cuda, T, d, E, I, Is, k):
    """The 128-row single-CTA tiles, the 256-row CTA-pair swap-AB tiles and the hybrid pair tiles
    (whole 256-token blocks non-swapped, the rest swap-AB) give the same block output (every form
    accumulates each output element over K in the same order, so bf16 results match), and all
    stay within the bf16 tolerance of the fp32 oracle."""
    x = syn.hidden_states(T, d, 1201, "bf16")
    Wg, _ = syn.router_weight(E, d, 1202, zipf_s=1.5, dtype="bf16")
    p = syn.qwen_expert_weights(E, d, I, Is, 1203, dtype="bf16")
    eng = qwen_engine(Wg, p, k, False, torch.bfloat16, cuda)
    xd = _t(x, torch.bfloat16, cuda)
    outs = []
    for rows in (128, 256, 512):
        eng.tile_rows = rows
        got = []
        # one segment after the other / routed and shared tiles interleaved, token- or
        # weight-block-major inside a group, with and without the L2 eviction policies and L2
        # prefetches: neither the order of the tiles nor the cache use changes a result
        for order, hints, ahead in ((0, 0, 0), (1, 0, 0), (0, 1, 0), (1, 1, 0), (2, 0, 0), (3, 0, 8),
                                    (6, 0, 12), (7, 1, 16)):
            eng.tile_order, eng.cache_hints, eng.l2_ahead = order, hints, ahead
            r = eng.forward(xd)
            torch.cuda.synchronize()
            eng.check()
            got.append(r["out"].clone())
        eng.tile_order, eng.cache_hints, eng.l2_ahead = 0, 0, 0
        for g in got[1:]:
            assert torch.equal(got[0], g)
        outs.append(got[0].float().cpu().numpy())
    y, *_ = O.qwen_forward(x, Wg, p, k, False, "bf16")
    for o in outs:
        assert O.max_rel_err(o, y) < BF16_TOL
    assert np.abs(outs[0] - outs[1]).max() <= 1e-2 * max(1.0, np.abs(outs[1]).max())
    assert np.abs(outs[0] - outs[2]).max() <= 1e-2 * max(1.0, np.abs(outs[2]).max())


def test_hybrid_pair_tiles_full_size(cuda):
    """Qwen1.5-MoE-A2.7B block, 4096 tokens (Zipf 1.5: the hot expert spans several whole
    256-token blocks), hybrid CTA-pair GEMM1 tiles: every token within 2e-2 of the fp32 torch
    restatement, and equal to the single-CTA tiles' output within bf16 rounding; the CTA-pair
    swap-AB tiles with gate and up halves per CTA (tile_rows 256) equal the single-CTA tiles'
    output exactly."""
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_swiglu

    T, d, E, I, Is, k = 4096, 2048, 60, 1408, 5632, 4
    x = syn.hidden_states(T, d, 811, "bf16")
    Wg, _ = syn.router_weight(E, d, 812, zipf_s=1.5, dtype="bf16")
    sgw = syn.bf16_round(syn.rng(814).standard_normal((1, d)).astype(np.float32) / np.sqrt(d))
    w = _device_qwen_weights(E, d, I, Is, 813, cuda)
    pe = pack_swiglu(w["gate"], w["up"], w["down"], shared=(w["s_gate"], w["s_up"], w["s_down"]),
                     dtype=torch.bfloat16, device=cuda)
    eng = MoEEngine(_t(Wg, torch.bfloat16, cuda), pe, top_k=k, route_mode=L.ROUTE_SOFTMAX_TOPK,
                    shared_gate_weight=_t(sgw, torch.bfloat16, cuda))
    xd = _t(x, torch.bfloat16, cuda)
    outs = {}
    for rows in (128, 256, 512, 512):
        eng.tile_rows = rows
        r = eng.forward(xd)
        torch.cuda.synchronize()
        eng.check()
        outs.setdefault(rows, []).append(r["out"].clone())
    assert torch.equal(outs[512][0], outs[512][1])
    assert torch.equal(outs[256][0], outs[128][0])
    ref = torch_ref.qwen_block_fp32(xd, r["topk_ids"], r["topk_w"], w, _t(sgw, torch.bfloat16, cuda))
    assert torch_ref.max_rel_err(outs[512][0], ref) < BF16_TOL
    assert torch_ref.max_rel_err(outs[512][0], outs[128][0]) < 1e-2
    assert int(r["counts"].max()) >= 512  # the hot expert has whole 256-token blocks


@pytest.mark.parametrize("T", [300, 4096])
def test_shared_handoff_changes_no_result(cuda, T):
    """Qwen1.5-MoE-A2.7B block shapes: GEMM2's shared-expert tiles starting on GEMM1's handoff
    flag (dsca_ffn_args.shared_handoff) instead of after all of GEMM1 give the same output bits
    as without the handoff and as the static tile schedule, over repeated forwards (every call
    leaves the ticket and handoff words zeroed)."""
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_swiglu

    d, E, I, Is, k = 2048, 60, 1408, 5632, 4
    x = syn.hidden_states(T, d, 821, "bf16")
    Wg, _ = syn.router_weight(E, d, 822, zipf_s=1.5, dtype="bf16")
    sgw = syn.bf16_round(syn.rng(824).standard_normal((1, d)).astype(np.float32) / np.sqrt(d))
    w = _device_qwen_weights(E, d, I, Is, 823, cuda)
    pe = pack_swiglu(w["gate"], w["up"], w["down"], shared=(w["s_gate"], w["s_up"], w["s_down"]),
                     dtype=torch.bfloat16, device=cuda)
    eng = MoEEngine(_t(Wg, torch.bfloat16, cuda), pe, top_k=k, route_mode=L.ROUTE_SOFTMAX_TOPK,
                    shared_gate_weight=_t(sgw, torch.bfloat16, cuda))
    xd = _t(x, torch.bfloat16, cuda)
    outs = []
    for handoff, dynamic in ((False, True), (True, True), (True, True), (True, True), (False, False)):
        eng.shared_handoff, eng.dynamic_tiles = handoff, dynamic
        r = eng.forward(xd)
        torch.cuda.synchronize()
        eng.check()
        outs.append(r["out"].clone())
    assert int(eng._tile_ctr.abs().sum()) == 0
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    ref = torch_ref.qwen_block_fp32(xd, r["topk_ids"], r["topk_w"], w, _t(sgw, torch.bfloat16, cuda))
    assert torch_ref.max_rel_err(outs[0], ref) < BF16_TOL


def test_host_pipeline_matches_forward(cuda):
    """HostPipeline (overlapped H2D / forward / D2H over pinned host batches) returns, for every
    batch, exactly what forward() returns for it."""
    from dsca_moe_b200.engine import HostPipeline
    T, d, E, I, Is, k = 300, 128, 16, 64, 128, 4
    Wg, _ = syn.router_weight(E, d, 1302, zipf_s=1.2, dtype="bf16")
    eng = qwen_engine(Wg, syn.qwen_expert_weights(E, d, I, Is, 1303, dtype="bf16"), k, False, torch.bfloat16, cuda)
    xs = [torch.from_numpy(syn.hidden_states(T, d, 1310 + i, "bf16")).to(torch.bfloat16).pin_memory() for i in range(5)]
    outs = [torch.empty(T, d, dtype=torch.bfloat16).pin_memory() for _ in range(5)]
    HostPipeline(eng, T).run(xs, outs)
    torch.cuda.synchronize()
    eng.check()
    for xh, oh in zip(xs, outs):
        ref = eng.forward(xh.to(cuda))["out"].cpu()
        assert torch.equal(oh, ref)


def test_host_pipeline_with_graphs_matches_forward(cuda):
    """HostPipeline replaying CUDA graphs of the forward (one per input buffer) returns, for every
    batch, exactly what forward() returns for it."""
    from dsca_moe_b200.engine import HostPipeline
    T, d, E, I, Is, k = 300, 128, 16, 64, 128, 4
    Wg, _ = syn.router_weight(E, d, 1352, zipf_s=1.2, dtype="bf16")
    eng = qwen_engine(Wg, syn.qwen_expert_weights(E, d, I, Is, 1353, dtype="bf16"), k, False, torch.bfloat16, cuda)
    xs = [torch.from_numpy(syn.hidden_states(T, d, 1360 + i, "bf16")).to(torch.bfloat16).pin_memory() for i in range(7)]
    outs = [torch.empty(T, d, dtype=torch.bfloat16).pin_memory() for _ in range(7)]
    HostPipeline(eng, T, graphs=True).run(xs, outs)
    torch.cuda.synchronize()
    eng.check()
    for xh, oh in zip(xs, outs):
        ref = eng.forward(xh.to(cuda))["out"].cpu()
        assert torch.equal(oh, ref)


@pytest.mark.parametrize("kind", ["qwen", "switch"])
def test_graph_replay_matches_eager(cuda, kind):
    """A forward captured as a CUDA graph (MoEEngine.capture) and replayed on new contents of its
    input buffer gives the eager forward's results bit for bit: routing, counts and output."""
    if kind == "qwen":
        T, d, E, I, Is, k = 1000, 2048, 60, 256, 512, 4
        Wg, _ = syn.router_weight(E, d, 1402, zipf_s=1.5, dtype="bf16")
        eng = qwen_engine(Wg, syn.qwen_expert_weights(E, d, I, Is, 1403, dtype="bf16"), k, False, torch.bfloat16,
                          cuda)
    else:
        T, d, E = 4096, 768, 64
        Wr, _ = syn.router_weight(E, d, 1412, zipf_s=1.0, dtype="bf16")
        wi, wo = syn.switch_expert_weights(E, d, 3072, 1413, dtype="bf16")
        eng = switch_engine(Wr, wi, wo, torch.bfloat16, cuda)
    xbuf = _t(syn.hidden_states(T, d, 1420, "bf16"), torch.bfloat16, cuda)
    graph = eng.capture(xbuf)
    for seed in (1421, 1422, 1421):
        xn = _t(syn.hidden_states(T, d, seed, "bf16"), torch.bfloat16, cuda)
        xbuf.copy_(xn)
        graph.replay()
        torch.cuda.synchronize()
        got = {key: graph.result[key].clone() for key in ("out", "topk_ids", "logits", "expert_index")}
        ref = eng.forward(xn)
        torch.cuda.synchronize()
        eng.check()
        for key, v in got.items():
            assert torch.equal(v, ref[key]), key


@pytest.mark.parametrize("T,d,E", [(131, 72, 64), (300, 2048, 60), (5, 64, 8), (1, 128, 64), (40, 2304, 16)])
def test_tensor_core_router_edge_values(cuda, T, d, E):
    """The optional tensor-core router (bf16 logits by exact fixed-point accumulation on int8
    tcgen05 MMAs) equals the oracle's fixed-point logits bit for bit on rows with zeros,
    subnormals, negated rows and exponent spreads past the 13-bit window, a width that is not a
    multiple of 16 and a token count that is not a multiple of 128."""
    g = np.random.default_rng(9 + T)
    x = g.standard_normal((T, d)) * np.exp2(g.integers(-24, 8, (T, d)))
    x[0] = 0.0
    if T > 3:
        x[1, : d // 2] = 0.0
        x[2] = 1e-40 * np.sign(x[2])  # bf16 subnormals
        x[3] = -np.abs(x[3])
    x = O.bf16_round(x.astype(np.float32))
    W = O.bf16_round((g.standard_normal((E, d)) * np.exp2(g.integers(-16, 2, (E, d)))).astype(np.float32))
    W[0] = 0.0
    wi, wo = syn.switch_expert_weights(E, d, 256, 5, dtype="bf16")
    eng = switch_engine(W, wi, wo, torch.bfloat16, cuda)
    eng.router_tensor_cores = True
    r = eng.forward(_t(x, torch.bfloat16, cuda))
    torch.cuda.synchronize()
    eng.check()
    lg = O.router_logits_fixed(x, W)
    assert np.array_equal(_np(r["logits"]).view(np.uint32), lg.view(np.uint32))
    assert np.array_equal(r["expert_index"].cpu().numpy(), O.route_top1(lg, "bf16")[0])


def test_tensor_core_router_qwen_block(cuda):
    """Tensor-core router on the Qwen block shape (60 experts + the shared gate row): logits,
    top-4 choices and weights and the shared gate follow the fixed-point oracle exactly, and the
    block output stays within the bf16 tolerance of the oracle."""
    T, d, E, k = 1000, 2048, 60, 4
    x = syn.hidden_states(T, d, 401, "bf16")
    Wg, _ = syn.router_weight(E, d, 402, zipf_s=1.5, dtype="bf16")
    p = syn.qwen_expert_weights(E, d, 64, 128, 403, dtype="bf16")
    eng = qwen_engine(Wg, p, k, False, torch.bfloat16, cuda)
    eng.router_tensor_cores = True
    r = eng.forward(_t(x, torch.bfloat16, cuda))
    torch.cuda.synchronize()
    eng.check()
    lg = O.router_logits_fixed(x, Wg)
    ids, w = O.route_topk(lg, k, False, "bf16")
    assert np.array_equal(_np(r["logits"]).view(np.uint32), lg.view(np.uint32))
    assert np.array_equal(r["topk_ids"].cpu().numpy(), ids)
    assert np.array_equal(r["topk_w"].cpu().numpy().view(np.uint32), w.view(np.uint32))
    z = O.router_logits_fixed(x, p["s_gate_w"])[:, 0].astype(np.float64)
    assert np.abs(r["shared_gate"].cpu().numpy() - 1.0 / (1.0 + np.exp(-z))).max() < 1e-6


@pytest.mark.parametrize("T,d,E,k", [(4096, 2048, 60, 4), (4100, 2048, 60, 4), (20000, 768, 63, 8),
                                     (70, 2304, 60, 4)])
def test_tensor_core_router_scan_and_exactness(cuda, T, d, E, k):
    """Tensor-core router (the fused one-kernel form for d <= 2048, the three-kernel form above
    it): logits and top-k choices equal the fixed-point oracle bit for bit, the fused last-CTA
    scan equals the separate scan launch and leaves its counter at zero, the permutation offsets
    follow the choices, and token counts that are not a multiple of the 128-token tile leave no
    stray histogram rows (the block output agrees across the three calls)."""
    x = syn.hidden_states(T, d, 1201, "bf16")
    Wg, _ = syn.router_weight(E, d, 1202, zipf_s=1.2, dtype="bf16")
    eng = qwen_engine(Wg, syn.qwen_expert_weights(E, d, 64, 128, 1203, dtype="bf16"), k, False,
                      torch.bfloat16, cuda)
    eng.router_tensor_cores = True
    keys = ("counts", "offsets", "block_base", "token_row", "out")
    ws = eng._workspace(T)
    xd = _t(x, torch.bfloat16, cuda)
    got = []
    for fused in (True, True, False):
        eng.fuse_scan = fused
        r = eng.forward(xd)
        torch.cuda.synchronize()
        eng.check()
        got.append({kk: (ws[kk] if kk in ws else r[kk]).clone() for kk in keys})
        assert int(eng._done_counter.item()) == 0
    for kk in keys:
        assert torch.equal(got[0][kk], got[2][kk]), kk
        assert torch.equal(got[1][kk], got[2][kk]), kk
    sample = np.arange(T) if T <= 4100 else syn.rng(1204).choice(T, 2000, replace=False)
    lg = O.router_logits_fixed(x[sample], Wg)
    ids, _ = O.route_topk(lg, k, False, "bf16")
    assert np.array_equal(_np(r["logits"])[sample].view(np.uint32), lg.view(np.uint32))
    assert np.array_equal(r["topk_ids"].cpu().numpy()[sample], ids)
    _, _, offs = O.permutation_world1(r["topk_ids"].cpu().numpy(), E)
    assert np.array_equal(got[0]["offsets"].cpu().numpy(), offs)


@pytest.mark.parametrize("T,d,E,I,Is", [(4096, 2048, 60, 1408, 5632), (300, 256, 16, 128, 384)])
def test_gemm1_overlapping_permute_is_bit_identical(cuda, T, d, E, I, Is):
    """GEMM1 launched as a programmatic dependent of the permute (shared-expert tiles first,
    routed tiles after griddepcontrol.wait) gives the serialized launch's output bit for bit."""
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_swiglu

    x = syn.hidden_states(T, d, 501, "bf16")
    Wg, _ = syn.router_weight(E, d, 502, zipf_s=1.5, dtype="bf16")
    sgw = syn.bf16_round(syn.rng(504).standard_normal((1, d)).astype(np.float32) / np.sqrt(d))
    w = _device_qwen_weights(E, d, I, Is, 503, cuda)
    pe = pack_swiglu(w["gate"], w["up"], w["down"], shared=(w["s_gate"], w["s_up"], w["s_down"]),
                     dtype=torch.bfloat16, device=cuda)
    eng = MoEEngine(_t(Wg, torch.bfloat16, cuda), pe, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK,
                    shared_gate_weight=_t(sgw, torch.bfloat16, cuda))
    xd = _t(x, torch.bfloat16, cuda)
    outs = []
    for pdl in (False, True, True):
        eng.pdl = pdl
        r = eng.forward(xd)
        torch.cuda.synchronize()
        eng.check()
        outs.append(r["out"].clone())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


def test_switch_block_programmatic_launches_are_bit_identical(cuda):
    """Switch layer (no shared expert: GEMM1 on CTA pairs, GEMM2 and the combine launched as
    programmatic dependents) gives the serialized launches' output bit for bit."""
    T, d, E, F = 4096, 768, 64, 3072
    x = syn.hidden_states(T, d, 601, "bf16")
    Wr, _ = syn.router_weight(E, d, 602, zipf_s=1.0, dtype="bf16")
    g = torch.Generator(device=cuda)
    g.manual_seed(603)
    wi = (torch.randn(E, F, d, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    wo = (torch.randn(E, d, F, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_relu

    eng = MoEEngine(_t(Wr, torch.bfloat16, cuda), pack_relu(wi, wo, device=cuda), top_k=1,
                    route_mode=L.ROUTE_SWITCH_TOP1)
    xd = _t(x, torch.bfloat16, cuda)
    outs = []
    for pdl in (False, True, True):
        eng.pdl = pdl
        r = eng.forward(xd)
        torch.cuda.synchronize()
        eng.check()
        outs.append(r["out"].clone())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
