"""fp8-e4m3 expert weights with per-output-channel fp32 scales: the block (f16 operands, fp32
accumulation, scales in the epilogue) against the fp32 oracle run on the dequantised weights
(q * scale) and the same inputs — 2e-2 max relative error.  Routing is unchanged by the weight
format and stays bit-exact.  Four kernel forms run: "split" (the e4m3 weights unconverted on
kind::f8f6f4 MMAs against two-term e4m3 tokens, the default: GEMM1 single-CTA tiles, GEMM2
CTA-pair tiles), "split-pair" (both GEMMs on CTA pairs), "smem" (weights converted to f16 in
shared memory) and "tmem" (converted into tensor memory, the MMA's A operand read from TMEM).
dsca_split_rows is bit-exact against the oracle's restatement."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from dsca_moe_b200 import synthetic as syn

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _qwen(dev, T, d, E, I, Is, seed):
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, dequantize_fp8, pack_swiglu, quantize_fp8, unpack_swiglu

    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def n(*s):
        return (torch.randn(*s, generator=g, device=dev) * 0.03).to(torch.bfloat16)

    pe = pack_swiglu(n(E, I, d), n(E, I, d), n(E, d, I), shared=(n(Is, d), n(Is, d), n(d, Is)), device=dev)
    q = quantize_fp8(pe)
    Wg, _ = syn.router_weight(E, d, seed + 1, zipf_s=1.5, dtype="bf16")
    sgw = syn.bf16_round(syn.rng(seed + 2).standard_normal((1, d)).astype(np.float32) / np.sqrt(d))
    eng = MoEEngine(torch.from_numpy(Wg).to(dev, torch.bfloat16), q, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK,
                    shared_gate_weight=torch.from_numpy(sgw).to(dev, torch.bfloat16))
    gate, up, down, shared = unpack_swiglu(dequantize_fp8(q))
    p = {"gate": gate.cpu().numpy(), "up": up.cpu().numpy(), "down": down.cpu().numpy(),
         "s_gate": shared[0].cpu().numpy(), "s_up": shared[1].cpu().numpy(), "s_down": shared[2].cpu().numpy(),
         "s_gate_w": sgw}
    return eng, Wg, p


FORMS = ["split", "split-pair", "smem", "tmem"]


def _form(eng, form):
    """split: GEMM1 on single-CTA tiles, GEMM2 on CTA pairs; split-pair: both GEMMs on CTA pairs."""
    eng.fp8_split = form.startswith("split")
    eng.tile_rows = 256 if form in ("tmem", "split-pair") else 0


@pytest.mark.parametrize("tile_rows", FORMS)
@pytest.mark.parametrize("T,d,E,I,Is", [(200, 256, 60, 128, 256), (77, 128, 8, 64, 128), (1, 64, 8, 32, 64),
                                        (300, 192, 8, 320, 384)])
def test_qwen_fp8_vs_oracle(cuda, T, d, E, I, Is, tile_rows):
    eng, Wg, p = _qwen(cuda, T, d, E, I, Is, 41)
    _form(eng, tile_rows)
    x = syn.hidden_states(T, d, 42, "bf16")
    r = eng.forward(torch.from_numpy(x).to(cuda, torch.bfloat16))
    torch.cuda.synchronize()
    eng.check()
    y, lg, ids, w, sg = O.qwen_forward(x, Wg, p, 4, False, "bf16")
    assert np.array_equal(r["topk_ids"].cpu().numpy(), ids)
    assert O.max_rel_err(r["out"].float().cpu().numpy(), y) < TOL


@pytest.mark.parametrize("tile_rows", FORMS)
def test_switch_fp8_vs_oracle(cuda, tile_rows):
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, dequantize_fp8, pack_relu, quantize_fp8

    T, d, E, F = 300, 256, 16, 512
    g = torch.Generator(device=cuda)
    g.manual_seed(51)
    wi = (torch.randn(E, F, d, generator=g, device=cuda) * 0.03).to(torch.bfloat16)
    wo = (torch.randn(E, d, F, generator=g, device=cuda) * 0.03).to(torch.bfloat16)
    q = quantize_fp8(pack_relu(wi, wo, device=cuda))
    Wr, _ = syn.router_weight(E, d, 52, zipf_s=1.0, dtype="bf16")
    eng = MoEEngine(torch.from_numpy(Wr).to(cuda, torch.bfloat16), q, top_k=1, route_mode=L.ROUTE_SWITCH_TOP1)
    _form(eng, tile_rows)
    x = syn.hidden_states(T, d, 53, "bf16")
    r = eng.forward(torch.from_numpy(x).to(cuda, torch.bfloat16))
    torch.cuda.synchronize()
    eng.check()
    dq = dequantize_fp8(q)
    wi_d = dq.w1[:, :F].cpu().numpy()
    wo_d = dq.w2[:, :d, :F].cpu().numpy()
    y, lg, idx, gate = O.switch_forward(x, Wr, wi_d, wo_d, "bf16")
    assert np.array_equal(r["expert_index"].cpu().numpy(), idx)
    assert O.max_rel_err(r["out"].float().cpu().numpy(), y) < TOL


@pytest.mark.parametrize("tile_rows", FORMS)
def test_qwen_fp8_full_size(cuda, tile_rows):
    """Qwen1.5-MoE-A2.7B shape, 4096 tokens: fp8 output vs the oracle on a token sample."""
    T, d, E, I, Is = 4096, 2048, 60, 1408, 5632
    eng, Wg, p = _qwen(cuda, T, d, E, I, Is, 61)
    _form(eng, tile_rows)
    x = syn.hidden_states(T, d, 62, "bf16")
    r = eng.forward(torch.from_numpy(x).to(cuda, torch.bfloat16))
    torch.cuda.synchronize()
    eng.check()
    sample = syn.rng(63).choice(T, 48, replace=False)
    y, *_ = O.qwen_forward(x[sample], Wg, p, 4, False, "bf16")
    assert O.max_rel_err(r["out"].float().cpu().numpy()[sample], y) < TOL


def test_fp8_forms_agree(cuda):
    """The two kernel forms on the same fp8 block: both accumulate exact f16 products in fp32, so
    they differ only by summation order and the f16 rounding of the intermediate (1e-2)."""
    T, d, E, I, Is = 1000, 512, 60, 384, 768
    eng, Wg, p = _qwen(cuda, T, d, E, I, Is, 71)
    x = torch.from_numpy(syn.hidden_states(T, d, 72, "bf16")).to(cuda, torch.bfloat16)
    outs = []
    for form in FORMS:
        _form(eng, form)
        outs.append(eng.forward(x)["out"].float().clone())
        torch.cuda.synchronize()
        eng.check()
    a = outs[0]
    for b in outs[1:]:
        assert torch.isfinite(b).all()
        assert ((a - b).abs().max() / a.abs().max()).item() < 1e-2


@pytest.mark.parametrize("rows,K,ld,bound", [(300, 2048, 2048, None), (77, 200, 208, None), (1000, 1408, 1408, 613),
                                             (5, 8, 8, None)])
def test_split_rows_bit_exact(cuda, lib, rows, K, ld, bound):
    """dsca_split_rows through the C-ABI against the oracle's restatement: the hi / lo bytes and
    1 / s bit for bit, rows of mixed magnitudes (zero, subnormal-scale, large) included; a
    device row count bounds the rows written."""
    import ctypes

    from dsca_moe_b200 import _lib as L

    g = np.random.default_rng(rows + K)
    x = g.standard_normal((rows, ld)).astype(np.float32) * np.exp2(g.integers(-30, 30, (rows, 1))).astype(np.float32)
    x[0] = 0.0
    if rows > 2:
        x[1, : K // 2] *= np.float32(2.0 ** -40)
        x[2] *= np.float32(2.0 ** 60)
    x = syn.bf16_round(x)
    kp = (K + 127) // 128 * 128
    src = torch.from_numpy(x).to(cuda, torch.bfloat16)
    dst = torch.full((rows, 2 * kp), 0xAB, dtype=torch.uint8, device=cuda)
    inv = torch.full((rows,), -1.0, dtype=torch.float32, device=cuda)
    nrow = torch.tensor([bound if bound is not None else rows], dtype=torch.int32, device=cuda)
    a = L.SplitArgs()
    a.src, a.ld, a.rows, a.K = src.data_ptr(), ld, rows, K
    a.rows_dev = nrow.data_ptr() if bound is not None else None
    a.dst, a.inv_scale = dst.data_ptr(), inv.data_ptr()
    L.check(lib.dsca_split_rows(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
            "dsca_split_rows")
    torch.cuda.synchronize()
    q, iv = O.split_e4m3(x[:, :K])
    n = bound if bound is not None else rows
    assert np.array_equal(dst.cpu().numpy()[:n], q[:n])
    assert np.array_equal(inv.cpu().numpy()[:n].view(np.uint32), iv[:n].view(np.uint32))
    if n < rows:  # rows past the device count untouched
        assert (dst[n:] == 0xAB).all() and (inv[n:] == -1.0).all()
