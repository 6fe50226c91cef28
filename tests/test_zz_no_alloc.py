"""dsca_grouped_ffn_static_scratch — the grouped expert FFN for callers that cannot allocate
device memory (code running inside a graph replay or a callback, or under a foreign allocator
with no room left).  It keeps the GEMM1 intermediate in a fixed array inside the library, so
the caller passes only inputs and outputs.

Checked here through the C ABI: its outputs match the allocating entry point
(dsca_grouped_ffn, same inputs) within the tolerance of the other tests (2e-2 bf16, 1e-4 f32),
on two calls in a row, for a SwiGLU block with a shared expert and for a ReLU block in bf16 and
in f32.  Before the checked calls, one call on unrelated inputs leaves different data in the
array, so a result that depended on what the array held before would show.  Sizes past the
array's limit, fp8 weights and caller-owned intermediates are refused before any work is
launched.  This file is collected last so that a run stopping at its first failure has already
run every other test.
"""
import ctypes

import pytest
import torch

from dsca_moe_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
F32_TOL = 1e-4


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _routed(eng, x):
    """Route and permute with the existing entry points; returns the expert-major rows."""
    r = eng.forward(x)
    ws = eng._workspace(x.shape[0])
    return ws["a"], ws["offsets"], r


def _ffn_args(eng, x, a, offsets, y, ys, h=None, hs=None):
    from dsca_moe_b200 import _lib as L

    pe = eng.experts
    f = L.FfnArgs()
    f.dtype = L.BF16 if eng.dtype == torch.bfloat16 else L.F32
    f.act, f.d = pe.act, eng.d
    f.n1p, f.ip, f.dp = pe.n1p, pe.ip, pe.dp
    f.num_groups, f.group_offsets, f.group_weight = eng.E, _p(offsets), None
    f.num_experts_w, f.capacity = pe.E, a.shape[0]
    f.a, f.w1, f.w2, f.h, f.y = _p(a), _p(pe.w1), _p(pe.w2), _p(h), _p(y)
    if pe.ws1 is not None:
        f.shared_rows, f.shared_n1p, f.shared_ip = x.shape[0], pe.s_n1p, pe.s_ip
        f.xs, f.ws1, f.ws2, f.hs, f.ys = _p(x), _p(pe.ws1), _p(pe.ws2), _p(hs), _p(ys)
    f.err, f.num_ctas, f.phases = _p(eng.err), 0, 0
    return f


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _engine(kind, dev, dtype=torch.bfloat16):
    from dsca_moe_b200 import _lib as L
    from dsca_moe_b200.engine import MoEEngine, pack_relu, pack_swiglu

    g = torch.Generator(device=dev)
    g.manual_seed(11)
    name = "bf16" if dtype == torch.bfloat16 else "f32"

    def n(*shape):
        return (torch.randn(*shape, generator=g, device=dev) * 0.02).to(dtype)

    if kind == "swiglu":
        T, d, E, I, Is = 256, 2048, 60, 1408, 5632
        Wr, _ = syn.router_weight(E, d, 12, zipf_s=1.5, dtype=name)
        pe = pack_swiglu(n(E, I, d), n(E, I, d), n(E, d, I), shared=(n(Is, d), n(Is, d), n(d, Is)), dtype=dtype,
                         device=dev)
        eng = MoEEngine(torch.from_numpy(Wr).to(dev, dtype), pe, top_k=4, route_mode=L.ROUTE_SOFTMAX_TOPK,
                        shared_gate_weight=n(d))
    else:
        T, d, E, F = 512, 768, 64, 3072
        Wr, _ = syn.router_weight(E, d, 13, zipf_s=1.0, dtype=name)
        pe = pack_relu(n(E, F, d), n(E, d, F), dtype=dtype, device=dev)
        eng = MoEEngine(torch.from_numpy(Wr).to(dev, dtype), pe, top_k=1, route_mode=L.ROUTE_SWITCH_TOP1)
    x = torch.from_numpy(syn.hidden_states(T, d, 14, name)).to(dev, dtype)
    return eng, x


@pytest.mark.parametrize("kind,dtype", [("swiglu", torch.bfloat16), ("relu", torch.bfloat16),
                                        ("swiglu", torch.float32), ("relu", torch.float32)])
def test_static_scratch_matches_allocating_entry_point(lib, cuda, kind, dtype):
    eng, x = _engine(kind, cuda, dtype)
    tol = BF16_TOL if dtype == torch.bfloat16 else F32_TOL
    a, offsets, _ = _routed(eng, x)
    R, T, d = a.shape[0], x.shape[0], eng.d
    pe = eng.experts
    shared = pe.ws1 is not None
    # reference: the allocating entry point with caller-owned intermediates
    h = torch.empty(R, pe.ip, dtype=dtype, device=cuda)
    hs = torch.empty(T, pe.s_ip, dtype=dtype, device=cuda) if shared else None
    y_ref = torch.empty(R, d, dtype=dtype, device=cuda)
    ys_ref = torch.empty(T, d, dtype=dtype, device=cuda) if shared else None
    f = _ffn_args(eng, x, a, offsets, y_ref, ys_ref, h=h, hs=hs)
    assert lib.dsca_grouped_ffn(ctypes.byref(f), _stream()) == 0
    # one call on unrelated rows first: the array then holds data that has nothing to do with
    # the checked calls, which must not depend on it
    a_other = torch.randn(R, d, device=cuda).mul_(3.0).to(dtype)
    x_other = torch.randn(T, d, device=cuda).mul_(3.0).to(dtype)
    y_other = torch.empty(R, d, dtype=dtype, device=cuda)
    ys_other = torch.empty(T, d, dtype=dtype, device=cuda) if shared else None
    g = _ffn_args(eng, x_other, a_other, offsets, y_other, ys_other)
    assert lib.dsca_grouped_ffn_static_scratch(ctypes.byref(g), _stream()) == 0
    # the variant, twice in a row on fresh output buffers
    for _ in range(2):
        y = torch.full((R, d), float("nan"), dtype=dtype, device=cuda)
        ys = torch.full((T, d), float("nan"), dtype=dtype, device=cuda) if shared else None
        g = _ffn_args(eng, x, a, offsets, y, ys)
        assert lib.dsca_grouped_ffn_static_scratch(ctypes.byref(g), _stream()) == 0
        torch.cuda.synchronize()
        assert lib.dsca_check_error(_p(eng.err), _stream()) == 0
        assert torch.isfinite(y.float()).all()
        assert _rel(y, y_ref) < tol
        if shared:
            assert torch.isfinite(ys.float()).all()
            assert _rel(ys, ys_ref) < tol


def test_static_scratch_refuses_oversized_and_owned_buffers(lib, cuda):
    from dsca_moe_b200 import _lib as L

    eng, x = _engine("relu", cuda)
    a, offsets, _ = _routed(eng, x)
    y = torch.empty(a.shape[0], eng.d, dtype=torch.bfloat16, device=cuda)
    g = _ffn_args(eng, x, a, offsets, y, None)
    # more rows than the 16 MiB array holds: refused before any launch
    g.capacity = L.STATIC_SCRATCH_BYTES // (eng.experts.ip * 2) + 1
    assert lib.dsca_grouped_ffn_static_scratch(ctypes.byref(g), _stream()) == L.ERR_CAPACITY
    # a caller-owned intermediate is not accepted (the scratch is internal)
    g = _ffn_args(eng, x, a, offsets, y, None, h=y)
    assert lib.dsca_grouped_ffn_static_scratch(ctypes.byref(g), _stream()) == L.ERR_BAD_ARG
    # fp8 weights go through dsca_grouped_ffn only
    g = _ffn_args(eng, x, a, offsets, y, None)
    g.dtype = L.F8E4M3
    assert lib.dsca_grouped_ffn_static_scratch(ctypes.byref(g), _stream()) == L.ERR_UNSUPPORTED
    torch.cuda.synchronize()
