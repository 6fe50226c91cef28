"""Expert weight packing (host side, CPU): the layouts the GEMM kernels read."""
import torch

from dsca_moe_b200.engine import pack_relu, pack_swiglu, unpack_swiglu


def test_swiglu_packing_blocks_and_round_trip():
    torch.manual_seed(0)
    E, I, d, Is = 3, 200, 64, 130
    gate, up, down = torch.randn(E, I, d), torch.randn(E, I, d), torch.randn(E, d, I)
    sh = (torch.randn(Is, d), torch.randn(Is, d), torch.randn(d, Is))
    pe = pack_swiglu(gate, up, down, shared=sh, dtype=torch.float32, device="cpu")
    # intermediate width rounded up to 128, so the gate+up rows are a multiple of 256
    assert pe.ip == 256 and pe.n1p == 512 and pe.n1p % 256 == 0 and pe.dp == 256
    assert pe.s_ip == 256 and pe.s_n1p == 512
    # 256-row blocks: 128 gate rows, then the 128 up rows of the same channels
    for blk in range(pe.n1p // 256):
        for half, src in ((0, gate), (1, up)):
            rows = pe.w1[:, blk * 256 + half * 128: blk * 256 + half * 128 + 128]
            ch0 = blk * 128
            n = max(0, min(128, I - ch0))
            assert torch.equal(rows[:, :n], src[:, ch0:ch0 + n])
            assert torch.count_nonzero(rows[:, n:]) == 0
    g2, u2, d2, (sg2, su2, sd2) = unpack_swiglu(pe)
    assert torch.equal(g2, gate) and torch.equal(u2, up) and torch.equal(d2, down)
    assert torch.equal(sg2, sh[0]) and torch.equal(su2, sh[1]) and torch.equal(sd2, sh[2])


def test_relu_packing_pads_to_256():
    wi, wo = torch.randn(2, 300, 64), torch.randn(2, 64, 300)
    pe = pack_relu(wi, wo, dtype=torch.float32, device="cpu")
    assert pe.n1p == 512 and pe.ip == 512 and pe.dp == 256
    assert torch.equal(pe.w1[:, :300], wi) and torch.count_nonzero(pe.w1[:, 300:]) == 0
    assert torch.equal(pe.w2[:, :64, :300], wo)
