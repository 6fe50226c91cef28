"""The two-term e4m3 token form of the fp8-weight path (oracle restatement of dsca_split_rows):
the e4m3 encoder against torch's float8_e4m3fn conversion, and the exactness of hi + lo."""
import numpy as np
import torch

from oracle import oracle as O


def test_e4m3_encoder_matches_torch():
    g = np.random.default_rng(3)
    v = np.concatenate([g.standard_normal(20000).astype(np.float32) * s for s in (1e-3, 0.05, 1.0, 30.0)])
    # ties and the subnormal range
    v = np.concatenate([v, np.arange(-64, 65, dtype=np.float32) * np.float32(2.0 ** -10),
                        np.array([0.0, -0.0, 448.0, -448.0, 2.0 ** -6, 2.0 ** -9, 3 * 2.0 ** -10], np.float32)])
    ours = O.e4m3_rn(v)
    ref = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, ref)
    back = torch.from_numpy(ours).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(O.e4m3_value(ours), back)


def test_split_reconstructs_bf16_rows():
    g = np.random.default_rng(5)
    x = g.standard_normal((64, 200)).astype(np.float32) * np.exp2(g.integers(-20, 20, (64, 1))).astype(np.float32)
    x = O.bf16_round(x)
    x[3] = 0.0
    q, inv = O.split_e4m3(x)
    kp = 256
    assert q.shape == (64, 2 * kp)
    assert not q[:, 200:kp].any() and not q[:, kp + 200:].any()
    rec = (O.e4m3_value(q[:, :200]).astype(np.float64) + O.e4m3_value(q[:, kp:kp + 200])) * inv[:, None]
    s_max = np.abs(x).max(axis=1, keepdims=True) / inv[:, None]
    assert np.all((s_max < 256) | (s_max == 0))
    big = np.abs(x) / inv[:, None] >= 0.25
    assert np.array_equal(rec[big], x[big].astype(np.float64))
    # the rest is below 2^-9 of the row's largest: absolute error under 2^-10 in scaled units
    assert np.all(np.abs(rec - x) * (1 / inv[:, None]) <= 2.0 ** -10 + 1e-30)
