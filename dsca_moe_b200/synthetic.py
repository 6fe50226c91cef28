"""Seeded synthetic inputs for the MoE-block forward.

The reference measures on WikiText/SST-2 token batches through whole Switch / Qwen models
(``README.md:41-48``); here the block is fed seeded N(0,1) hidden states with the same
batch x sequence shapes, and random-init expert weights of the named architectures.

Router skew.  The reference's own skew generator (``src/harmonymoe/router.py:65-142``)
prescribes per-expert counts directly and sets every probability to 1, which does not
exercise a softmax router.  Here the router stays a bias-free ``Linear`` (so it still fits the
plugin's ``router_tensor_path`` weight) and each row ``e`` of a base matrix ``W0 ~ N(0, 1/d)``
is scaled by ``alpha_e``; ``alpha`` is calibrated by multiplicative updates until the top-1
histogram on a seeded calibration batch follows Zipf(s): ``p_e ∝ (e+1)^-s`` (expert 0 hottest).

Everything here is numpy with ``PCG64`` streams, so the same seed gives the same bits on any
x86-64 host; large expert tensors for the throughput run are drawn on the device instead
(see ``device_normal``).
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "rng", "bf16_round", "hidden_states", "zipf_targets", "calibrate_zipf_alpha",
    "router_weight", "switch_expert_weights", "qwen_expert_weights", "exflow_uneven_placement",
]


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returns float32 holding them."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    nan = np.isnan(a)
    out = r.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.nan
    return out


def hidden_states(T: int, d: int, seed: int, dtype: str = "f32") -> np.ndarray:
    x = rng(seed).standard_normal((T, d), dtype=np.float32)
    return bf16_round(x) if dtype == "bf16" else x


def zipf_targets(E: int, s: float) -> np.ndarray:
    w = (np.arange(1, E + 1, dtype=np.float64)) ** (-float(s))
    return w / w.sum()


def calibrate_zipf_alpha(base_logits: np.ndarray, s: float, iters: int = 2000,
                         tol: float = 0.01, step: float = 0.2) -> tuple[np.ndarray, np.ndarray]:
    """Scale factors ``alpha[E]`` so that argmax(base_logits * alpha) follows Zipf(s).

    ``base_logits`` is the [T_cal, E] matrix X·W0ᵀ of the calibration batch.  The update works on
    log(alpha): ``la += step * (log target - log achieved)`` (achieved floored at 1/(2T)),
    re-centred to mean 0 and clipped to [-6, 6]; it stops when every
    |achieved - target| <= tol * max(target).  Returns (alpha, achieved_histogram).
    """
    T, E = base_logits.shape
    target = zipf_targets(E, s)
    la = np.zeros(E, dtype=np.float64)
    bl = base_logits.astype(np.float64)
    ach = None
    for _ in range(iters):
        top = np.argmax(bl * np.exp(la)[None, :], axis=1)
        ach = np.bincount(top, minlength=E).astype(np.float64) / T
        if np.max(np.abs(ach - target)) <= tol * target.max():
            break
        la += step * (np.log(target) - np.log(np.maximum(ach, 0.5 / T)))
        la -= la.mean()
        la = np.clip(la, -6.0, 6.0)
    return np.exp(la).astype(np.float32), ach


def router_weight(E: int, d: int, seed: int, zipf_s: float | None = None,
                  calib_tokens: int = 8192, dtype: str = "f32") -> tuple[np.ndarray, dict]:
    """Router weight [E, d].  ``zipf_s=None`` gives the unscaled N(0, 1/d) router (near uniform)."""
    g = rng(seed)
    w0 = (g.standard_normal((E, d), dtype=np.float32) / np.float32(np.sqrt(d))).astype(np.float32)
    info: dict = {"zipf_s": zipf_s}
    if zipf_s is not None:
        xc = rng(seed + 7919).standard_normal((calib_tokens, d), dtype=np.float32)
        alpha, ach = calibrate_zipf_alpha(xc.astype(np.float64) @ w0.T.astype(np.float64), zipf_s)
        w0 = (w0 * alpha[:, None]).astype(np.float32)
        info["alpha"] = alpha.tolist()
        info["calib_top1_hist"] = ach.tolist()
    if dtype == "bf16":
        w0 = bf16_round(w0)
    return w0, info


def switch_expert_weights(E: int, d: int, F: int, seed: int, std: float = 0.02,
                          dtype: str = "f32") -> tuple[np.ndarray, np.ndarray]:
    """Switch ``DenseActDense`` experts: wi [E, F, d], wo [E, d, F] (nn.Linear layout)."""
    g = rng(seed)
    wi = (g.standard_normal((E, F, d), dtype=np.float32) * np.float32(std)).astype(np.float32)
    wo = (g.standard_normal((E, d, F), dtype=np.float32) * np.float32(std)).astype(np.float32)
    if dtype == "bf16":
        wi, wo = bf16_round(wi), bf16_round(wo)
    return wi, wo


def qwen_expert_weights(E: int, d: int, I: int, Is: int, seed: int, std: float = 0.02,
                        dtype: str = "f32") -> dict:
    """Qwen2-MoE experts in nn.Linear layout plus the shared expert and its gate."""
    g = rng(seed)

    def n(*shape):
        a = (g.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
        return bf16_round(a) if dtype == "bf16" else a

    p = {
        "gate": n(E, I, d), "up": n(E, I, d), "down": n(E, d, I),
        "s_gate": n(Is, d), "s_up": n(Is, d), "s_down": n(d, Is),
    }
    sg = (g.standard_normal((1, d), dtype=np.float32) / np.float32(np.sqrt(d))).astype(np.float32)
    p["s_gate_w"] = bf16_round(sg) if dtype == "bf16" else sg
    return p


def exflow_uneven_placement(E: int, G: int, num_layers: int = 1) -> list:
    """The exflow placement format ``[layer][gpu] -> [expert ids]`` with contiguous blocks,
    the first ``E % G`` GPUs holding one expert more (60 on 8 -> 4 x 8 + 4 x 7)."""
    base, extra = divmod(E, G)
    layer, e = [], 0
    for gpu in range(G):
        n = base + (1 if gpu < extra else 0)
        layer.append(list(range(e, e + n)))
        e += n
    return [layer for _ in range(num_layers)]
