"""ORACLE — test infrastructure only.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and its
``--impl reference`` arm) may import this module, and only as the checker / the CPU baseline.
The product path (``dsca_moe_b200``) never imports it and has no CPU fallback.

CPU restatement of the DSCA-MoE MoE-block forward hot path:

* routing   — C (``routing.c``) in the CUDA kernel's fixed arithmetic order, bit-exact;
* FFN math  — numpy in float64 on the same (bf16-representable) inputs and weights: the
              "fp32 reference" the tolerances are quoted against;
* plan      — ``harmony_schedule`` restates ``Scheduler.schedule_harmony``
              (src/harmonymoe/scheduler.py:324-372) over any expert->GPU placement, and
              ``schedule_fixed`` (:268-279);
* layout    — ``send_order`` restates ``Scheduler.distribute_tokens`` (:101-124) and
              ``recv_expert_lists`` restates ``generate_expert_mask`` (:185-213) with a stable
              order inside each expert.

Parity is pinned against fixtures generated from the reference's own code
(``tests/golden/make_golden.py``) by ``tests/test_oracle_golden.py``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def build() -> str:
    """Compile routing.c into oracle/_build (make); returns the library path."""
    path = os.path.join(_HERE, "_build", "liboracle_routing.so")
    src = os.path.join(_HERE, "routing.c")
    if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return path


def lib():
    global _LIB
    if _LIB is None:
        _LIB = ctypes.CDLL(build())
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        c_int = ctypes.c_int
        _LIB.oracle_exp_neg.argtypes = [ctypes.c_float]
        _LIB.oracle_exp_neg.restype = ctypes.c_float
        _LIB.oracle_round_bf16.argtypes = [ctypes.c_float]
        _LIB.oracle_round_bf16.restype = ctypes.c_float
        _LIB.oracle_router_logits.argtypes = [f32p, f32p, c_int, c_int, c_int, c_int, f32p]
        _LIB.oracle_router_logits_fixed.argtypes = [f32p, f32p, c_int, c_int, c_int, f32p]
        _LIB.oracle_scale_pow2.argtypes = [ctypes.c_float, c_int]
        _LIB.oracle_scale_pow2.restype = ctypes.c_float
        _LIB.oracle_route_top1.argtypes = [f32p, c_int, c_int, c_int, i32p, f32p]
        _LIB.oracle_route_topk.argtypes = [f32p, c_int, c_int, c_int, c_int, c_int, i32p, f32p]
        _LIB.oracle_softmax.argtypes = [f32p, c_int, c_int, f32p]
        _LIB.oracle_exp_neg_array.argtypes = [f32p, f32p, ctypes.c_long]
    return _LIB


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def bf16_round(a: np.ndarray) -> np.ndarray:
    a = _f32(a)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).copy()


# ------------------------------------------------------------------------------ routing
def exp_neg(x) -> np.ndarray:
    """The routing exp (routing.c: oracle_exp_neg) over an array."""
    x = _f32(x)
    y = np.empty_like(x)
    lib().oracle_exp_neg_array(x, y, x.size)
    return y


def router_logits(x, W, tau: str) -> np.ndarray:
    """logits[T,E] in tau ('bf16' or 'f32') by the chunked fp32 fma order of the CUDA-core
    router (routing.c: oracle_router_logits)."""
    x, W = _f32(x), _f32(W)
    T, d = x.shape
    E = W.shape[0]
    out = np.empty((T, E), np.float32)
    lib().oracle_router_logits(x, W, T, d, E, 1 if tau == "bf16" else 0, out)
    return out


def router_logits_fixed(x, W) -> np.ndarray:
    """bf16 logits[T,E] of the tensor-core router: exact fixed-point accumulation of the bf16
    inputs, one rounding to fp32, then to bf16 (routing.c: oracle_router_logits_fixed)."""
    x, W = bf16_round(x), bf16_round(W)
    T, d = x.shape
    out = np.empty((T, W.shape[0]), np.float32)
    lib().oracle_router_logits_fixed(x, W, T, d, W.shape[0], out)
    return out


def tensor_core_router_default(tau: str, d: int, rows: int) -> bool:
    """The engine's default router form: the tensor-core router for bf16 with d <= 2048 and at most
    64 router rows (experts plus the shared-expert gate), the CUDA-core router otherwise."""
    return tau == "bf16" and d <= 2048 and rows <= 64


def router_logits_for(x, W, tau: str, tensor_cores: bool | None = None, rows: int | None = None) -> np.ndarray:
    """The logits of the router form an engine ran: ``router_logits_fixed`` (exact fixed-point
    products, the tensor-core router) for bf16 with ``tensor_cores``, else ``router_logits`` (the
    CUDA-core router's fixed fp32 chunk order).  ``tensor_cores=None``: the engine's default for
    `rows` router rows (default: W's rows)."""
    if tensor_cores is None:
        tensor_cores = tensor_core_router_default(tau, np.shape(x)[1], np.shape(W)[0] if rows is None else rows)
    if tensor_cores and tau == "bf16":
        return router_logits_fixed(x, W)
    return router_logits(x, W, tau)


def softmax(logits) -> np.ndarray:
    lg = _f32(logits)
    out = np.empty_like(lg)
    lib().oracle_softmax(lg, lg.shape[0], lg.shape[1], out)
    return out


def route_top1(logits, tau: str):
    """Switch routing (src/harmonymoe/router.py:52-63): (expert_index[T], gate[T])."""
    lg = _f32(logits)
    T, E = lg.shape
    idx = np.empty(T, np.int32)
    g = np.empty(T, np.float32)
    lib().oracle_route_top1(lg, T, E, 1 if tau == "bf16" else 0, idx, g)
    return idx, g


def route_topk(logits, k: int, norm_topk: bool, act: str):
    """Qwen routing (qwen_ep_adapter/qwen_ep.py:48-53): (ids[T,k], w[T,k])."""
    lg = _f32(logits)
    T, E = lg.shape
    ids = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    lib().oracle_route_topk(lg, T, E, k, int(norm_topk), 1 if act == "bf16" else 0, ids, w)
    return ids, w


def near_tie_tokens(logits, k: int, tau: str, rel: float = 2.0 ** -7) -> np.ndarray:
    """Tokens whose routing decision sits within ``rel`` (relative) of a tie between the k-th
    and (k+1)-th probability.  Different-but-valid accumulation orders (cuBLAS, ATen CPU) can
    flip these; fixtures are compared exactly on every other token."""
    p = softmax(logits).astype(np.float64)
    ps = -np.sort(-p, axis=1)
    a, b = ps[:, k - 1], ps[:, k] if ps.shape[1] > k else np.zeros(len(ps))
    return np.abs(a - b) <= rel * np.maximum(a, 1e-30)


# ------------------------------------------------------------------------------ layout
def expert_token_lists(ids: np.ndarray, E: int) -> list:
    """Per expert, the ascending list of (token) rows routed to it (ids is [T] or [T,k]).
    Restates the nonzero lists of src/qosmoe/moe_layer.py:300-303 / qwen_ep.py:86."""
    ids = ids.reshape(ids.shape[0], -1)
    return [np.nonzero((ids == e).any(axis=1))[0] for e in range(E)]


def permutation_world1(ids: np.ndarray, E: int):
    """Expert-major order (stable in token id): rows[R] = token, slot[R]; offsets[E+1].
    src/qosmoe/moe_layer.py:206-215 sorts by expert (the build defines the sort as stable)."""
    ids = ids.reshape(ids.shape[0], -1)
    T, k = ids.shape
    rows, slots, offs = [], [], [0]
    for e in range(E):
        t, j = np.nonzero(ids == e)
        o = np.argsort(t, kind="stable")
        rows.append(t[o])
        slots.append(j[o])
        offs.append(offs[-1] + len(t))
    return np.concatenate(rows).astype(np.int64), np.concatenate(slots).astype(np.int64), np.array(offs)


# ------------------------------------------------------------------------------ plan
def schedule_fixed(meta: np.ndarray, expert_to_gpu) -> np.ndarray:
    """S[src, e, owner(e)] = meta[src, e]  (src/harmonymoe/scheduler.py:268-279)."""
    G, E = meta.shape
    S = np.zeros((G, E, G), np.int64)
    S[:, np.arange(E), np.asarray(expert_to_gpu)] = meta
    return S


def harmony_schedule(meta: np.ndarray, expert_to_gpu, eq_tokens: int) -> np.ndarray:
    """Restatement of Scheduler.schedule_harmony (src/harmonymoe/scheduler.py:324-372).

    Ties go to the first index (torch.argmax / argmin).  One guard is added: an outer pass
    that moves no token ends the loop (the reference would spin forever there, e.g. with
    eq_tokens = 0 and the least-loaded GPU exactly at the average)."""
    meta = np.asarray(meta, np.int64)
    G, E = meta.shape
    S = schedule_fixed(meta, expert_to_gpu)
    avg = int(meta.sum()) // G
    amt = S.sum(axis=(0, 1))
    while (amt > avg).any():
        over = int(np.argmax(amt))
        least = int(np.argmin(amt))
        if least == over or amt[least] + eq_tokens > avg:
            break
        send = S[:, :, over].sum(axis=0)
        e = int(np.argmax(send))
        if send[e] < eq_tokens:
            break
        amount_over = int(amt[over] - avg)
        moved = 0
        while amount_over > 0 and avg - amt[least] > 0:
            senders = S[:, e, over]
            src = int(np.argmax(senders))
            tok = int(senders[src])
            if tok <= 0:
                break
            n = min(tok, int(avg - amt[least]))
            S[src, e, over] -= n
            S[src, e, least] += n
            amt[over] -= n
            amt[least] += n
            amount_over -= n
            moved += n
        if moved == 0:
            break
    return S


def send_order(S: np.ndarray, rank: int, token_lists: list):
    """distribute_tokens (src/harmonymoe/scheduler.py:101-124): the send buffer lists, for
    dst = 0..G-1 and e = 0..E-1, the next S[rank,e,dst] entries of expert e's ascending token
    list.  Returns (rows[token], expert[rows], send_splits[G])."""
    G, E, _ = S.shape
    filled = [0] * E
    rows, exps, splits = [], [], []
    for dst in range(G):
        n0 = len(rows)
        for e in range(E):
            a = int(S[rank, e, dst])
            if a:
                rows.extend(token_lists[e][filled[e]:filled[e] + a].tolist())
                exps.extend([e] * a)
                filled[e] += a
        splits.append(len(rows) - n0)
    return np.array(rows, np.int64), np.array(exps, np.int64), splits


def recv_expert_lists(S: np.ndarray, rank: int) -> list:
    """generate_expert_mask (src/harmonymoe/scheduler.py:185-213) with a stable sort: for each
    expert, its positions in the receive buffer (src ascending, then sender order)."""
    G, E, _ = S.shape
    amounts = S[:, :, rank]
    owner = np.repeat(np.tile(np.arange(E), G), amounts.reshape(-1))
    pos = np.arange(len(owner))
    order = np.argsort(owner, kind="stable")
    counts = amounts.sum(axis=0)
    out, o = [], 0
    for e in range(E):
        out.append(pos[order[o:o + counts[e]]])
        o += counts[e]
    return out


# ------------------------------------------------------------------------------ FFN
def _silu(v):
    return v / (1.0 + np.exp(-v))


def switch_forward(x, Wr, wi, wo, tau: str, compute=np.float64, tensor_cores=None):
    """Switch top-1 block (src/qosmoe/moe_layer.py:196-269 with router.py:52-63):
    y[t] = g[t] * wo[e] ReLU(wi[e] x[t]).  Returns (y, logits, idx, gate).  `compute` is the
    FFN arithmetic type: float64 for checking, float32 for the timed CPU baseline;
    `tensor_cores` the router form (None: the engine's default, router_logits_for)."""
    c = compute
    xc = np.asarray(x, c)
    logits = router_logits_for(x, Wr, tau, tensor_cores)
    idx, gate = route_top1(logits, tau)
    E = wi.shape[0]
    y = np.zeros_like(xc)
    for e in range(E):
        t = np.nonzero(idx == e)[0]
        if len(t) == 0:
            continue
        h = np.maximum(xc[t] @ np.asarray(wi[e], c).T, 0.0)
        y[t] = (h @ np.asarray(wo[e], c).T) * gate[t, None].astype(c)
    return y, logits, idx, gate


def qwen_forward(x, Wg, p: dict, k: int, norm_topk: bool, act: str, compute=np.float64, tensor_cores=None):
    """Qwen top-k + shared-expert block (qwen_ep_adapter/qwen_ep.py:44-97):
    y[t] = sum_j w[t,j] D_c(SiLU(G_c x) * U_c x) + sigmoid(g . x) * D_s(SiLU(G_s x) * U_s x).
    Returns (y, logits, ids, w, shared_gate_sigmoid).  `compute` and `tensor_cores` as in
    switch_forward (the router rows count the shared-expert gate)."""
    c = compute
    xc = np.asarray(x, c)
    logits = router_logits_for(x, Wg, "bf16" if act == "bf16" else "f32", tensor_cores, rows=np.shape(Wg)[0] + 1)
    ids, w = route_topk(logits, k, norm_topk, act)
    E = p["gate"].shape[0]
    y = np.zeros_like(xc)
    for e in range(E):
        t, j = np.nonzero(ids == e)
        if len(t) == 0:
            continue
        xe = xc[t]
        h = _silu(xe @ np.asarray(p["gate"][e], c).T) * (xe @ np.asarray(p["up"][e], c).T)
        y[t] += (h @ np.asarray(p["down"][e], c).T) * w[t, j][:, None].astype(c)
    hs = _silu(xc @ np.asarray(p["s_gate"], c).T) * (xc @ np.asarray(p["s_up"], c).T)
    sg = 1.0 / (1.0 + np.exp(-(xc @ np.asarray(p["s_gate_w"], c).T)))
    y += (hs @ np.asarray(p["s_down"], c).T) * sg
    return y, logits, ids, w, sg[:, 0]


def e4m3_rn(v) -> np.ndarray:
    """float32 values (|v| < 464) -> e4m3 bytes, round to nearest even (the sign of zero kept)."""
    v = np.asarray(v, np.float32).astype(np.float64)
    a = np.abs(v)
    _, ex = np.frexp(np.where(a > 0, a, 1.0))
    e = np.maximum(ex.astype(np.float64) - 1.0, -6.0)  # subnormals: quantum 2^-9
    q = np.exp2(e - 3.0)
    r = np.rint(a / q) * q
    _, ex2 = np.frexp(np.where(r > 0, r, 1.0))
    e2 = ex2.astype(np.int64) - 1
    normal = (r > 0) & (e2 >= -6)
    expf = np.where(normal, e2 + 7, 0)
    mant = np.where(normal, np.rint((r / np.exp2(e2.astype(np.float64)) - 1.0) * 8.0), np.rint(r / 2.0 ** -9))
    bits = (expf.astype(np.int64) << 3) | mant.astype(np.int64)
    bits = np.where(r > 0, bits, 0) | np.where(np.signbit(v), 0x80, 0)
    return bits.astype(np.uint8)


def e4m3_value(b) -> np.ndarray:
    """e4m3 bytes -> float32 values."""
    b = np.asarray(b, np.int64)
    expf, mant = (b >> 3) & 15, b & 7
    mag = np.where(expf > 0, np.exp2(expf - 7.0) * (1.0 + mant / 8.0), np.exp2(-9.0) * mant)
    return np.where(b & 0x80, -mag, mag).astype(np.float32)


def split_e4m3(x) -> tuple[np.ndarray, np.ndarray]:
    """Two-term e4m3 rows of bf16 rows x [rows, K] (values given as float32), the restatement of
    dsca_split_rows: per row s = 2^(134 - E) with E the bf16 exponent field of max|x| clamped to
    [8, 254]; v = x s, hi = RN(v), lo = RN(v - hi) in float32 arithmetic.  Returns (bytes
    [rows, 2 Kp] = [hi | lo], Kp = K rounded up to 128, zero padded; 1 / s [rows] float32)."""
    x = np.asarray(x, np.float32)
    rows, K = x.shape
    kp = (K + 127) // 128 * 128
    mx = np.abs(x).max(axis=1) if K else np.zeros(rows, np.float32)
    E = (mx.view(np.uint32) >> 23).astype(np.int64) & 0xFF
    E = np.clip(E, 8, 254)
    s = ((261 - E).astype(np.uint32) << 23).view(np.float32)
    inv = ((E - 7).astype(np.uint32) << 23).view(np.float32)
    v = (x * s[:, None]).astype(np.float32)
    hi = e4m3_rn(v)
    lo = e4m3_rn((v - e4m3_value(hi)).astype(np.float32))
    out = np.zeros((rows, 2 * kp), np.uint8)
    out[:, :K] = hi
    out[:, kp:kp + K] = lo
    return out, inv


def max_rel_err(a, ref) -> float:
    """max|a - ref| / max|ref| over the tensor."""
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.abs(ref).max()
    return float(np.abs(a - ref).max() / (den if den > 0 else 1.0))


# ------------------------------------------------------------------------------ QoS planner
def qos_token_scores(x, x_prev, logits, expert_index, seq_priority, remaining, valid, d_model,
                     alpha=1.0, beta=0.1, delta=0.5, target_batch=64, eps=1e-6, mode="router_var"):
    """QoSPlanner.compute_token_scores (src/qosmoe/planner.py:63-151) for per-token inputs of the
    token count: info gain = |x - x_prev| (|x| when x_prev is missing or of another shape,
    :100-110), attention factor = population variance of the logits row (:52-61), small-batch
    penalty = target / (count of the token's expert + eps) (:117-123), priority = P (1 + gain
    (1 + attn) / (alpha d + beta rem + delta penalty)), invalid tokens -1e9 (:135-151).
    float64 arithmetic on the float32 inputs."""
    x = np.asarray(x, np.float64)
    if x_prev is not None and np.shape(x_prev) == x.shape:
        gain = np.linalg.norm(x - np.asarray(x_prev, np.float64), axis=1)
    else:
        gain = np.linalg.norm(x, axis=1)
    lg = np.asarray(logits, np.float64)
    attn = lg.var(axis=1) if mode == "router_var" else np.zeros(len(x))
    ei = np.asarray(expert_index, np.int64)
    cnt = np.bincount(ei, minlength=lg.shape[1]).astype(np.float64)
    penalty = target_batch / (cnt[ei] + eps)
    denom = alpha * d_model + beta * np.asarray(remaining, np.float64) + delta * penalty
    pri = np.asarray(seq_priority, np.float64) * (1.0 + gain * (1.0 + attn) / denom)
    ok = np.asarray(valid) != 0
    return np.where(ok, pri, -1e9)


def qos_expert_priority(scores, topk_ids, E: int):
    """QoSPlanner.aggregate_expert_priority (src/qosmoe/planner.py:153-170): per expert, the sum
    of the scores of its tokens (every (token, slot) assignment with top-k routing)."""
    ids = np.asarray(topk_ids).reshape(len(scores), -1)
    out = np.zeros(E, np.float64)
    for j in range(ids.shape[1]):
        np.add.at(out, ids[:, j], np.asarray(scores, np.float64))
    return out


def qos_exec_plan(active, priority, cache: list, cache_size: int):
    """QoSPlanner.build_exec_plan (src/qosmoe/planner.py:172-237): resident experts first, then
    the others, each by priority descending (stable: expert id ascending on ties); the slots for
    the experts to load cycle through the free slots, then the resident experts' slots from the
    lowest priority up.  Returns (expert_order, slot_idxs, need_loading)."""
    act = [e for e in range(len(priority)) if e in set(active)]
    loaded = sorted([e for e in act if e in cache], key=lambda e: -priority[e])
    unloaded = sorted([e for e in act if e not in cache], key=lambda e: -priority[e])
    if not unloaded:
        return loaded, [cache.index(e) for e in loaded], []
    low_to_high = [cache.index(e) for e in sorted(loaded, key=lambda e: priority[e])]
    used = set(low_to_high)
    cand = [s for s in range(cache_size) if s not in used] + low_to_high
    cand = cand or [0]
    order, slots, need = loaded + unloaded, [], []
    c = 0
    for e in order:
        if e in cache:
            slots.append(cache.index(e))
        else:
            slots.append(cand[c % len(cand)])
            c += 1
            need.append(e)
    return order, slots, need
