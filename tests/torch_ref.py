"""fp32 torch restatement of the MoE block on the GPU, for full-size checks.

The oracle (numpy float64) checks the kernels at sizes it finishes in seconds; at full size
(4096 tokens of the Qwen1.5-MoE-A2.7B block, 1.1 GB of weights) the same formula is computed here
in fp32 with torch on the device from the same bf16 inputs and weights, for every token, with the
routing (expert ids and weights) taken from the kernel once that routing has been checked
bit-exact against the oracle.  Follows qwen_ep_adapter/qwen_ep.py:44-97 (top-k + shared expert
with its sigmoid gate) and src/qosmoe/moe_layer.py:196-269 (Switch top-1).
"""
import torch
import torch.nn.functional as F


def qwen_block_fp32(x, ids, wts, w, shared_gate_w):
    """x [T, d] bf16; ids / wts [T, k]; w: gate/up [E, I, d], down [E, d, I], s_gate/s_up [Is, d],
    s_down [d, Is] (bf16 device tensors); shared_gate_w [d].  Returns y [T, d] fp32."""
    xf = x.float()
    y = torch.zeros_like(xf)
    ids = ids.long()
    wts = wts.float()
    for e in range(w["gate"].shape[0]):
        t, j = (ids == e).nonzero(as_tuple=True)
        if t.numel() == 0:
            continue
        xe = xf[t]
        h = F.silu(xe @ w["gate"][e].float().T) * (xe @ w["up"][e].float().T)
        y.index_add_(0, t, (h @ w["down"][e].float().T) * wts[t, j, None])
    sg = torch.sigmoid(xf @ shared_gate_w.float().reshape(-1))
    hs = F.silu(xf @ w["s_gate"].float().T) * (xf @ w["s_up"].float().T)
    return y + (hs @ w["s_down"].float().T) * sg[:, None]


def switch_block_fp32(x, idx, gate, wi, wo):
    """Switch top-1: y[t] = gate[t] * wo[e] ReLU(wi[e] x[t]), e = idx[t]."""
    xf = x.float()
    y = torch.zeros_like(xf)
    idx = idx.long().reshape(-1)
    gate = gate.float().reshape(-1)
    for e in range(wi.shape[0]):
        t = (idx == e).nonzero(as_tuple=True)[0]
        if t.numel() == 0:
            continue
        h = torch.relu(xf[t] @ wi[e].float().T)
        y[t] = (h @ wo[e].float().T) * gate[t, None]
    return y


def max_rel_err(a, ref) -> float:
    """max|a - ref| / max|ref| over the whole tensor."""
    a, ref = a.float(), ref.float()
    return float((a - ref).abs().max() / ref.abs().max().clamp_min(1e-30))
