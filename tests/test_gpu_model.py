"""Whole models through the plugin on the GPU: small random-init Switch and Qwen2-MoE models from
transformers, their MoE blocks swapped for the CUDA block by replace_qosmoe_layer
(src/qosmoe/utils.py:16-84) or, for Qwen, by patch() (qwen_ep_adapter/qwen_ep.py:100-109).

* f32: the swapped model's logits equal the unswapped model's within 1e-4 (max|d| / max|ref|).
* bf16: every swapped block is compared with the transformers block it replaced, on the hidden
  states that reached it inside the swapped model, within 2e-2 on the tokens whose routing is
  not a near-tie (transformers routes the Switch block in fp32 and accumulates in its own order);
  the model's logits stay finite and near the unswapped model's (norm-wise within 0.25: a token
  routed to another expert at a near-tie changes its whole MoE output, and later layers mix it).
"""
import copy

import pytest
import torch

from hf_models import QWEN_PLUGIN, SWITCH_PLUGIN, moe_blocks, qwen_model, switch_model, token_batch
from oracle import oracle as O
from dsca_moe_b200 import QoSMoEConfig, RequestStateTable, get_qosmoe_layers, patch, replace_qosmoe_layer

pytestmark = pytest.mark.gpu
pytest.importorskip("transformers")

F32_TOL, BF16_TOL = 1e-4, 2e-2


def _swap(model, plugin_args, B, S):
    cfg = QoSMoEConfig(rank=0, world_size=1, expert_cache_size=1 << 10)
    replace_qosmoe_layer(model, config=cfg, **plugin_args)
    layers = get_qosmoe_layers(model)
    ctx = RequestStateTable(cfg).build_context({"attention_mask": torch.ones(B, S, dtype=torch.long)})
    for layer in layers:
        layer.set_runtime_context(ctx)
    return layers


def _norm_rel(a, ref):
    a, ref = a.double(), ref.double()
    return float((a - ref).norm() / ref.norm())


@torch.no_grad()
def test_switch_model_f32_through_plugin(cuda):
    model = switch_model(seed=3).to(cuda)
    ids = token_batch(model.config.vocab_size, 4, 64, seed=4).to(cuda)
    dec = token_batch(model.config.vocab_size, 4, 16, seed=5).to(cuda)
    ref = model(input_ids=ids, decoder_input_ids=dec).logits
    layers = _swap(model, SWITCH_PLUGIN, 4, 64)
    assert len(layers) == 4 and not moe_blocks(model, "SwitchTransformersSparseMLP")
    got = model(input_ids=ids, decoder_input_ids=dec).logits
    torch.cuda.synchronize()
    for layer in layers:
        layer.engine.check()
    assert O.max_rel_err(got.cpu().numpy(), ref.cpu().numpy()) < F32_TOL


@pytest.mark.parametrize("route", ["plugin", "patch"])
@torch.no_grad()
def test_qwen_model_f32(cuda, route):
    model = qwen_model(seed=7, layers=3).to(cuda)
    ids = token_batch(model.config.vocab_size, 4, 64, seed=8).to(cuda)
    ref = model(input_ids=ids).logits
    if route == "plugin":
        assert len(_swap(model, QWEN_PLUGIN, 4, 64)) == 3
    else:
        assert patch(model, 0, 1) == 3
    assert not moe_blocks(model, "Qwen2MoeSparseMoeBlock")
    got = model(input_ids=ids).logits
    torch.cuda.synchronize()
    assert O.max_rel_err(got.cpu().numpy(), ref.cpu().numpy()) < F32_TOL


def _block_checks(model, hf_type, plugin_args, run, B, S, k):
    """Swap, run the model once with hooks on the swapped blocks, then rerun every saved
    transformers block on the same input and compare token by token."""
    originals = [copy.deepcopy(b) for b in moe_blocks(model, hf_type)]
    layers = _swap(model, plugin_args, B, S)
    seen = []
    hooks = [m.register_forward_hook(lambda mod, inp, out: seen.append((inp[0].clone(), out)))
             for m in layers]
    got = run()
    torch.cuda.synchronize()
    for h in hooks:
        h.remove()
    assert len(seen) == len(originals) == len(layers)
    for layer, hf_block, (x, out) in zip(layers, originals, seen):
        y = out[0] if isinstance(out, tuple) else out
        y_ref = hf_block(x)
        y_ref = y_ref[0] if isinstance(y_ref, tuple) else y_ref
        xs = x.reshape(-1, x.shape[-1]).float().cpu().numpy()
        w = layer.engine.router_weight.float().cpu().numpy()
        logits = O.router_logits(xs, w, "bf16")
        # bf16 logits are within half an ulp (2^-5 at |logit| ~ 4) of transformers' fp32 ones:
        # tokens whose top-k / (k+1) gap is that small may route differently
        keep = ~O.near_tie_tokens(logits, k, "bf16", rel=2.0 ** -4)
        assert keep.mean() > 0.8
        a = y.reshape(-1, y.shape[-1]).float().cpu().numpy()[keep]
        r = y_ref.reshape(-1, y_ref.shape[-1]).float().cpu().numpy()[keep]
        assert O.max_rel_err(a, r) < BF16_TOL
    return got


@torch.no_grad()
def test_switch_model_bf16_blocks(cuda):
    model = switch_model(seed=13).to(cuda, torch.bfloat16)
    ids = token_batch(model.config.vocab_size, 4, 64, seed=14).to(cuda)
    dec = token_batch(model.config.vocab_size, 4, 16, seed=15).to(cuda)
    ref = model(input_ids=ids, decoder_input_ids=dec).logits
    got = _block_checks(model, "SwitchTransformersSparseMLP", SWITCH_PLUGIN,
                        lambda: model(input_ids=ids, decoder_input_ids=dec).logits, 4, 64, 1)
    assert torch.isfinite(got).all() and _norm_rel(got, ref) < 0.25


@torch.no_grad()
def test_qwen_model_bf16_blocks(cuda):
    model = qwen_model(seed=17, layers=3).to(cuda, torch.bfloat16)
    ids = token_batch(model.config.vocab_size, 4, 64, seed=18).to(cuda)
    ref = model(input_ids=ids).logits
    got = _block_checks(model, "Qwen2MoeSparseMoeBlock", QWEN_PLUGIN, lambda: model(input_ids=ids).logits,
                        4, 64, 4)
    assert torch.isfinite(got).all() and _norm_rel(got, ref) < 0.25


@pytest.mark.parametrize("world", [2, 4])
def test_qwen_model_expert_parallel_matches_single_gpu(world):
    """A small Qwen2-MoE model swapped at world_size 2 / 4 through replace_qosmoe_layer (one rank
    per GPU, tests/model_ep_check.py): every rank's logits equal the same model's at world_size 1
    and stay within 1e-4 of the unswapped transformers model.  Skipped with fewer GPUs."""
    import json
    import os
    import socket
    import subprocess
    import sys

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(root, "tests", "model_ep_check.py")]
    p = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True, timeout=700)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    res = json.loads([line for line in p.stdout.splitlines() if line.startswith("{")][-1])
    assert res["ok"], res
