"""Whole-model integration through the plugin, on the CPU.

replace_qosmoe_layer (src/qosmoe/utils.py:16-84) is run on small random-init transformers models
(Switch encoder-decoder, Qwen2-MoE causal LM) with the block it builds swapped for a stand-in
that evaluates the oracle on the arguments the plugin extracted.  The swapped model must give the
unswapped model's logits, which checks in one go: the module-tree walk and layer numbering, the
expert extraction (ModuleDict of DenseActDense, transformers-5.x fused Qwen experts), the router
weight path, the top-k / norm / shared-expert pick-up, the return form the installed
transformers' callers expect, and the oracle's block semantics against transformers' own MoE
blocks.  The same models run through the CUDA block in test_gpu_model.py.
"""
import numpy as np
import pytest
import torch

from hf_models import QWEN_PLUGIN, SWITCH_PLUGIN, moe_blocks, qwen_model, switch_model, token_batch
from oracle import oracle as O
from dsca_moe_b200 import QoSMoEConfig, plugin
from dsca_moe_b200.layers import experts_from_fused, experts_from_list, hf_callers_unpack_tuples

pytest.importorskip("transformers")


class OracleBlock(torch.nn.Module):
    """Stands in for QoSMoELayer: same config in, the oracle's block forward out."""

    built = []

    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        ex = cfg.experts
        self.spec = experts_from_fused(ex) if hasattr(ex, "gate_up_proj") else experts_from_list(list(ex))
        self.w_router = cfg.router_weights.detach().float().numpy()
        OracleBlock.built.append(self)

    def forward(self, h):
        cfg = self.cfg
        x = h.reshape(-1, cfg.d_model).detach().float().numpy()
        if self.spec[0] == "relu":
            y, logits, idx, _ = O.switch_forward(x, self.w_router, self.spec[1].float().numpy(),
                                                 self.spec[2].float().numpy(), "f32")
        else:
            sd = {k: v.detach().float().numpy() for k, v in cfg.shared_expert.state_dict().items()}
            p = dict(gate=self.spec[1].float().numpy(), up=self.spec[2].float().numpy(),
                     down=self.spec[3].float().numpy(), s_gate=sd["gate_proj.weight"],
                     s_up=sd["up_proj.weight"], s_down=sd["down_proj.weight"],
                     s_gate_w=cfg.shared_expert_gate.weight.detach().float().numpy())
            y, logits, idx, _, _ = O.qwen_forward(x, self.w_router, p, cfg.top_k, cfg.norm_topk_prob, "f32")
            idx = idx[:, 0]
        out = torch.from_numpy(y.astype(np.float32)).view(h.shape)
        if not cfg.return_router_tuple:
            return out
        return out, (torch.from_numpy(logits), torch.from_numpy(idx.astype(np.int64)))


@pytest.fixture
def oracle_blocks(monkeypatch):
    OracleBlock.built = []
    monkeypatch.setattr(plugin, "QoSMoELayer", OracleBlock)
    return OracleBlock.built


def _cfg():
    return QoSMoEConfig(rank=0, world_size=1, expert_cache_size=1 << 10)


@torch.no_grad()
def test_switch_model_swap_matches_transformers(oracle_blocks):
    model = switch_model(seed=3)
    ids = token_batch(model.config.vocab_size, 2, 24, seed=4)
    dec = token_batch(model.config.vocab_size, 2, 8, seed=5)
    ref = model(input_ids=ids, decoder_input_ids=dec).logits
    hf_blocks = moe_blocks(model, "SwitchTransformersSparseMLP")
    assert len(hf_blocks) == 4  # layers 1 and 3 of the encoder and of the decoder
    router_ws = [b.router.classifier.weight.detach().clone() for b in hf_blocks]

    plugin.replace_qosmoe_layer(model, config=_cfg(), **SWITCH_PLUGIN)

    assert not moe_blocks(model, "SwitchTransformersSparseMLP")
    assert [b.cfg.layer_idx for b in oracle_blocks] == [0, 1, 2, 3]
    for b, w in zip(oracle_blocks, router_ws):  # traversal order = layer order, encoder first
        assert torch.equal(b.cfg.router_weights, w)
        assert (b.cfg.num_experts, b.cfg.d_model, b.cfg.top_k) == (8, 64, 1)
        assert b.cfg.return_router_tuple == hf_callers_unpack_tuples()
    got = model(input_ids=ids, decoder_input_ids=dec).logits
    assert O.max_rel_err(got.numpy(), ref.numpy()) < 1e-4


@pytest.mark.parametrize("norm", [False, True])
@torch.no_grad()
def test_qwen_model_swap_matches_transformers(oracle_blocks, norm):
    model = qwen_model(norm_topk=norm, seed=7)
    ids = token_batch(model.config.vocab_size, 2, 32, seed=8)
    ref = model(input_ids=ids).logits
    assert len(moe_blocks(model, "Qwen2MoeSparseMoeBlock")) == 2

    plugin.replace_qosmoe_layer(model, config=_cfg(), **QWEN_PLUGIN)

    assert len(oracle_blocks) == 2 and not moe_blocks(model, "Qwen2MoeSparseMoeBlock")
    for i, b in enumerate(oracle_blocks):
        assert b.cfg.layer_idx == i
        assert (b.cfg.top_k, b.cfg.norm_topk_prob, b.cfg.num_experts) == (4, norm, 8)
        assert b.cfg.shared_expert is not None and b.cfg.shared_expert_gate is not None
    got = model(input_ids=ids).logits
    assert O.max_rel_err(got.numpy(), ref.numpy()) < 1e-4


def test_fused_expert_extraction_matches_module():
    """transformers-5.x Qwen2MoeExperts: gate rows first in gate_up_proj."""
    model = qwen_model(seed=11)
    blk = moe_blocks(model, "Qwen2MoeSparseMoeBlock")[0]
    kind, g, u, dn = experts_from_fused(blk.experts)
    assert kind == "swiglu" and g.shape == (8, 32, 64) and u.shape == (8, 32, 64) and dn.shape == (8, 64, 32)
    x = torch.randn(5, 64, generator=torch.Generator().manual_seed(0))
    ids = torch.full((5, 1), 3)
    w = torch.ones(5, 1)
    with torch.no_grad():
        ref = blk.experts(x, ids, w)
        got = (torch.nn.functional.silu(x @ g[3].T) * (x @ u[3].T)) @ dn[3].T
    assert torch.allclose(got, ref, rtol=1e-5, atol=1e-6)


def test_no_matching_parent_swaps_nothing(oracle_blocks):
    model = switch_model(seed=1)
    plugin.replace_qosmoe_layer(model, "NoSuchParent", "SwitchTransformersSparseMLP", "experts",
                                "router.classifier", _cfg())
    assert not oracle_blocks and len(moe_blocks(model, "SwitchTransformersSparseMLP")) == 4
