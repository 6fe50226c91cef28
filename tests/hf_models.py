"""Small random-init Hugging Face models for the whole-model plugin tests.

Switch: SwitchTransformersForConditionalGeneration shaped like switch-base-64 scaled down (MoE in
every other encoder and decoder layer, top-1 ReLU experts, no expert capacity drop at these
sizes).  Qwen: Qwen2MoeForCausalLM shaped like Qwen1.5-MoE-A2.7B scaled down (every layer
sparse, softmax top-4, shared expert with a sigmoid gate).  The MoE parameters are re-drawn from
a seeded N(0, s^2) so that routing has no exact ties (the Qwen router starts at zero in
transformers) and the experts contribute at a scale comparable to the residual stream.

The plugin arguments are the reference's command-line values (src/args.py:186-215,
README.md:66-69) for transformers 4.x; transformers 5.x keeps the Switch names and fuses the
Qwen experts into one module (`experts`, router `gate`).
"""
from __future__ import annotations

import torch

SWITCH_PLUGIN = dict(moe_parent_type="SwitchTransformersLayerFF", moe_type="SwitchTransformersSparseMLP",
                     name_experts="experts", router_tensor_path="router.classifier")
QWEN_PLUGIN = dict(moe_parent_type="Qwen2MoeDecoderLayer", moe_type="Qwen2MoeSparseMoeBlock",
                   name_experts="experts", router_tensor_path="gate")


def _redraw(module: torch.nn.Module, gen: torch.Generator, scale: float):
    with torch.no_grad():
        for p in module.parameters():
            fan_in = p.shape[-1]
            p.copy_(torch.randn(p.shape, generator=gen) * (scale / fan_in ** 0.5))


def switch_model(d=64, d_ff=128, E=8, layers=4, seed=0):
    from transformers import SwitchTransformersConfig, SwitchTransformersForConditionalGeneration

    cfg = SwitchTransformersConfig(vocab_size=256, d_model=d, d_kv=16, d_ff=d_ff, num_layers=layers,
                                   num_decoder_layers=layers, num_heads=4, num_experts=E,
                                   expert_capacity=1 << 20, encoder_sparse_step=2, decoder_sparse_step=2,
                                   router_jitter_noise=0.0, dropout_rate=0.0, decoder_start_token_id=0,
                                   pad_token_id=0, eos_token_id=1)
    torch.manual_seed(seed)
    model = SwitchTransformersForConditionalGeneration(cfg).eval()
    gen = torch.Generator().manual_seed(seed + 1)
    for name, mod in model.named_modules():
        if type(mod).__name__ == "SwitchTransformersSparseMLP":
            _redraw(mod.router, gen, 4.0)
            _redraw(mod.experts, gen, 1.0)
    return model


def qwen_model(d=64, I=32, Is=64, E=8, k=4, layers=2, norm_topk=False, seed=0):
    from transformers import Qwen2MoeConfig, Qwen2MoeForCausalLM

    cfg = Qwen2MoeConfig(vocab_size=256, hidden_size=d, intermediate_size=2 * d, moe_intermediate_size=I,
                         shared_expert_intermediate_size=Is, num_hidden_layers=layers, num_attention_heads=4,
                         num_key_value_heads=2, num_experts=E, num_experts_per_tok=k, norm_topk_prob=norm_topk,
                         decoder_sparse_step=1, mlp_only_layers=[], max_position_embeddings=512)
    torch.manual_seed(seed)
    model = Qwen2MoeForCausalLM(cfg).eval()
    gen = torch.Generator().manual_seed(seed + 1)
    for name, mod in model.named_modules():
        if type(mod).__name__ == "Qwen2MoeSparseMoeBlock":
            _redraw(mod, gen, 1.0)
            _redraw(mod.gate, gen, 4.0)
    return model


def moe_blocks(model, type_name: str) -> list:
    return [m for m in model.modules() if type(m).__name__ == type_name]


def token_batch(vocab: int, B: int, S: int, seed: int):
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(2, vocab, (B, S), generator=gen)
