"""Seeded random-init weights for the Qwen2.5-1.5B architecture (test oracle).

TEST INFRASTRUCTURE ONLY: used by tests/ and the golden-fixture script to give
the reference model, the oracle model and the product model one identical
state dict.  Weights and biases ~ N(0, 0.02) (config.json
initializer_range, reference model.py:35), RMSNorm weights = 1.  Each tensor
has its own generator seeded from (seed, index in a fixed name order), so
the result does not depend on torch's global RNG state.
"""
from __future__ import annotations

import torch

HIDDEN, LAYERS, HEADS, KV_HEADS, HEAD_DIM, INTER, VOCAB = 1536, 28, 12, 2, 128, 8960, 151936


def param_shapes() -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) of every parameter of the reference Qwen2ForCausalLM
    (model.py:78-149), in a fixed order."""
    out = [("embed_tokens.weight", (VOCAB, HIDDEN))]
    for i in range(LAYERS):
        p = f"layers.{i}."
        out += [
            (p + "input_layernorm.weight", (HIDDEN,)),
            (p + "self_attn.q_proj.weight", (HEADS * HEAD_DIM, HIDDEN)),
            (p + "self_attn.q_proj.bias", (HEADS * HEAD_DIM,)),
            (p + "self_attn.k_proj.weight", (KV_HEADS * HEAD_DIM, HIDDEN)),
            (p + "self_attn.k_proj.bias", (KV_HEADS * HEAD_DIM,)),
            (p + "self_attn.v_proj.weight", (KV_HEADS * HEAD_DIM, HIDDEN)),
            (p + "self_attn.v_proj.bias", (KV_HEADS * HEAD_DIM,)),
            (p + "self_attn.o_proj.weight", (HIDDEN, HEADS * HEAD_DIM)),
            (p + "post_attention_layernorm.weight", (HIDDEN,)),
            (p + "mlp.gate_proj.weight", (INTER, HIDDEN)),
            (p + "mlp.up_proj.weight", (INTER, HIDDEN)),
            (p + "mlp.down_proj.weight", (HIDDEN, INTER)),
        ]
    out.append(("norm.weight", (HIDDEN,)))
    return out


def random_state_dict(seed: int, dtype: torch.dtype = torch.float32, std: float = 0.02) -> dict:
    sd = {}
    for i, (name, shape) in enumerate(param_shapes()):
        if name.endswith("layernorm.weight") or name == "norm.weight":
            sd[name] = torch.ones(shape, dtype=dtype)
            continue
        g = torch.Generator().manual_seed(seed * 1_000_003 + i)
        sd[name] = torch.randn(shape, generator=g, dtype=torch.float32).mul_(std).to(dtype)
    return sd
