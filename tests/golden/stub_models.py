"""Seeded stand-ins for the checkpoints the reference splits (test infrastructure).

Both the fixture generator (make_golden.py, which runs the reference's own
split_dense and DesdemonaEngine on them) and the GPU tests (which run this
repository's split_dense and engine on them) build these models from the same
CPU generator seeds, so the tests need only the reference's outputs, not the
large weight files.
"""
from __future__ import annotations

import types

import torch

H = 4096


def _lin(g, o, i, std=0.02):
    return types.SimpleNamespace(weight=types.SimpleNamespace(data=(torch.randn(o, i, generator=g) * std).half()))


def _norm(g, n):
    return types.SimpleNamespace(weight=types.SimpleNamespace(data=(1.0 + 0.1 * torch.randn(n, generator=g)).half()))


def engine_stub_model(seed: int = 11, n_layers: int = 2, inter: int = 64, vocab: int = 64):
    """A 2-layer causal LM with Llama attention geometry (hidden 4096, 32
    query / 8 key-value heads of 128), a small SwiGLU FFN and a small
    vocabulary: only the attributes split_dense reads (the reference's
    splitter.py:151-183, :195-198, :265-289)."""
    g = torch.Generator().manual_seed(seed)
    layers = []
    for _ in range(n_layers):
        attn = types.SimpleNamespace(q_proj=_lin(g, H, H), k_proj=_lin(g, 1024, H), v_proj=_lin(g, 1024, H),
                                     o_proj=_lin(g, H, H))
        mlp = types.SimpleNamespace(gate_proj=_lin(g, inter, H), up_proj=_lin(g, inter, H),
                                    down_proj=_lin(g, H, inter))
        layers.append(types.SimpleNamespace(self_attn=attn, mlp=mlp, input_layernorm=_norm(g, H),
                                            post_attention_layernorm=_norm(g, H)))
    inner = types.SimpleNamespace(layers=layers, embed_tokens=_lin(g, vocab, H, std=1.0), norm=_norm(g, H))
    cfg = types.SimpleNamespace(hidden_size=H, num_hidden_layers=n_layers, intermediate_size=inter,
                                vocab_size=vocab, num_attention_heads=32, num_key_value_heads=8,
                                rope_theta=10000.0, rms_norm_eps=1e-5, hidden_act="silu",
                                model_type="llama", max_position_embeddings=64)
    return types.SimpleNamespace(config=cfg, model=inner, lm_head=_lin(g, vocab, H))


def engine_stub_profile(seed: int = 12, n_layers: int = 2, inter: int = 64) -> dict:
    """profile.json contents: seeded activation frequencies per layer."""
    g = torch.Generator().manual_seed(seed)
    return {"layers": {str(li): {"expert_0": torch.rand(inter, generator=g).tolist()} for li in range(n_layers)}}


def engine_stub_predictor_params(layer: int, seed: int = 13, inter: int = 64, rank: int = 16):
    """Predictor weights of one layer (down [rank, H], up [inter, rank], bias
    [inter]): small weights and biases of +-(3..4), so every logit sits far
    from the 0.5 threshold and any fp32 evaluation order selects the same set."""
    g = torch.Generator().manual_seed(seed * 100 + layer)
    down = torch.randn(rank, H, generator=g) * 0.02
    up = torch.randn(inter, rank, generator=g) * 0.02
    sign = torch.where(torch.rand(inter, generator=g) < 0.5, -1.0, 1.0)
    bias = sign * (3.0 + torch.rand(inter, generator=g))
    return down, up, bias
