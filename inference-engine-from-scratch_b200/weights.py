"""Seeded random-init weights and synthetic token-ID prompts for the BASELINE configs.

BASELINE config 1 specifies Qwen3 weights drawn N(0, 0.02) from seed 0 with RMSNorm weights 1,
and prompts of token IDs (no tokenizer, no checkpoint download). ``make_weights`` fixes one draw
order so that the CPU oracle, the reference (loaded with ``load_state_dict``) and the CUDA path
all see the same tensors. The parameter names are the Hugging Face / reference ones
(nanoengine/src/nanoengine/models/qwen3.py:71-203).
"""

from __future__ import annotations

import torch

from .config import Qwen3Config

INIT_STD = 0.02
MOTIF_LENGTH = 16


def make_weights(cfg: Qwen3Config, seed: int = 0, std: float = INIT_STD) -> dict[str, torch.Tensor]:
    """fp32 CPU state dict. Draw order: embedding, then per layer q,k,v,o,gate,up,down, then head."""
    g = torch.Generator().manual_seed(seed)

    def normal(rows: int, cols: int) -> torch.Tensor:
        return torch.empty(rows, cols).normal_(0.0, std, generator=g)

    h, d = cfg.hidden_size, cfg.head_dim
    w: dict[str, torch.Tensor] = {"model.embed_tokens.weight": normal(cfg.vocab_size, h)}
    for layer in range(cfg.num_hidden_layers):
        p = f"model.layers.{layer}."
        w[p + "self_attn.q_proj.weight"] = normal(cfg.num_attention_heads * d, h)
        w[p + "self_attn.k_proj.weight"] = normal(cfg.num_key_value_heads * d, h)
        w[p + "self_attn.v_proj.weight"] = normal(cfg.num_key_value_heads * d, h)
        w[p + "self_attn.o_proj.weight"] = normal(h, cfg.num_attention_heads * d)
        w[p + "mlp.gate_proj.weight"] = normal(cfg.intermediate_size, h)
        w[p + "mlp.up_proj.weight"] = normal(cfg.intermediate_size, h)
        w[p + "mlp.down_proj.weight"] = normal(h, cfg.intermediate_size)
        w[p + "self_attn.q_norm.weight"] = torch.ones(d)
        w[p + "self_attn.k_norm.weight"] = torch.ones(d)
        w[p + "input_layernorm.weight"] = torch.ones(h)
        w[p + "post_attention_layernorm.weight"] = torch.ones(h)
    w["model.norm.weight"] = torch.ones(h)
    if not cfg.tie_word_embeddings:
        w["lm_head.weight"] = normal(cfg.vocab_size, h)
    return w


def cast_weights(weights: dict[str, torch.Tensor], dtype: torch.dtype) -> dict[str, torch.Tensor]:
    return {name: t.to(dtype) for name, t in weights.items()}


def make_prompt(vocab_size: int, length: int, seed: int, motif: bool) -> list[int]:
    """A seeded prompt: a 16-token motif repeated (``motif``) or uniform random IDs."""
    g = torch.Generator().manual_seed(seed)
    if motif:
        base = torch.randint(0, vocab_size, (MOTIF_LENGTH,), generator=g).tolist()
        return (base * (length // MOTIF_LENGTH + 1))[:length]
    return torch.randint(0, vocab_size, (length,), generator=g).tolist()


def make_prompts(num_users: int, vocab_size: int, length: int = 64, seed: int = 0) -> list[list[int]]:
    """short_chat prompts: even users motif-repeated, odd users uniform (config 2).

    User 0 with seed 0 is config 1's prompt (a seed-0 16-token motif repeated 4 times).
    """
    return [make_prompt(vocab_size, length, seed + u, motif=(u % 2 == 0)) for u in range(num_users)]
