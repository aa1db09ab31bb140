"""Qwen3 forward over a paged KV pool, restated on the CPU in torch (TEST INFRASTRUCTURE).

Restates, in order of use (paths relative to ``nanoengine/src/nanoengine``):

* ``RMSNorm.forward``              models/qwen3.py:39-44   fp32 statistics, cast back, then x weight
* ``build_rotary_tables``          models/qwen3.py:47-57   fp32 angles, cos/sin cast to model dtype
* ``rotate_half`` / ``apply_rotary_embedding``  models/qwen3.py:60-68
* ``Qwen3Attention.forward``       models/qwen3.py:89-115  q/k RMSNorm before RoPE, GQA
* ``write_to_cache``               models/attention_context.py:42-54
* ``read_from_cache``              models/attention_context.py:57-63
* ``build_attention_mask``         models/attention_context.py:32-39
* ``run_cached_attention``         models/attention_context.py:66-109 (SDPA with ``enable_gqa``)
* ``Qwen3MLP.forward``             models/qwen3.py:127-129
* ``Qwen3DecoderLayer.forward``    models/qwen3.py:140-150
* ``Qwen3Model.forward``           models/qwen3.py:164-178
* ``compute_logits``               models/qwen3.py:197-203
* ``quantize_vectors``             models/int8_quantization.py:30-34
* ``Int8Linear.forward``           models/int8_quantization.py:55-57
* ``KVCachePool``                  engine/memory/kv_cache_pool.py:34-69 (scratch slot = num_slots)

Weights are a plain ``dict[str, Tensor]`` with Hugging Face parameter names, so the same tensors
can be loaded into the reference model (``load_state_dict``) and into the CUDA path.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch.nn import functional

INT8_MAX = 127
MIN_SCALE = 1e-8
QUANTIZED_PROJECTIONS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def rms_norm(hidden: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """models/qwen3.py:39-44."""
    input_dtype = hidden.dtype
    hidden = hidden.float()
    variance = hidden.pow(2).mean(dim=-1, keepdim=True)
    hidden = hidden * torch.rsqrt(variance + eps)
    return weight * hidden.to(input_dtype)


def rotary_tables(positions: torch.Tensor, head_dim: int, theta: float, dtype: torch.dtype):
    """models/qwen3.py:47-57; ``positions`` is ``[b, q]``, returns ``[b, 1, q, d]`` cos and sin."""
    exponents = torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim
    inverse = 1.0 / (theta**exponents)
    angles = positions.float()[..., None] * inverse
    angles = torch.cat((angles, angles), dim=-1).unsqueeze(1)
    return angles.cos().to(dtype), angles.sin().to(dtype)


def rotate_half(vectors: torch.Tensor) -> torch.Tensor:
    """models/qwen3.py:60-62."""
    first, second = vectors.chunk(2, dim=-1)
    return torch.cat((-second, first), dim=-1)


def apply_rotary(vectors: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """models/qwen3.py:65-68."""
    return vectors * cos + rotate_half(vectors) * sin


def quantize_vectors(values: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """models/int8_quantization.py:30-34: one symmetric int8 scale per last-dim vector."""
    scales = values.abs().amax(dim=-1, keepdim=True).float().clamp(min=MIN_SCALE) / INT8_MAX
    quantized = torch.round(values.float() / scales).clamp(-INT8_MAX, INT8_MAX).to(torch.int8)
    return quantized, scales.to(values.dtype)


def quantize_weights(weights: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """models/int8_quantization.py:50-73: q/k/v/o/gate/up/down become int8 + per-row scale.

    Returns a new dict where each quantized ``<name>.weight`` is replaced by
    ``<name>.weight_int8`` (int8 ``[out, in]``) and ``<name>.weight_scale`` (``[out]`` in the
    weight dtype). Embeddings, norms and the output head stay as they are.
    """
    out: dict[str, torch.Tensor] = {}
    for name, tensor in weights.items():
        base = name[: -len(".weight")] if name.endswith(".weight") else name
        if base.rsplit(".", 1)[-1] in QUANTIZED_PROJECTIONS:
            q, s = quantize_vectors(tensor)
            out[base + ".weight_int8"] = q
            out[base + ".weight_scale"] = s.squeeze(-1)
        else:
            out[name] = tensor
    return out


def linear(weights: dict[str, torch.Tensor], base: str, inputs: torch.Tensor) -> torch.Tensor:
    """``nn.Linear`` (no bias) or ``Int8Linear.forward`` (models/int8_quantization.py:55-57)."""
    full = weights.get(base + ".weight")
    if full is not None:
        return functional.linear(inputs, full)
    weight = weights[base + ".weight_int8"].to(inputs.dtype) * weights[base + ".weight_scale"][:, None]
    return functional.linear(inputs, weight)


@dataclass
class KVPool:
    """engine/memory/kv_cache_pool.py:34-69: per layer ``[num_slots + 1, kv_heads, d]``."""

    key_caches: list[torch.Tensor]
    value_caches: list[torch.Tensor]
    key_scales: list[torch.Tensor] | None
    value_scales: list[torch.Tensor] | None
    num_slots: int

    @property
    def scratch_slot(self) -> int:
        return self.num_slots

    @classmethod
    def create(cls, cfg, num_slots: int, dtype: torch.dtype, int8: bool = False) -> "KVPool":
        shape = (num_slots + 1, cfg.num_key_value_heads, cfg.head_dim)
        scale_shape = (num_slots + 1, cfg.num_key_value_heads, 1)
        cache_dtype = torch.int8 if int8 else dtype
        layers = range(cfg.num_hidden_layers)
        keys = [torch.zeros(shape, dtype=cache_dtype) for _ in layers]
        values = [torch.zeros(shape, dtype=cache_dtype) for _ in layers]
        key_scales = [torch.zeros(scale_shape, dtype=dtype) for _ in layers] if int8 else None
        value_scales = [torch.zeros(scale_shape, dtype=dtype) for _ in layers] if int8 else None
        return cls(keys, values, key_scales, value_scales, num_slots)


@dataclass
class StepContext:
    """models/attention_context.py:16-29 (padded ``[b, q]`` step over ``c`` context tokens)."""

    positions: torch.Tensor  # [b, q]
    slot_mapping: torch.Tensor  # [b, q]; padding -> scratch slot
    context_slots: torch.Tensor  # [b, c]
    attention_mask: torch.Tensor  # [b, 1, q, c]


def attention_mask(positions: torch.Tensor, context_lengths: torch.Tensor, context_length: int):
    """models/attention_context.py:32-39: causal and length mask."""
    keys = torch.arange(context_length)
    causal = keys[None, None, :] <= positions[:, :, None]
    inside = keys[None, None, :] < context_lengths[:, None, None]
    return (causal & inside).unsqueeze(1)


def _write(cache, scales, slots, vectors):
    """models/attention_context.py:42-54."""
    if scales is None:
        cache.index_copy_(0, slots, vectors)
        return
    quantized, vector_scales = quantize_vectors(vectors)
    cache.index_copy_(0, slots, quantized)
    scales.index_copy_(0, slots, vector_scales)


def _read(cache, scales, slots, dtype):
    """models/attention_context.py:57-63 (gather + int8 dequant in the model dtype)."""
    if scales is None:
        return cache[slots]
    return cache[slots].to(dtype) * scales[slots]


def cached_attention(queries, keys, values, ctx: StepContext, pool: KVPool, layer: int):
    """models/attention_context.py:66-109."""
    key_scales = pool.key_scales[layer] if pool.key_scales else None
    value_scales = pool.value_scales[layer] if pool.value_scales else None
    slots = ctx.slot_mapping.reshape(-1)
    shape = (-1, keys.shape[1], keys.shape[3])
    _write(pool.key_caches[layer], key_scales, slots, keys.transpose(1, 2).reshape(shape))
    _write(pool.value_caches[layer], value_scales, slots, values.transpose(1, 2).reshape(shape))
    context_keys = _read(pool.key_caches[layer], key_scales, ctx.context_slots, queries.dtype)
    context_values = _read(pool.value_caches[layer], value_scales, ctx.context_slots, queries.dtype)
    return functional.scaled_dot_product_attention(
        queries,
        context_keys.transpose(1, 2),
        context_values.transpose(1, 2),
        attn_mask=ctx.attention_mask,
        enable_gqa=True,
    )


def forward(weights, cfg, token_ids: torch.Tensor, ctx: StepContext | None, pool: KVPool | None):
    """models/qwen3.py:164-178 (+ the layers it calls). Returns final-normed hidden ``[b, q, H]``.

    Without ``ctx`` the whole sequence is recomputed with causal SDPA (models/qwen3.py:105-111).
    """
    eps = cfg.rms_norm_eps
    hidden = functional.embedding(token_ids, weights["model.embed_tokens.weight"])
    dtype = hidden.dtype
    if ctx is None:
        positions = torch.arange(token_ids.shape[1]).expand(token_ids.shape)
    else:
        positions = ctx.positions
    # (tables from CPU positions; moved to the weights' device when they live on a GPU)
    cos, sin = (t.to(hidden.device) for t in rotary_tables(positions.cpu(), cfg.head_dim, cfg.rope_theta, dtype))
    b, q, _ = hidden.shape
    nh, nkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    for layer in range(cfg.num_hidden_layers):
        p = f"model.layers.{layer}."
        x = rms_norm(hidden, weights[p + "input_layernorm.weight"], eps)
        qs = linear(weights, p + "self_attn.q_proj", x).view(b, q, nh, d)
        ks = linear(weights, p + "self_attn.k_proj", x).view(b, q, nkv, d)
        vs = linear(weights, p + "self_attn.v_proj", x).view(b, q, nkv, d)
        qs = rms_norm(qs, weights[p + "self_attn.q_norm.weight"], eps).transpose(1, 2)
        ks = rms_norm(ks, weights[p + "self_attn.k_norm.weight"], eps).transpose(1, 2)
        vs = vs.transpose(1, 2)
        qs = apply_rotary(qs, cos, sin)
        ks = apply_rotary(ks, cos, sin)
        if ctx is None:
            group = nh // nkv
            attn = functional.scaled_dot_product_attention(
                qs, ks.repeat_interleave(group, 1), vs.repeat_interleave(group, 1), is_causal=True
            )
        else:
            attn = cached_attention(qs, ks, vs, ctx, pool, layer)
        attn = attn.transpose(1, 2).reshape(b, q, -1)
        hidden = hidden + linear(weights, p + "self_attn.o_proj", attn)
        x = rms_norm(hidden, weights[p + "post_attention_layernorm.weight"], eps)
        gated = functional.silu(linear(weights, p + "mlp.gate_proj", x)) * linear(
            weights, p + "mlp.up_proj", x
        )
        hidden = hidden + linear(weights, p + "mlp.down_proj", gated)
    return rms_norm(hidden, weights["model.norm.weight"], eps)


def compute_logits(weights, cfg, hidden: torch.Tensor) -> torch.Tensor:
    """models/qwen3.py:197-203 (tied embeddings unless ``lm_head.weight`` is present)."""
    head = weights.get("lm_head.weight")
    if head is None or cfg.tie_word_embeddings:
        head = weights["model.embed_tokens.weight"]
    return functional.linear(hidden, head)
