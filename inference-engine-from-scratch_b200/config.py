"""Model shapes and the ``NANOENGINE_*`` settings of the B200 speculative step.

``Qwen3Config`` keeps the field names of the reference (nanoengine/src/nanoengine/models/qwen3.py:13-28).
``SpeculativeSettings`` mirrors the reference's speculation flags
(nanoengine/src/nanoengine/config.py:63-67 plus ``kv_block_size``, ``kv_cache_dtype``, ``quantization``,
``cuda_graphs``, ``max_model_len``, ``max_num_seqs``, ``dtype``, ``device``) with the same
``NANOENGINE_`` environment prefix and value names, and adds two flags:

* ``NANOENGINE_SPECULATIVE_BACKEND`` = ``torch`` (the reference path, default) or ``b200``;
* ``NANOENGINE_TENSOR_PARALLEL_SIZE`` (1 for the data-parallel replicas of Qwen3-0.6B).

The reference rejects speculation with a batched scheduler (config.py:91-97); with the ``b200``
backend speculation runs batched, so that check is relaxed only for this backend.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, fields


@dataclass(frozen=True)
class Qwen3Config:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float
    rope_theta: float
    tie_word_embeddings: bool

    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def shard(self, tp_size: int) -> "Qwen3Config":
        """The per-rank shape under tensor parallelism (heads and MLP columns split)."""
        if tp_size == 1:
            return self
        if self.num_attention_heads % tp_size or self.num_key_value_heads % tp_size:
            raise ValueError(f"heads do not split over tensor_parallel_size={tp_size}")
        if self.intermediate_size % tp_size:
            raise ValueError(f"intermediate_size does not split over {tp_size}")
        return Qwen3Config(
            self.vocab_size,
            self.hidden_size,
            self.intermediate_size // tp_size,
            self.num_hidden_layers,
            self.num_attention_heads // tp_size,
            self.num_key_value_heads // tp_size,
            self.head_dim,
            self.rms_norm_eps,
            self.rope_theta,
            self.tie_word_embeddings,
        )


# BASELINE configs 1-4 (Qwen3-0.6B) and 5b (Qwen3-8B shape, untied head as in the real model).
QWEN3_0_6B = Qwen3Config(151936, 1024, 3072, 28, 16, 8, 128, 1e-6, 1e6, True)
QWEN3_8B_SHAPE = Qwen3Config(151936, 4096, 12288, 36, 32, 8, 128, 1e-6, 1e6, False)
# A small model with the same head_dim for fast parity tests (every GEMM dim tiles by 128).
SMALL_TEST = Qwen3Config(4096, 256, 512, 2, 4, 2, 128, 1e-6, 1e6, True)

SPECULATIVE_NONE = "none"
SPECULATIVE_NGRAM = "ngram"
BACKEND_TORCH = "torch"
BACKEND_B200 = "b200"
ENV_PREFIX = "NANOENGINE_"


@dataclass(frozen=True)
class SpeculativeSettings:
    """The subset of ``EngineSettings`` (config.py:23-102) the speculative step reads."""

    device: str = "cuda"
    dtype: str = "bfloat16"
    max_model_len: int = 4096
    max_num_seqs: int = 64
    kv_cache_memory_mb: int = 1024
    kv_block_size: int = 16
    kv_cache_dtype: str = "auto"
    quantization: str = "none"
    cuda_graphs: bool = True
    speculative: str = SPECULATIVE_NGRAM
    num_speculative_tokens: int = 4
    ngram_max_size: int = 3
    speculative_backend: str = BACKEND_B200
    tensor_parallel_size: int = 1
    scheduler: str = "continuous"

    def __post_init__(self) -> None:
        if self.speculative not in (SPECULATIVE_NONE, SPECULATIVE_NGRAM, "draft"):
            raise ValueError(f"speculative={self.speculative!r}")
        if self.speculative_backend not in (BACKEND_TORCH, BACKEND_B200):
            raise ValueError(f"speculative_backend={self.speculative_backend!r}")
        if self.kv_cache_dtype not in ("auto", "int8") or self.quantization not in ("none", "int8"):
            raise ValueError("kv_cache_dtype must be auto|int8 and quantization none|int8")
        if self.dtype not in ("float32", "float16", "bfloat16"):
            raise ValueError(f"dtype={self.dtype!r}")
        if self.num_speculative_tokens < 1 or self.ngram_max_size < 1 or self.kv_block_size < 1:
            raise ValueError("num_speculative_tokens, ngram_max_size and kv_block_size must be >= 1")
        uses_speculation = self.speculative != SPECULATIVE_NONE
        if uses_speculation and self.speculative_backend == BACKEND_TORCH and self.scheduler != "serial":
            # the reference's own rule (config.py:91-97) still holds for its torch backend
            raise ValueError("speculative decoding needs scheduler=serial, a KV cache and no prefix cache")
        if self.speculative_backend == BACKEND_B200:
            if self.dtype != "bfloat16":
                raise ValueError("the b200 speculative backend computes in bfloat16")
            if self.kv_block_size != 16:
                raise ValueError("the b200 speculative backend uses 16-token KV blocks")

    @property
    def is_int8_kv_cache(self) -> bool:
        return self.kv_cache_dtype == "int8"

    @classmethod
    def from_env(cls, environ=None, **overrides) -> "SpeculativeSettings":
        """Read ``NANOENGINE_<FIELD>`` variables (same names as the reference's settings)."""
        environ = os.environ if environ is None else environ
        values = {}
        for f in fields(cls):
            raw = environ.get(ENV_PREFIX + f.name.upper())
            if raw is None:
                continue
            if f.type in ("int", int):
                values[f.name] = int(raw)
            elif f.type in ("bool", bool):
                values[f.name] = raw.strip().lower() in ("1", "true", "yes", "on")
            else:
                values[f.name] = raw
        values.update(overrides)
        return cls(**values)
