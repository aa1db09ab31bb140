"""Tensor parallelism for the Qwen3-8B shape: how a model is split over ``world`` GPUs.

One process per GPU. Rank r holds:

* whole KV heads ``[r * nkv/T, (r+1) * nkv/T)`` and the query heads of their groups (q/k/v rows,
  o_proj columns): column-parallel attention, row-parallel o_proj;
* intermediate features ``[r * I/T, (r+1) * I/T)`` (gate/up rows, down_proj columns);
* a contiguous run of whole 128-row tiles of the LM head (the vocabulary split as evenly as the
  1,187 tiles of 151,936 allow); embedding and norms whole.

The row-parallel outputs (o_proj, down_proj) are fp32 partial sums. For steps of up to
``exchange_rows`` rows the GEMM stores them straight into every rank's exchange region over NVLink
and the next RMSNorm launch sums them (``ne_model_tp_exchange_create`` / ``_open`` in
include/nespec.h); larger steps add them with an NCCL all-reduce (``ne_model_set_tp``). Either
way the sum joins the residual stream before the norm, and the argmax keys of the vocabulary
shards are max-reduced. Random-init weights for the big shape are drawn on the GPU one
tensor at a time from a per-tensor seed, so every rank (and an unsplit run) sees the same full
tensors and keeps only its shard.
"""

from __future__ import annotations

import ctypes
import dataclasses
from dataclasses import dataclass

import torch

from . import _lib
from .config import Qwen3Config
from .weights import INIT_STD


@dataclass(frozen=True)
class TensorParallel:
    rank: int
    world: int
    unique_id: bytes  # 128 bytes from ne_tp_unique_id on rank 0, the same on every rank
    nccl_library: str
    # steps of up to this many rows exchange partial rows through peer memory (0: NCCL only);
    # needs torch.distributed initialised (the IPC handles are gathered over it)
    exchange_rows: int = 512


@dataclass(frozen=True)
class ShardPlan:
    rank: int
    world: int
    q_heads: tuple[int, int]    # [begin, end) query heads
    kv_heads: tuple[int, int]   # [begin, end) KV heads
    inter: tuple[int, int]      # [begin, end) intermediate features
    vocab: tuple[int, int]      # [begin, end) LM-head rows


def shard_plan(cfg: Qwen3Config, rank: int, world: int) -> ShardPlan:
    nh, nkv, inter, vocab = (cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size,
                             cfg.vocab_size)
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if nkv % world or nh % world or inter % world:
        raise ValueError(f"{world} ranks do not split {nkv} KV heads, {nh} heads and {inter} features evenly")
    if (inter // world) % 64 or vocab % 128:
        raise ValueError("each rank needs whole 64-feature gate/up groups and whole 128-row vocab tiles")
    kv = nkv // world
    q = nh // world
    f = inter // world
    tiles = vocab // 128
    base, extra = divmod(tiles, world)
    t0 = rank * base + min(rank, extra)
    t1 = t0 + base + (1 if rank < extra else 0)
    return ShardPlan(rank, world, (rank * q, (rank + 1) * q), (rank * kv, (rank + 1) * kv),
                     (rank * f, (rank + 1) * f), (t0 * 128, t1 * 128))


def rank_config(cfg: Qwen3Config, plan: ShardPlan) -> Qwen3Config:
    """The per-rank shape (heads and intermediate features of this rank; vocabulary whole)."""
    return dataclasses.replace(cfg, num_attention_heads=plan.q_heads[1] - plan.q_heads[0],
                               num_key_value_heads=plan.kv_heads[1] - plan.kv_heads[0],
                               intermediate_size=plan.inter[1] - plan.inter[0])


def shard_tensor(name: str, t: torch.Tensor, cfg: Qwen3Config, plan: ShardPlan) -> torch.Tensor:
    """This rank's slice of one full (HF-named) tensor."""
    d = cfg.head_dim
    if name.endswith("self_attn.q_proj.weight"):
        return t[plan.q_heads[0] * d: plan.q_heads[1] * d]
    if name.endswith(("self_attn.k_proj.weight", "self_attn.v_proj.weight")):
        return t[plan.kv_heads[0] * d: plan.kv_heads[1] * d]
    if name.endswith("self_attn.o_proj.weight"):
        return t[:, plan.q_heads[0] * d: plan.q_heads[1] * d]
    if name.endswith(("mlp.gate_proj.weight", "mlp.up_proj.weight")):
        return t[plan.inter[0]: plan.inter[1]]
    if name.endswith("mlp.down_proj.weight"):
        return t[:, plan.inter[0]: plan.inter[1]]
    if name == "lm_head.weight":
        return t[plan.vocab[0]: plan.vocab[1]]
    return t


def shard_weights(weights: dict[str, torch.Tensor], cfg: Qwen3Config, plan: ShardPlan) -> dict[str, torch.Tensor]:
    """A full state dict cut down to this rank (the LM head is untied: tied models repeat the
    embedding as ``lm_head.weight`` first)."""
    full = dict(weights)
    if "lm_head.weight" not in full:
        full["lm_head.weight"] = full["model.embed_tokens.weight"]
    return {name: shard_tensor(name, t, cfg, plan).contiguous() for name, t in full.items()}


def make_sharded_weights(cfg: Qwen3Config, plan: ShardPlan, seed: int, device, dtype=torch.bfloat16,
                         std: float = INIT_STD) -> dict[str, torch.Tensor]:
    """Seeded N(0, std) weights drawn on ``device`` tensor by tensor (tensor i from seed
    ``seed * 100003 + i``), each cut to this rank's shard at once: the same full tensors on every
    rank and at any split, without ever holding the whole model."""
    h, d = cfg.hidden_size, cfg.head_dim
    shapes: list[tuple[str, tuple[int, int] | None]] = [("model.embed_tokens.weight", (cfg.vocab_size, h))]
    for layer in range(cfg.num_hidden_layers):
        p = f"model.layers.{layer}."
        shapes += [
            (p + "self_attn.q_proj.weight", (cfg.num_attention_heads * d, h)),
            (p + "self_attn.k_proj.weight", (cfg.num_key_value_heads * d, h)),
            (p + "self_attn.v_proj.weight", (cfg.num_key_value_heads * d, h)),
            (p + "self_attn.o_proj.weight", (h, cfg.num_attention_heads * d)),
            (p + "mlp.gate_proj.weight", (cfg.intermediate_size, h)),
            (p + "mlp.up_proj.weight", (cfg.intermediate_size, h)),
            (p + "mlp.down_proj.weight", (h, cfg.intermediate_size)),
            (p + "self_attn.q_norm.weight", None), (p + "self_attn.k_norm.weight", None),
            (p + "input_layernorm.weight", None), (p + "post_attention_layernorm.weight", None),
        ]
    shapes += [("model.norm.weight", None), ("lm_head.weight", (cfg.vocab_size, h))]
    out: dict[str, torch.Tensor] = {}
    g = torch.Generator(device=device)
    for i, (name, shape) in enumerate(shapes):
        if shape is None:
            n = d if "q_norm" in name or "k_norm" in name else h
            out[name] = torch.ones(n, dtype=dtype, device=device)
            continue
        g.manual_seed(seed * 100003 + i)
        full = torch.empty(shape, dtype=torch.float32, device=device).normal_(0.0, std, generator=g)
        out[name] = shard_tensor(name, full, cfg, plan).to(dtype).contiguous()
        del full
    return out


def unique_id(nccl_library: str) -> bytes:
    """ne_tp_unique_id (call on rank 0, then hand the bytes to every rank)."""
    lib = _lib.load()
    buf = (ctypes.c_char * 128)()
    _lib.check(lib.ne_tp_unique_id(nccl_library.encode(), buf), "ne_tp_unique_id")
    return bytes(buf)


def nccl_library_path() -> str:
    from .build import nccl_library

    path = nccl_library()
    if path is None:
        raise RuntimeError("no NCCL library found next to PyTorch (nvidia.nccl)")
    return path


def open_exchange(lib, handle, tp: TensorParallel, max_rows: int) -> bool:
    """Create this rank's exchange region, gather every rank's IPC handle over torch.distributed
    and map the peers' regions (collective: every rank calls it with the same ``max_rows``)."""
    import torch.distributed as dist

    rows = min(tp.exchange_rows, max_rows)
    if tp.world < 2 or rows <= 0:
        return False
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() != tp.world:
        raise RuntimeError("the peer exchange gathers IPC handles over torch.distributed: initialise it first")
    buf = (ctypes.c_char * _lib.TP_HANDLE_BYTES)()
    _lib.check(lib.ne_model_tp_exchange_create(handle, rows, buf), "ne_model_tp_exchange_create")
    gathered: list = [None] * tp.world
    dist.all_gather_object(gathered, bytes(buf))
    if dist.get_rank() != tp.rank:
        raise RuntimeError(f"torch.distributed rank {dist.get_rank()} is not the split's rank {tp.rank}")
    joined = b"".join(gathered)
    _lib.check(lib.ne_model_tp_exchange_open(handle, ctypes.create_string_buffer(joined, len(joined))),
               "ne_model_tp_exchange_open")
    return True


def quiesce(device) -> None:
    """Every rank's work on a split model finished (the peers write into this rank's exchange
    region): synchronise, then a barrier. Call before destroying a model with an open exchange."""
    import torch.distributed as dist

    torch.cuda.synchronize(device)
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
