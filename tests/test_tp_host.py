"""Host-side logic of tensor parallelism (no GPU): the shard plan, weight sharding and the rank
handshake over a world-size-2 gloo process group."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.conftest import package, submodule


def _tp():
    return submodule("tp")


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_plan_partitions_the_8b_shape(world) -> None:
    tp = _tp()
    cfg = package().QWEN3_8B_SHAPE
    plans = [tp.shard_plan(cfg, r, world) for r in range(world)]
    for field, total in (("q_heads", cfg.num_attention_heads), ("kv_heads", cfg.num_key_value_heads),
                         ("inter", cfg.intermediate_size), ("vocab", cfg.vocab_size)):
        spans = [getattr(p, field) for p in plans]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    for p in plans:
        assert (p.vocab[1] - p.vocab[0]) % 128 == 0 and (p.inter[1] - p.inter[0]) % 64 == 0
        # whole GQA groups: the rank's query heads are exactly the groups of its KV heads
        group = cfg.num_attention_heads // cfg.num_key_value_heads
        assert p.q_heads == (p.kv_heads[0] * group, p.kv_heads[1] * group)
    sizes = [p.vocab[1] - p.vocab[0] for p in plans]
    assert max(sizes) - min(sizes) <= 128


def test_shard_plan_rejects_uneven_splits() -> None:
    tp = _tp()
    with pytest.raises(ValueError):
        tp.shard_plan(package().QWEN3_8B_SHAPE, 0, 3)


SMALL_TP = dict(vocab_size=2048, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                num_attention_heads=8, num_key_value_heads=4, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
                tie_word_embeddings=False)


def _small_cfg():
    return package().Qwen3Config(**SMALL_TP)


def test_shards_reassemble_the_full_weights() -> None:
    tp = _tp()
    cfg = _small_cfg()
    full = package().make_weights(cfg, seed=0)
    shards = [tp.shard_weights(full, cfg, tp.shard_plan(cfg, r, 2)) for r in range(2)]
    for name, t in full.items():
        parts = [s[name] for s in shards]
        if name.endswith(("o_proj.weight", "down_proj.weight")):
            assert torch.equal(torch.cat(parts, dim=1), t)
        elif name.endswith(("q_proj.weight", "k_proj.weight", "v_proj.weight", "gate_proj.weight",
                            "up_proj.weight")) or name == "lm_head.weight":
            assert torch.equal(torch.cat(parts, dim=0), t)
        else:
            assert all(torch.equal(p, t) for p in parts)


def test_sharded_init_is_the_unsplit_init_cut_up() -> None:
    tp = _tp()
    cfg = _small_cfg()
    whole = tp.make_sharded_weights(cfg, tp.shard_plan(cfg, 0, 1), seed=3, device="cpu", dtype=torch.float32)
    shards = [tp.make_sharded_weights(cfg, tp.shard_plan(cfg, r, 2), seed=3, device="cpu", dtype=torch.float32)
              for r in range(2)]
    expected = [tp.shard_weights(whole, cfg, tp.shard_plan(cfg, r, 2)) for r in range(2)]
    for got, want in zip(shards, expected):
        assert got.keys() == want.keys()
        assert all(torch.equal(got[k], want[k]) for k in got)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _handshake(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    tp = _tp()
    cfg = package().QWEN3_8B_SHAPE
    # rank 0 makes the id (random bytes stand in for ncclGetUniqueId on a CPU host), everyone gets it
    box = [os.urandom(128) if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    plan = tp.shard_plan(cfg, rank, world)
    gathered = [None] * world
    dist.all_gather_object(gathered, (box[0], plan))
    out[rank] = gathered
    dist.destroy_process_group()


def test_rank_handshake_over_gloo() -> None:
    world = 2
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_handshake, args=(world, _free_port(), out), nprocs=world, join=True)
    ids = {g[0] for r in range(world) for g in out[r]}
    assert len(ids) == 1 and len(next(iter(ids))) == 128
    plans = [g[1] for g in out[0]]
    assert [p.rank for p in plans] == [0, 1]
    assert plans[0].kv_heads[1] == plans[1].kv_heads[0] and plans[0].vocab[1] == plans[1].vocab[0]
