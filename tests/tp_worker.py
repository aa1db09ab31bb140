"""One rank of the tensor-parallel GPU test (launched by tests/test_gpu_tp.py under torchrun).

Every rank serves the same prompts on its shard of a small Qwen3-8B-like model (TP = world size,
greedy): with the peer exchange for every call (eagerly and through CUDA graphs), with the
exchange for the steps only (prefill through NCCL), through NCCL only, and with the two-phase
exchange. Then rank 0 prefills
alone on a split model, so that its bounded exchange waits run out. Rank 0 finally serves the
prompts on the unsplit model (TP = 1, the oracle for the split: the same seeded weights, the same
per-projection launch sequence) and scores, where a split output leaves the unsplit one, the
unsplit model's logits at that token. Each rank
writes its outputs to ``<out>.<rank>.json``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))

from tests.conftest import package, submodule  # noqa: E402

SMALL_TP = dict(vocab_size=2048, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                num_attention_heads=8, num_key_value_heads=4, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
                tie_word_embeddings=False)


def serve(model, prompts, graphs: bool):
    eng = submodule("engine").B200SpeculativeEngine(model, k=4, max_ngram=3, max_seqs=4, max_model_len=256,
                                                    num_blocks=96, cuda_graphs=graphs)
    outs = eng.generate(prompts, 32)
    model.raise_on_device_error()
    del eng  # its CUDA graphs hold the model's NCCL calls: release them first
    return outs


class _Scored:
    """A sequence as ``B200ModelRunner.score_tokens`` reads it, over the first blocks of the pool."""

    block_size = 16

    def __init__(self, token_ids: list[int]) -> None:
        self.token_ids, self.num_cached_tokens = token_ids, 0

    def block_table(self, sequence) -> list[int]:
        return list(range(-(-len(self.token_ids) // self.block_size)))


def near_ties(model, prompts, split, unsplit) -> dict[int, list]:
    """For each request whose split outputs leave the unsplit ones: [index i of the first
    difference, the unsplit model's logit of its own token i minus that of the split's token i, its
    top-2 gap], from one scoring pass of the unsplit model over the prompt and tokens 0..i-1."""
    ties = {}
    for r, (a, b) in enumerate(zip(split, unsplit)):
        i = next((j for j, (x, y) in enumerate(zip(a, b)) if x != y), None)
        if i is None:
            continue
        scored = _Scored(list(prompts[r]) + list(b[:i]))
        row = submodule("serial").B200ModelRunner(model, scored).score_tokens(scored, len(scored.token_ids))[-1]
        row = row.float()
        top = torch.topk(row, 2).values
        ties[r] = [i, float(row[b[i]] - row[a[i]]), float(top[0] - top[1])]
    return ties


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    pkg, tp, model_mod = package(), submodule("tp"), submodule("model")
    submodule("build").build()
    cfg = pkg.Qwen3Config(**SMALL_TP)
    lib_path = tp.nccl_library_path()
    plan = tp.shard_plan(cfg, rank, world)
    weights = tp.make_sharded_weights(cfg, plan, seed=0, device=device)
    prompts = pkg.make_prompts(4, cfg.vocab_size, length=48, seed=1)
    result = {"rank": rank, "plan": [plan.q_heads, plan.kv_heads, plan.inter, plan.vocab]}

    def split_model(exchange_rows: int):
        box = [tp.unique_id(lib_path) if rank == 0 else None]  # one NCCL id per communicator
        dist.broadcast_object_list(box, src=0)
        return model_mod.B200Model(tp.rank_config(cfg, plan), weights, num_slots=128 * 16, device=device,
                                   max_positions=512, max_rows=512, max_seqs=4,
                                   tp=tp.TensorParallel(rank, world, box[0], lib_path, exchange_rows=exchange_rows),
                                   lm_offset=plan.vocab[0])

    # peer exchange for every call (prefill of 192 rows and the steps)
    model = split_model(512)
    result["peer_exchange"] = model.peer_exchange
    result["eager"] = serve(model, prompts, graphs=False)
    result["graphs"] = serve(model, prompts, graphs=True)
    model.close()
    # prefill through NCCL (192 rows > 64), steps (20 rows) through the exchange; then NCCL only
    for name, rows in (("mixed", 64), ("nccl", 0)):
        model = split_model(rows)
        result[name] = serve(model, prompts, graphs=True)
        model.close()
    # the two-phase exchange (reduce-scatter in the GEMM, all-gather by the middle launch), which
    # the split uses from eight ranks up, forced on two
    os.environ["NE_TP_TWO_PHASE"] = "1"
    model = split_model(512)
    result["two_phase"] = serve(model, prompts, graphs=True)
    model.close()
    del os.environ["NE_TP_TWO_PHASE"]
    # a rank that stops taking part: rank 0 prefills alone, its bounded waits run out (1 s per
    # exchange) and the device status reports the timeout; rank 1 launches nothing
    model = split_model(512)
    if rank == 0:
        eng = submodule("engine").B200SpeculativeEngine(model, k=4, max_ngram=3, max_seqs=4, max_model_len=256,
                                                        num_blocks=96, cuda_graphs=False)
        slot = eng.add_request(prompts[0], 8, ignore_eos=True)
        try:
            eng.prefill([slot])
            result["lone_rank"] = "no error"
        except Exception as exc:  # NativeError naming the device status
            result["lone_rank"] = str(exc)
        del eng
    model.close()
    if rank == 0:
        whole_plan = tp.shard_plan(cfg, 0, 1)
        whole = model_mod.B200Model(cfg, tp.make_sharded_weights(cfg, whole_plan, seed=0, device=device),
                                    num_slots=128 * 16, device=device, max_positions=512, max_rows=512, max_seqs=4)
        # the unsplit model on the same launch sequence as the split one (the persistent step
        # kernel, opt-in, adds its partials in another order)
        os.environ["NE_STEP_KERNEL"] = "0"
        result["unsplit"] = serve(whole, prompts, graphs=True)
        result["ties"] = near_ties(whole, prompts, result["graphs"], result["unsplit"])
        del os.environ["NE_STEP_KERNEL"]
        whole.close()
    Path(f"{args.out}.{rank}.json").write_text(json.dumps(result))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
