"""One rank of the tensor-parallel GPU test (launched by tests/test_gpu_tp.py under torchrun).

Every rank serves the same prompts on its shard of a small Qwen3-8B-like model (TP = world size,
greedy, CUDA graphs); rank 0 then serves them again on the unsplit model (TP = 1, the oracle for
the split: the same seeded weights). Each rank writes its outputs to ``<out>.<rank>.json``.
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
    box = [tp.unique_id(lib_path) if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    plan = tp.shard_plan(cfg, rank, world)
    weights = tp.make_sharded_weights(cfg, plan, seed=0, device=device)
    prompts = pkg.make_prompts(4, cfg.vocab_size, length=48, seed=1)
    result = {"rank": rank, "plan": [plan.q_heads, plan.kv_heads, plan.inter, plan.vocab]}
    model = model_mod.B200Model(tp.rank_config(cfg, plan), weights, num_slots=128 * 16, device=device,
                                max_positions=512, max_rows=512, max_seqs=4,
                                tp=tp.TensorParallel(rank, world, box[0], lib_path), lm_offset=plan.vocab[0])
    result["eager"] = serve(model, prompts, graphs=False)
    result["graphs"] = serve(model, prompts, graphs=True)
    model.close()
    if rank == 0:
        whole_plan = tp.shard_plan(cfg, 0, 1)
        whole = model_mod.B200Model(cfg, tp.make_sharded_weights(cfg, whole_plan, seed=0, device=device),
                                    num_slots=128 * 16, device=device, max_positions=512, max_rows=512, max_seqs=4)
        result["unsplit"] = serve(whole, prompts, graphs=True)
        whole.close()
    Path(f"{args.out}.{rank}.json").write_text(json.dumps(result))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
