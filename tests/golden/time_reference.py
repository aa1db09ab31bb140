"""Time the unmodified reference's serial speculative path beside the oracle port that
``bench.py --impl reference`` runs (the reference's Python sources cannot go to the GPU box, so the
bench's CPU arm is the port; this shows the port is a fair stand-in for the reference's speed).

Both serve config 1's request (Qwen3-0.6B random-init seed 0, fp32, the 64-token motif prompt,
128 greedy outputs, n-gram n=3 k=4, 16-token paged KV) again and again, one at a time, for the
same number of seconds on the same host threads, and report accepted tokens per second. The
reference side is nanoengine's own ``SpeculativeGenerator`` over its ``ModelRunner``,
``KVCachePool``, ``PagedSlotAllocator`` and ``NgramProposer``
(engine/speculative/speculative_generator.py:21-90, the path engine/runtime.py:162-171 builds).

    python tests/golden/time_reference.py [--seconds 20] [--reference-src PATH]
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys
import time
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from tests.conftest import package, reference_src  # noqa: E402

K, NGRAM, PROMPT, MAX_NEW, BLOCKS = 4, 3, 64, 128, 64


def time_reference(src: Path, seconds: float) -> tuple[float, int, int]:
    make_golden = importlib.import_module("make_golden")
    ref = make_golden.Ref(str(src))
    pkg = package()
    cfg = pkg.QWEN3_0_6B
    model = make_golden.build_model(ref, cfg, pkg.make_weights(cfg, seed=0), torch.float32)
    prompt = pkg.make_prompt(cfg.vocab_size, PROMPT, 0, True)
    cpu = torch.device("cpu")
    emitted = requests = 0
    elapsed = 0.0  # generate() only: the runtime builds its pool and runner once, not per request
    warm = True    # the first request warms up and is not counted
    while elapsed < seconds:
        pool = ref.pool.KVCachePool(model.config, BLOCKS * 16, cpu, torch.float32)
        allocator = ref.paged.PagedSlotAllocator(BLOCKS, 16, cpu)
        runner = ref.runner.ModelRunner(model, pool, allocator, cpu)
        gen = ref.specgen.SpeculativeGenerator(runner, ref.proposers.NgramProposer(NGRAM), K, frozenset(), cpu, None)
        request = ref.iface.GenerationRequest(f"t{requests}", list(prompt),
                                              ref.iface.SamplingParams(max_new_tokens=MAX_NEW, ignore_eos=True))
        start = time.perf_counter()
        tokens = sum(1 for _ in gen.generate(request))
        if warm:
            warm = False
            continue
        elapsed += time.perf_counter() - start
        emitted += tokens
        requests += 1
    return emitted / elapsed, emitted, requests


def time_port(seconds: float) -> tuple[float, int, int]:
    bench = importlib.import_module("bench")
    emitted, elapsed, steps = bench.cpu_oracle_run(package(), seconds, warmup_steps=10)
    return emitted / elapsed, emitted, steps


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--seconds", type=float, default=20.0)
    ap.add_argument("--reference-src", default=None)
    args = ap.parse_args()
    src = Path(args.reference_src) if args.reference_src else reference_src()
    if src is None:
        raise SystemExit("the reference's Python sources are not on this host")
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    ref_rate, ref_tokens, ref_requests = time_reference(src, args.seconds)
    port_rate, port_tokens, port_steps = time_port(args.seconds)
    print(json.dumps({"threads": threads, "seconds": args.seconds,
                      "reference": {"tok_s": round(ref_rate, 2), "tokens": ref_tokens, "requests": ref_requests},
                      "port": {"tok_s": round(port_rate, 2), "tokens": port_tokens, "steps": port_steps},
                      "port_over_reference": round(port_rate / ref_rate, 3)}))


if __name__ == "__main__":
    main()
