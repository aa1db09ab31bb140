"""Generate the golden fixtures in this directory by running the REAL reference on the CPU.

Usage (build container only -- the reference is not present on the GPU box):

    python tests/golden/make_golden.py --reference <reference checkout>/nanoengine/src [--skip-full]

The reference (``ak7270090/inference-engine-from-scratch``, nanoengine) is pure Python; it is
imported unmodified. Its random draws (``torch.rand`` inside ``verify_proposal`` and
``torch.multinomial`` inside ``sample_from_probabilities``) are replaced by an injected uniform
stream (Philox4x32-10 per request, ``oracle/philox.py``) so that sampled acceptance decisions are
reproducible by the CUDA path; every other line runs as shipped.

Fixtures written (all small):

* ``ngram_cases.json``       NgramProposer.propose on known answers and seeded random histories
* ``verify_cases.pt``        verify_proposal (greedy and T/top-p sampled) with injected uniforms
* ``top_p_cases.pt``         compute_token_probabilities (softmax + apply_top_p)
* ``quant_cases.pt``         quantize_vectors
* ``spec_small_<mode>.pt``   serial speculative runs of a small d=128 Qwen3 (fp32, bf16, int8,
                             sampled): per step draft, block table, logits digest, new tokens
* ``spec_small_draft_bf16.pt`` / ``spec_small_draft_same_bf16.pt``
                             the same with DraftModelProposer drafts: a one-layer draft (seed 1),
                             and the target itself as its own draft (every guess accepted)
* ``spec_small_draft_sampled.pt``  the one-layer draft, sampled (T=0.8, top-p 0.95): drafts drawn
                             from the draft's distribution on the request's stream, verified
                             against it (rejection sampling with the draft's rows)
* ``spec_config1_fp32.pt``   BASELINE config 1 exactly (Qwen3-0.6B fp32, seed 0, 64-token motif
                             prompt, 128 greedy tokens, n=3, k=4, 16-token blocks)
* ``spec_full_bf16.pt``      the benchmarked shape: Qwen3-0.6B (28 layers, vocab 151,936) in bf16,
                             config 1's prompt and two config-2 short_chat prompts, 40 greedy
                             tokens each, n=3, k=4
* ``spec_full_int8.pt``      the same model with int8 weights and int8 KV (config 3's arithmetic),
                             k=8
* ``spec_small_stop_draft.pt`` / ``spec_small_stop.pt`` / ``spec_small_stop_sampled.pt``
                             stop tokens (tests/engine/test_speculative_decoding.py:100-112): with
                             the target as its own draft the stop id is a token the stop-free run
                             emits as a KEPT GUESS in the middle of one step's accepted run, so
                             the step must be cut there; the n-gram runs (greedy, sampled) stop
                             at a token's first appearance
"""

from __future__ import annotations

import argparse
import importlib
import json
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.dont_write_bytecode = True
sys.path.insert(0, str(REPO))

DIGEST_IDS = 128  # logits kept per row at fixed vocab ids (plus argmax / top-2)


def digest_ids(vocab: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(1234)
    return torch.randperm(vocab, generator=g)[:DIGEST_IDS].sort().values


def digest(logits: torch.Tensor, ids: torch.Tensor) -> dict:
    """Per row: argmax (lowest index on ties), top-2 values, logits at ``ids``."""
    f = logits.float()
    top2 = torch.topk(f, 2, dim=-1).values
    return {
        "argmax": torch.argmax(logits, dim=-1).to(torch.int32),
        "top2": top2,
        "at_ids": f[:, ids],
    }


class UniformInjector:
    """Routes the reference's random draws to the current request's Philox stream."""

    def __init__(self, ref) -> None:
        from oracle import philox, verify

        self.philox = philox
        self.verify = verify
        self.stream = None
        self.count = 0
        self.ref = ref
        real_torch = torch

        injector = self

        class TorchProxy:
            def __getattr__(self, name):
                return getattr(real_torch, name)

            @staticmethod
            def rand(*args, **kwargs):
                injector.count += 1
                return real_torch.tensor(next(injector.stream), dtype=real_torch.float32)

        def sample(probabilities, generator):
            injector.count += 1
            return verify.inverse_cdf(probabilities, next(injector.stream))

        ref.verifier.torch = TorchProxy()
        ref.verifier.sample_from_probabilities = sample
        ref.sampling.sample_from_probabilities = sample
        ref.proposers.sample_from_probabilities = sample  # DraftModelProposer's sampled drafts

    def start(self, seed: int) -> None:
        self.stream = self.philox.UniformStream(seed)
        self.count = 0


class Ref:
    def __init__(self, src: str) -> None:
        sys.path.insert(0, src)
        self.qwen3 = importlib.import_module("nanoengine.models.qwen3")
        self.int8 = importlib.import_module("nanoengine.models.int8_quantization")
        self.pool = importlib.import_module("nanoengine.engine.memory.kv_cache_pool")
        self.paged = importlib.import_module("nanoengine.engine.memory.paged_allocator")
        self.runner = importlib.import_module("nanoengine.engine.generation.model_runner")
        self.iface = importlib.import_module("nanoengine.engine.interface")
        self.seq = importlib.import_module("nanoengine.engine.sequence_state")
        self.proposers = importlib.import_module("nanoengine.engine.speculative.proposers")
        self.verifier = importlib.import_module("nanoengine.engine.speculative.verifier")
        self.specgen = importlib.import_module("nanoengine.engine.speculative.speculative_generator")
        self.sampling = importlib.import_module("nanoengine.engine.sampling")
        self.metrics = importlib.import_module("nanoengine.engine.metrics")


def build_model(ref: Ref, cfg, weights, dtype):
    rcfg = ref.qwen3.Qwen3Config(**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__})
    model = ref.qwen3.Qwen3ForCausalLM(rcfg)
    model.load_state_dict({k: v.to(dtype) for k, v in weights.items()}, strict=True)
    return model.to(dtype).eval().requires_grad_(False)


def ngram_cases(ref: Ref) -> list[dict]:
    cases = []

    def run(history, k, max_ngram):
        seq = ref.seq.Sequence.from_request(
            ref.iface.GenerationRequest("n", list(history), ref.iface.SamplingParams(max_new_tokens=8)),
            torch.device("cpu"),
        )
        out = ref.proposers.NgramProposer(max_ngram).propose(seq, k).token_ids
        cases.append({"history": list(history), "k": k, "max_ngram": max_ngram, "expected": out})

    run([1, 2, 3, 4, 5, 9, 1, 2], 3, 2)  # tests/engine/test_speculative_decoding.py:35-42
    run([1, 2, 3, 4], 3, 2)
    run([7], 4, 3)
    run([7, 7], 4, 3)
    run([5, 5, 5, 5, 5], 4, 3)
    g = torch.Generator().manual_seed(99)
    for i in range(300):
        length = int(torch.randint(1, 200, (1,), generator=g))
        vocab = int(torch.randint(2, 12, (1,), generator=g)) if i % 3 else 151936
        history = torch.randint(0, vocab, (length,), generator=g).tolist()
        k = int(torch.randint(1, 9, (1,), generator=g))
        n = int(torch.randint(1, 5, (1,), generator=g))
        run(history, k, n)
    return cases


def verify_cases(ref: Ref, inj: UniformInjector) -> dict:
    params = ref.iface.SamplingParams
    out = []
    # tests/engine/test_speculative_decoding.py:45-55 known answer
    logits = torch.full((4, 6), -10.0)
    for row, best in enumerate([2, 4, 1, 5]):
        logits[row, best] = 10.0
    for guesses in ([2, 4, 1], [2, 3, 1]):
        inj.start(0)
        got = ref.verifier.verify_proposal(
            ref.proposers.Proposal(guesses), logits, params(max_new_tokens=8), torch.Generator()
        )
        out.append({"logits": logits.clone(), "guesses": guesses, "temperature": 0.0, "top_p": 1.0,
                    "seed": 0, "expected": got, "draws": inj.count})
    g = torch.Generator().manual_seed(5)
    for i in range(192):
        vocab = [7, 64, 1000, 2048][i % 4]
        k = int(torch.randint(0, 9, (1,), generator=g))
        temperature = [0.0, 0.8, 1.0, 0.3][(i // 4) % 4]
        top_p = [1.0, 0.95, 0.5][(i // 16) % 3]
        scale = [1.0, 4.0, 12.0][(i // 48) % 3]
        logits = torch.randn(k + 1, vocab, generator=g) * scale
        if i % 5 == 0:
            logits = logits.to(torch.bfloat16)
        best = torch.argmax(logits.float(), dim=-1)
        guesses = []
        for j in range(k):  # mostly the target's favourite so that several guesses survive
            r = float(torch.rand((), generator=g))
            guesses.append(int(best[j]) if r < 0.6 else int(torch.randint(0, vocab, (1,), generator=g)))
        seed = 1000 + i
        inj.start(seed)
        got = ref.verifier.verify_proposal(
            ref.proposers.Proposal(guesses), logits,
            params(max_new_tokens=64, temperature=temperature, top_p=top_p), torch.Generator(),
        )
        out.append({"logits": logits, "guesses": guesses, "temperature": temperature, "top_p": top_p,
                    "seed": seed, "expected": got, "draws": inj.count})
    return {"cases": out}


def top_p_cases(ref: Ref) -> dict:
    g = torch.Generator().manual_seed(11)
    cases = []
    for i in range(40):
        vocab = [5, 100, 1000, 4096][i % 4]
        logits = torch.randn(3, vocab, generator=g) * [0.5, 3.0, 10.0][i % 3]
        temperature = [0.8, 1.0][i % 2]
        top_p = [0.95, 0.5, 0.99, 1.0][(i // 2) % 4]
        params = ref.iface.SamplingParams(max_new_tokens=8, temperature=temperature, top_p=top_p)
        probs = ref.sampling.compute_token_probabilities(logits, params)
        cases.append({"logits": logits, "temperature": temperature, "top_p": top_p,
                      "kept": (probs > 0), "probs": probs})
    return {"cases": cases}


def quant_cases(ref: Ref) -> dict:
    g = torch.Generator().manual_seed(3)
    cases = []
    for dtype in (torch.float32, torch.bfloat16):
        values = (torch.randn(6, 8, 128, generator=g) * 3).to(dtype)
        values[0, 0] = 0  # an all-zero vector hits the MIN_SCALE clamp
        q, s = ref.int8.quantize_vectors(values)
        cases.append({"values": values, "quantized": q, "scales": s})
    return {"cases": cases}


def spec_run(ref: Ref, inj: UniformInjector, cfg, weights, dtype, prompts, *, max_new, k, max_ngram,
             num_blocks, int8=False, temperature=0.0, top_p=1.0, seeds=None, stop_ids=frozenset(), draft=None):
    """``draft`` = (config, weights): DraftModelProposer over that model (its own paged cache of
    ``num_blocks`` blocks) instead of NgramProposer; the draft's top-2 logits per guess are kept."""
    model = build_model(ref, cfg, weights, dtype)
    if int8:
        ref.int8.quantize_linear_layers(model)
    cpu = torch.device("cpu")
    pool = ref.pool.KVCachePool(model.config, num_blocks * 16, cpu, dtype, is_int8_cache=int8)
    allocator = ref.paged.PagedSlotAllocator(num_blocks, 16, cpu)
    ids = digest_ids(cfg.vocab_size)
    records: list[dict] = []
    current: dict = {}

    class RecordingRunner(ref.runner.ModelRunner):
        def run_step(self, sequences, token_counts=None):
            current["prefill_table"] = allocator.block_table(sequences[0])
            return super().run_step(sequences, token_counts)

        def _sample(self, logits, sequences):  # the prefill's last-row logits (the first token's row)
            current["prefill_logits"] = digest(logits, ids)
            return super()._sample(logits, sequences)

        def score_tokens(self, sequence, token_count):
            table = allocator.block_table(sequence)
            logits = super().score_tokens(sequence, token_count)
            current["steps"].append({"block_table": table, "logits": digest(logits, ids),
                                     "draft": list(sequence.token_ids[len(sequence.token_ids) - token_count + 1:])})
            return logits

    runner = RecordingRunner(model, pool, allocator, cpu)
    real_verify = ref.specgen.verify_proposal

    def recording_verify(proposal, logits, params, generator):
        before = inj.count
        got = real_verify(proposal, logits, params, generator)
        current["steps"][-1]["new_tokens"] = list(got)
        current["steps"][-1]["draws"] = inj.count - before
        return got

    ref.specgen.verify_proposal = recording_verify
    metrics = ref.metrics.EngineMetrics()
    if draft is None:
        proposer = ref.proposers.NgramProposer(max_ngram)
    else:
        draft_cfg, draft_weights = draft
        draft_model = build_model(ref, draft_cfg, draft_weights, dtype)
        draft_pool = ref.pool.KVCachePool(draft_model.config, num_blocks * 16, cpu, dtype)
        draft_allocator = ref.paged.PagedSlotAllocator(num_blocks, 16, cpu)
        pending_top2: list = []

        class DraftRecordingRunner(ref.runner.ModelRunner):
            def score_tokens(self, sequence, token_count):
                logits = super().score_tokens(sequence, token_count)
                pending_top2.append(torch.topk(logits[-1].float(), 2).values)
                return logits

        proposer = ref.proposers.DraftModelProposer(
            DraftRecordingRunner(draft_model, draft_pool, draft_allocator, cpu), cpu)
        real_score = RecordingRunner.score_tokens

        def score_with_draft_record(self, sequence, token_count):
            logits = real_score(self, sequence, token_count)
            current["steps"][-1]["draft_top2"] = torch.stack(pending_top2) if pending_top2 else torch.empty(0, 2)
            pending_top2.clear()
            return logits

        RecordingRunner.score_tokens = score_with_draft_record
    gen = ref.specgen.SpeculativeGenerator(runner, proposer, k, stop_ids, cpu, metrics)
    try:
        for index, prompt in enumerate(prompts):
            seed = None if seeds is None else seeds[index]
            inj.start(0 if seed is None else seed)
            current.clear()
            current["steps"] = []
            params = ref.iface.SamplingParams(max_new_tokens=max_new, temperature=temperature,
                                              top_p=top_p, seed=seed, ignore_eos=not stop_ids)
            request = ref.iface.GenerationRequest(f"r{index}", list(prompt), params)
            events = list(gen.generate(request))
            records.append({
                "prompt": list(prompt),
                "tokens": [e.token_id for e in events],
                "finish_reason": events[-1].finish_reason,
                "prefill_block_table": current["prefill_table"],
                "prefill_logits": current.get("prefill_logits"),
                "steps": current["steps"],
                "seed": seed,
                "free_blocks_after": allocator.num_free_blocks,
            })
    finally:
        ref.specgen.verify_proposal = real_verify
    proposed = metrics.registry.get_sample_value("nanoengine_speculative_proposed_tokens_total")
    accepted = metrics.registry.get_sample_value("nanoengine_speculative_accepted_tokens_total")
    return {"records": records, "digest_ids": ids, "proposed": proposed, "accepted": accepted,
            "k": k, "max_ngram": max_ngram, "max_new": max_new, "num_blocks": num_blocks,
            "temperature": temperature, "top_p": top_p, "int8": int8, "dtype": str(dtype),
            "proposer": "ngram" if draft is None else "draft"}


def pick_stop_token(run: dict, mid_run: bool) -> tuple[int, int] | None:
    """(record index, token) such that the token first appears in that record's output at a step
    after the prefill, with ``mid_run`` as a kept guess that has more tokens after it in the same
    step (the step must be cut), else anywhere in a step's tokens."""
    for index, record in enumerate(run["records"]):
        seen = set(record["tokens"][:1])  # the prefill's first token
        for step in record["steps"]:
            new = step["new_tokens"]
            for j, token in enumerate(new):
                if token not in seen and (not mid_run or j < len(new) - 1):
                    return index, token
                seen.add(token)
    return None


def stop_fixtures(ref: Ref, inj: UniformInjector, pkg) -> None:
    """Random-init greedy output collapses to one repeated token, so an n-gram guess is kept only
    once that token has appeared already: a mid-run cut needs guesses the target keeps while its
    output still changes, which a draft model equal to the target gives (every guess kept). The
    n-gram runs stop at a token's first appearance wherever it falls in its step."""
    cfg = pkg.SMALL_TEST
    weights = pkg.make_weights(cfg, seed=0)
    prompts = [pkg.make_prompt(cfg.vocab_size, 48, 0, True), pkg.make_prompt(cfg.vocab_size, 40, 1, False),
               pkg.make_prompt(cfg.vocab_size, 33, 2, True)]
    common = dict(max_new=40, k=4, max_ngram=3, num_blocks=64)
    cases = (("spec_small_stop_draft.pt", True, dict(draft=(cfg, weights))),
             ("spec_small_stop.pt", False, {}),
             ("spec_small_stop_sampled.pt", False, dict(temperature=0.8, top_p=0.95, seeds=[11, 12, 13])))
    for name, mid_run, extra in cases:
        free = spec_run(ref, inj, cfg, weights, torch.bfloat16, prompts, **common, **extra)
        pick = pick_stop_token(free, mid_run)
        if pick is None:
            raise RuntimeError(f"{name}: no token to stop on")
        index, token = pick
        run = spec_run(ref, inj, cfg, weights, torch.bfloat16, prompts, stop_ids=frozenset({token}), **common, **extra)
        assert run["records"][index]["finish_reason"] == "stop", run["records"][index]["finish_reason"]
        run["stop_ids"] = [token]
        run["stop_record"] = index
        torch.save(run, HERE / name)
        print(name, "stop", token, "record", index, "tokens", run["records"][index]["tokens"][:12], flush=True)


def full_fixtures(ref: Ref, inj: UniformInjector, pkg) -> None:
    full = pkg.QWEN3_0_6B
    weights = pkg.make_weights(full, seed=0)
    short_chat = pkg.make_prompts(3, full.vocab_size, 64, seed=0)  # user 0 is config 1's prompt
    torch.save(spec_run(ref, inj, full, weights, torch.bfloat16, short_chat, max_new=40, k=4, max_ngram=3,
                        num_blocks=32), HERE / "spec_full_bf16.pt")
    torch.save(spec_run(ref, inj, full, weights, torch.bfloat16, short_chat, max_new=40, k=8, max_ngram=3,
                        num_blocks=32, int8=True), HERE / "spec_full_int8.pt")


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="the reference's nanoengine/src directory")
    parser.add_argument("--skip-full", action="store_true", help="skip the Qwen3-0.6B config-1 run")
    parser.add_argument("--only-draft", action="store_true", help="write only the draft-model fixtures")
    parser.add_argument("--only", choices=("stop", "full"), help="write only the stop-token or full-shape fixtures")
    args = parser.parse_args()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref = Ref(args.reference)
    inj = UniformInjector(ref)
    pkg = importlib.import_module("inference-engine-from-scratch_b200")
    if args.only == "stop":
        stop_fixtures(ref, inj, pkg)
        return
    if args.only == "full":
        full_fixtures(ref, inj, pkg)
        return

    cfg = pkg.SMALL_TEST
    weights = pkg.make_weights(cfg, seed=0)
    prompts = [pkg.make_prompt(cfg.vocab_size, 48, 0, True), pkg.make_prompt(cfg.vocab_size, 40, 1, False),
               pkg.make_prompt(cfg.vocab_size, 33, 2, True)]
    common = dict(max_new=40, k=4, max_ngram=3, num_blocks=64)
    # DraftModelProposer: a one-layer draft of the same family (seed 1), and the target itself
    draft_cfg = pkg.Qwen3Config(**{**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__}, "num_hidden_layers": 1})
    torch.save(spec_run(ref, inj, cfg, weights, torch.bfloat16, prompts,
                        draft=(draft_cfg, pkg.make_weights(draft_cfg, seed=1)), **common),
               HERE / "spec_small_draft_bf16.pt")
    torch.save(spec_run(ref, inj, cfg, weights, torch.bfloat16, prompts, draft=(cfg, weights), **common),
               HERE / "spec_small_draft_same_bf16.pt")
    torch.save(spec_run(ref, inj, cfg, weights, torch.bfloat16, prompts, temperature=0.8, top_p=0.95,
                        seeds=[11, 12, 13], draft=(draft_cfg, pkg.make_weights(draft_cfg, seed=1)), **common),
               HERE / "spec_small_draft_sampled.pt")
    if args.only_draft:
        return

    (HERE / "ngram_cases.json").write_text(json.dumps(ngram_cases(ref)))
    torch.save(verify_cases(ref, inj), HERE / "verify_cases.pt")
    torch.save(top_p_cases(ref), HERE / "top_p_cases.pt")
    torch.save(quant_cases(ref), HERE / "quant_cases.pt")

    torch.save(spec_run(ref, inj, cfg, weights, torch.float32, prompts, **common), HERE / "spec_small_fp32.pt")
    torch.save(spec_run(ref, inj, cfg, weights, torch.bfloat16, prompts, **common), HERE / "spec_small_bf16.pt")
    torch.save(spec_run(ref, inj, cfg, weights, torch.bfloat16, prompts, int8=True, **common),
               HERE / "spec_small_int8.pt")
    torch.save(spec_run(ref, inj, cfg, weights, torch.bfloat16, prompts, temperature=0.8, top_p=0.95,
                        seeds=[11, 12, 13], **common), HERE / "spec_small_sampled.pt")
    if not args.skip_full:
        full = pkg.QWEN3_0_6B
        weights = pkg.make_weights(full, seed=0)
        prompt = pkg.make_prompt(full.vocab_size, 64, 0, True)
        torch.save(spec_run(ref, inj, full, weights, torch.float32, [prompt], max_new=128, k=4,
                            max_ngram=3, num_blocks=64), HERE / "spec_config1_fp32.pt")
        full_fixtures(ref, inj, pkg)
    stop_fixtures(ref, inj, pkg)


if __name__ == "__main__":
    main()
