"""Stop tokens end a request inside a speculative step (tests/engine/test_speculative_decoding.py:100-112,
engine/sampling.py:54-62): the emitted tokens stop at the first stop id, the rest of the step's
kept guesses are dropped, and the finish reason is ``stop``.

* ``spec_small_stop_draft.pt`` (the target as its own draft: every guess kept) stops on a kept
  guess in the middle of a step's run; ``spec_small_stop.pt`` (n-gram) stops at a token's first
  appearance. Both greedy, compared with the reference's own runs token for token, through the
  serial seam and through the batched engine (eager and CUDA graphs).
* Sampled: a stop id taken from the GPU's own stop-free run cuts the same run at that token's
  first appearance (serial seam and batched engine).
"""

from __future__ import annotations

import pytest

from tests import reference_seam as seam
from tests.conftest import load_golden, package, submodule

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small():
    submodule("build").build()
    pkg = package()
    cfg = pkg.SMALL_TEST
    weights = pkg.make_weights(cfg, seed=0)
    mk = submodule("model").B200Model

    def make():
        return mk(cfg, weights, num_slots=64 * 16, device="cuda:0", max_positions=512, max_rows=512, max_seqs=8)

    target, draft = make(), make()
    yield cfg, target, draft
    target.close()
    draft.close()


def _proposer(serial, golden, draft_model):
    if golden["proposer"] == "draft":
        return serial.DraftModelProposer(serial.B200ModelRunner(draft_model, seam.PagedSlotAllocator(64, 16)), "cuda:0")
    return serial.NgramProposer(golden["max_ngram"], max_model_len=256, device="cuda:0")


@pytest.mark.parametrize("name", ["spec_small_stop_draft.pt", "spec_small_stop.pt"])
def test_serial_seam_stops_where_the_reference_stops(small, name) -> None:
    _, target, draft = small
    serial = submodule("serial")
    golden = load_golden(name)
    target.kv.zero_()
    allocator = seam.PagedSlotAllocator(golden["num_blocks"], 16)
    runner = serial.B200ModelRunner(target, allocator)
    proposer = _proposer(serial, golden, draft)
    for index, record in enumerate(golden["records"]):
        gen = seam.SpeculativeGenerator(runner, proposer, golden["k"], frozenset(golden["stop_ids"]))
        params = seam.SamplingParams(max_new_tokens=golden["max_new"])
        events = list(gen.generate(seam.GenerationRequest(f"r{index}", record["prompt"], params)))
        assert [e.token_id for e in events] == record["tokens"]
        assert events[-1].finish_reason == record["finish_reason"]
        assert all(not e.is_finished for e in events[:-1])
    assert golden["records"][golden["stop_record"]]["finish_reason"] == "stop"
    assert allocator.num_free_blocks == golden["num_blocks"]
    target.raise_on_device_error()


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("name", ["spec_small_stop_draft.pt", "spec_small_stop.pt"])
def test_batched_engine_stops_where_the_reference_stops(small, name, graphs) -> None:
    _, target, draft = small
    golden = load_golden(name)
    target.kv.zero_()
    draft.kv.zero_()
    kw = dict(draft_model=draft) if golden["proposer"] == "draft" else {}
    eng = submodule("engine").B200SpeculativeEngine(target, k=golden["k"], max_ngram=golden["max_ngram"], max_seqs=1,
                                                    max_model_len=256, num_blocks=64, cuda_graphs=graphs,
                                                    stop_token_ids=golden["stop_ids"], **kw)
    for record in golden["records"]:
        slot = eng.add_request(record["prompt"], golden["max_new"], ignore_eos=False)
        res = eng.prefill([slot])
        tokens = list(res.tokens[slot])
        finish = res.finish[slot]
        while finish is None:
            res = eng.step([slot])
            tokens += res.tokens[slot]
            finish = res.finish[slot]
        assert tokens == record["tokens"]
        assert finish == record["finish_reason"]
        eng.release([slot])
    assert eng.state.num_free_blocks() == 64
    target.raise_on_device_error()


def _first_new(tokens: list[int]) -> int:
    """Index (>= 1) of the first token that did not appear before it in ``tokens``."""
    for i in range(1, len(tokens)):
        if tokens[i] not in tokens[:i]:
            return i
    raise AssertionError("the run repeats its first token throughout")


def test_sampled_serial_run_stops_at_the_first_stop_token(small) -> None:
    cfg, target, draft = small
    serial = submodule("serial")
    prompt = package().make_prompts(1, cfg.vocab_size, length=48, seed=9)[0]

    def run(stop_ids):
        target.kv.zero_()
        allocator = seam.PagedSlotAllocator(64, 16)
        runner = serial.B200ModelRunner(target, allocator)
        proposer = serial.NgramProposer(3, max_model_len=256, device="cuda:0")
        gen = seam.SpeculativeGenerator(runner, proposer, 4, frozenset(stop_ids))
        params = seam.SamplingParams(max_new_tokens=32, temperature=0.8, top_p=0.95, seed=42)
        return list(gen.generate(seam.GenerationRequest("s", prompt, params)))

    free = [e.token_id for e in run(())]
    cut = _first_new(free)
    events = run([free[cut]])
    assert [e.token_id for e in events] == free[: cut + 1]
    assert events[-1].finish_reason == "stop"
    target.raise_on_device_error()


@pytest.mark.parametrize("graphs", [False, True])
def test_sampled_batched_run_stops_at_the_first_stop_token(small, graphs) -> None:
    cfg, target, _ = small
    prompts = package().make_prompts(3, cfg.vocab_size, length=40, seed=21)

    def run(stop_ids):
        target.kv.zero_()
        eng = submodule("engine").B200SpeculativeEngine(target, k=4, max_ngram=3, max_seqs=3, max_model_len=256,
                                                        num_blocks=64, cuda_graphs=graphs, sampling=True,
                                                        stop_token_ids=stop_ids)
        return eng.generate(prompts, 24, ignore_eos=False, temperature=0.8, top_p=0.95, seeds=[5, 6, 7])

    free = run(())
    cut = _first_new(free[1])
    stop = free[1][cut]
    stopped = run([stop])
    for f, s in zip(free, stopped):
        end = f.index(stop) + 1 if stop in f else len(f)
        assert s == f[:end]
    assert stopped[1] == free[1][: cut + 1]
    target.raise_on_device_error()

