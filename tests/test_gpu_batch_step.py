"""The batch executor (``batch_step``, the part of the nanoengine backend that runs a batch
scheduler's plans) over the real B200 engine.

A small driver plays the reference's ``BatchEngineLoop`` (engine/scheduling/batch_engine_loop.py:
90-150: run the plan, append each token, finish on ``find_finish_reason``, free) with the seam's
``Sequence`` objects; the reference's loop itself runs around the same executor in the CPU tests
(``tests/test_nanoengine_backend.py``). Checked here on the GPU:

* three requests served together stream exactly the reference's recorded serial outputs
  (``spec_small_stop.pt``: two length finishes and a stop-token cut), eager and with CUDA graphs;
* a request preempted mid-run (freed, its cache forgotten, prefilled again from its whole
  history) streams the same tokens;
* a sampled request preempted mid-run resumes its Philox stream where it stopped
  (``draws_used``), and runs with the same preemption stream the same tokens.
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
    model = submodule("model").B200Model(cfg, weights, num_slots=64 * 16, device="cuda:0", max_positions=512,
                                         max_rows=512, max_seqs=8)
    yield cfg, model
    model.close()


class Plan:
    def __init__(self, sequences, is_prefill: bool) -> None:
        self.sequences, self.is_prefill, self.prefill_chunks = sequences, is_prefill, []


def drive(executor, sequences, stop_ids, preempt_at: dict[str, int] | None = None):
    """Prefill every sequence, then step the running ones until all finish; ``preempt_at``: free a
    request after that many decode steps and load it again at the next step."""
    preempt_at = dict(preempt_at or {})
    events = {s.request_id: [] for s in sequences}
    running, waiting, steps = [], list(sequences), 0

    def emit(pairs):
        for seq, token in pairs:
            seq.token_ids.append(token)
            reason = seam.find_finish_reason(token, seq.num_generated_tokens, seq.sampling_params, stop_ids)
            events[seq.request_id].append((token, reason))
            if reason is not None:
                running.remove(seq)
                executor.release(seq)

    while waiting or running:
        if waiting:
            admitted, waiting = waiting, []
            running.extend(admitted)
            emit(executor.execute(Plan(admitted, True)))
            continue
        emit(executor.execute(Plan(list(running), False)))
        steps += 1
        for seq in list(running):
            if preempt_at.get(seq.request_id) == steps:
                del preempt_at[seq.request_id]
                running.remove(seq)
                executor.release(seq)
                seq.forget_cache()
                waiting.append(seq)
    return events


def sequences_of(golden):
    return [seam.Sequence.from_request(seam.GenerationRequest(
        f"r{i}", list(r["prompt"]), seam.SamplingParams(max_new_tokens=golden["max_new"])))
        for i, r in enumerate(golden["records"])]


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("preempt", [False, True])
def test_executor_streams_the_reference_outputs(small, graphs, preempt) -> None:
    _, model = small
    golden = load_golden("spec_small_stop.pt")
    stop_ids = frozenset(golden["stop_ids"]) if isinstance(golden["stop_ids"], (list, tuple)) \
        else frozenset([golden["stop_ids"]])
    model.kv.zero_()
    eng = submodule("engine").B200SpeculativeEngine(model, k=golden["k"], max_ngram=golden["max_ngram"], max_seqs=4,
                                                    max_model_len=256, num_blocks=64, cuda_graphs=graphs,
                                                    stop_token_ids=tuple(stop_ids))
    executor = submodule("batch_step").SpeculativeBatchExecutor(eng, stop_ids)
    events = drive(executor, sequences_of(golden), stop_ids, {"r0": 2, "r2": 1} if preempt else None)
    for i, record in enumerate(golden["records"]):
        got = events[f"r{i}"]
        assert [t for t, _ in got] == record["tokens"]
        assert got[-1][1] == record["finish_reason"]
        assert all(reason is None for _, reason in got[:-1])
    assert executor.num_active == 0
    assert eng.state.num_free_blocks() == 64
    model.raise_on_device_error()


def test_sampled_request_resumes_its_stream_after_preemption(small) -> None:
    """A preempted sampled request keeps the count of uniforms it drew and resumes its Philox
    stream there (no uniform is used twice); runs with the same preemption are reproducible."""
    cfg, model = small
    prompts = package().make_prompts(2, cfg.vocab_size, length=40, seed=33)

    def make():
        model.kv.zero_()
        eng = submodule("engine").B200SpeculativeEngine(model, k=4, max_ngram=3, max_seqs=4, max_model_len=256,
                                                        num_blocks=64, cuda_graphs=False, sampling=True)
        seqs = [seam.Sequence.from_request(seam.GenerationRequest(
            f"s{i}", list(p), seam.SamplingParams(max_new_tokens=32, temperature=0.8, top_p=0.95, seed=100 + i)))
            for i, p in enumerate(prompts)]
        return eng, submodule("batch_step").SpeculativeBatchExecutor(eng), seqs

    def run():
        eng, executor, seqs = make()
        events = drive(executor, seqs, frozenset(), {"s1": 3})
        assert executor.num_active == 0 and eng.state.num_free_blocks() == 64
        return [[t for t, _ in events[f"s{i}"]] for i in range(len(prompts))]

    first = run()
    assert run() == first
    assert all(len(t) == 32 for t in first)

    eng, executor, seqs = make()
    seq = seqs[1]
    for token in [t for _, t in executor.prefill([seq])]:
        seq.token_ids.append(token)
    for _ in range(3):
        for _, token in executor.step([seq]):
            seq.token_ids.append(token)
    drawn = eng.draws_used(executor.slot_of(seq))
    assert drawn > 0
    executor.release(seq)
    seq.forget_cache()
    executor.prefill([seq])
    assert eng.draws_used(executor.slot_of(seq)) >= drawn
    executor.release(seq)
    model.raise_on_device_error()


def test_executor_serves_draft_model_drafts() -> None:
    """speculative=draft through the executor: the engine with a one-layer draft model (its own KV
    pool) serves the reference's recorded runs (``spec_small_draft_bf16.pt``), with a preemption."""
    submodule("build").build()
    pkg = package()
    cfg = pkg.SMALL_TEST
    dcfg = pkg.Qwen3Config(**{**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__}, "num_hidden_layers": 1})
    mk = submodule("model").B200Model
    target = mk(cfg, pkg.make_weights(cfg, seed=0), num_slots=64 * 16, device="cuda:0", max_positions=512,
                max_rows=512, max_seqs=8)
    draft = mk(dcfg, pkg.make_weights(dcfg, seed=1), num_slots=64 * 16, device="cuda:0", max_positions=512,
               max_rows=512, max_seqs=8)
    try:
        golden = load_golden("spec_small_draft_bf16.pt")
        eng = submodule("engine").B200SpeculativeEngine(target, k=golden["k"], max_ngram=golden["max_ngram"],
                                                        max_seqs=4, max_model_len=256, num_blocks=64,
                                                        cuda_graphs=True, draft_model=draft, draft_num_blocks=64)
        executor = submodule("batch_step").SpeculativeBatchExecutor(eng)
        events = drive(executor, sequences_of(golden), frozenset(), {"r1": 2})
        for i, record in enumerate(golden["records"]):
            assert [t for t, _ in events[f"r{i}"]] == record["tokens"]
        assert executor.num_active == 0 and eng.state.num_free_blocks() == 64
        target.raise_on_device_error()
        draft.raise_on_device_error()
    finally:
        target.close()
        draft.close()
