"""The batched speculative step under nanoengine's own batch scheduler and engine loop (CPU).

The reference's ``BatchEngineLoop`` and ``ContinuousBatchScheduler`` run unchanged around the
B200 batch executor (``nanoengine_backend``); the engine underneath is the CPU stand-in
(``tests/oracle_engine.py``, the oracle handing out its steps as the engine would), so these tests
check the binding: admission, the guess-room KV account, preemption and reload, streaming of
several tokens per step, stop-token and length finishes, frees and metrics. Every request must
stream exactly what the reference's own serial ``SpeculativeGenerator`` emits for it.

Skipped where the reference's sources are absent (GPU hosts); the GPU test of the executor over
the real engine is ``tests/test_gpu_batch_step.py``.
"""

from __future__ import annotations

import asyncio
import importlib
import sys

import pytest
import torch

from tests.conftest import REPO, package, reference_src, submodule
from tests.oracle_engine import OracleSpecEngine

K, NGRAM, MAX_NEW, PROMPT = 4, 3, 24, 112


@pytest.fixture(scope="module")
def ref():
    src = reference_src()
    if src is None:
        pytest.skip("the reference's sources are not present on this host")
    sys.path.insert(0, str(REPO / "tests" / "golden"))
    try:
        make_golden = importlib.import_module("make_golden")
    finally:
        sys.path.remove(str(REPO / "tests" / "golden"))
    ref_mod = make_golden.Ref(str(src))
    return make_golden, ref_mod, submodule("nanoengine_backend")


@pytest.fixture(scope="module")
def tiny(ref):
    make_golden, ref_mod, _ = ref
    pkg = package()
    cfg = pkg.SMALL_TEST  # 2 layers: 2,048 KV bytes per bf16 token, so 1 MB of KV is 32 blocks
    weights = pkg.make_weights(cfg, seed=0)
    model = make_golden.build_model(ref_mod, cfg, weights, torch.float32)
    prompts = [pkg.make_prompt(cfg.vocab_size, PROMPT, i, i % 2 == 0) for i in range(4)]
    return cfg, weights, model, prompts


def settings(backend_mod, **overrides):
    values = dict(device="cpu", dtype="bfloat16", scheduler="continuous", kv_cache="paged", speculative="ngram",
                  speculative_backend="b200", num_speculative_tokens=K, ngram_max_size=NGRAM, max_num_seqs=4,
                  kv_cache_memory_mb=1)
    values.update(overrides)
    return backend_mod.B200EngineSettings(**values)


def serial_reference(ref_mod, model, prompts, stop_ids, draft_model=None) -> list[list[tuple[int, bool, str | None]]]:
    """The reference's own serial speculative path, request by request (engine/runtime.py:162-171),
    with n-gram drafts or (``draft_model``) DraftModelProposer drafts."""
    cpu = torch.device("cpu")
    out = []
    for index, prompt in enumerate(prompts):
        pool = ref_mod.pool.KVCachePool(model.config, 64 * 16, cpu, torch.float32)
        allocator = ref_mod.paged.PagedSlotAllocator(64, 16, cpu)
        runner = ref_mod.runner.ModelRunner(model, pool, allocator, cpu)
        proposer = ref_mod.proposers.NgramProposer(NGRAM)
        if draft_model is not None:
            draft_pool = ref_mod.pool.KVCachePool(draft_model.config, 64 * 16, cpu, torch.float32)
            proposer = ref_mod.proposers.DraftModelProposer(
                ref_mod.runner.ModelRunner(draft_model, draft_pool, ref_mod.paged.PagedSlotAllocator(64, 16, cpu), cpu),
                cpu)
        gen = ref_mod.specgen.SpeculativeGenerator(runner, proposer, K, frozenset(stop_ids), cpu, None)
        params = ref_mod.iface.SamplingParams(max_new_tokens=MAX_NEW, ignore_eos=not stop_ids)
        out.append([(e.token_id, e.is_finished, e.finish_reason)
                    for e in gen.generate(ref_mod.iface.GenerationRequest(f"r{index}", list(prompt), params))])
    return out


def serve(backend_mod, ref_mod, model, cfg, weights, prompts, stop_ids, draft=None, **setting_overrides):
    """Every prompt submitted at once to the b200 loop; the events each request streams.
    ``draft``: (config, weights, reference model) of a draft model."""
    s = settings(backend_mod, **setting_overrides)
    metrics = ref_mod.metrics.EngineMetrics()
    fake = OracleSpecEngine(weights, cfg, K, NGRAM, s.max_num_seqs, stop_ids,
                            draft=draft[:2] if draft is not None else None)
    loop = backend_mod.create_b200_engine(model, frozenset(stop_ids), s, metrics,
                                          draft_model=draft[2] if draft is not None else None, engine=fake)

    async def run():
        await loop.start()
        try:
            streams = [loop.submit(ref_mod.iface.GenerationRequest(
                f"r{i}", list(p), ref_mod.iface.SamplingParams(max_new_tokens=MAX_NEW, ignore_eos=not stop_ids)))
                for i, p in enumerate(prompts)]

            async def drain(stream):
                return [(e.token_id, e.is_finished, e.finish_reason) async for e in stream]

            return await asyncio.wait_for(asyncio.gather(*(drain(st) for st in streams)), timeout=120)
        finally:
            await loop.stop()

    events = asyncio.run(run())
    return events, loop, fake, metrics


def metric(metrics, name: str, labels: dict | None = None) -> float:
    return metrics.registry.get_sample_value(name, labels or {}) or 0.0


def test_settings_accept_batched_speculation_only_on_the_b200_backend(ref) -> None:
    _, _, backend = ref
    assert settings(backend).speculative_backend == "b200"
    with pytest.raises(ValueError, match="scheduler=serial"):  # the reference's own rule, torch backend
        settings(backend, speculative_backend="torch")
    with pytest.raises(ValueError, match="no prefix_cache"):
        settings(backend, prefix_cache=True)
    with pytest.raises(ValueError, match="kv_block_size=16"):
        settings(backend, kv_block_size=32)
    with pytest.raises(ValueError, match="needs scheduler=continuous"):
        settings(backend, scheduler="static")
    with pytest.raises(ValueError, match="scheduler=continuous"):  # the reference's rule on chunked prefill
        settings(backend, chunked_prefill=True, scheduler="static")
    # the serial torch path stays the reference's
    assert settings(backend, speculative_backend="torch", scheduler="serial").scheduler == "serial"


def test_settings_read_the_backend_from_the_environment(ref, monkeypatch) -> None:
    _, _, backend = ref
    for name, value in dict(SPECULATIVE_BACKEND="b200", SPECULATIVE="ngram", SCHEDULER="continuous",
                            KV_CACHE="paged", DTYPE="bfloat16", NUM_SPECULATIVE_TOKENS="6").items():
        monkeypatch.setenv("NANOENGINE_" + name, value)
    s = backend.B200EngineSettings()
    assert (s.speculative_backend, s.num_speculative_tokens, s.scheduler) == ("b200", 6, "continuous")


@pytest.mark.parametrize("with_stop", [False, True])
def test_batch_loop_streams_the_reference_serial_outputs(ref, tiny, with_stop) -> None:
    _, ref_mod, backend = ref
    cfg, weights, model, prompts = tiny
    stop_ids: list[int] = []
    if with_stop:
        free = serial_reference(ref_mod, model, prompts[:1], ())
        stop_ids = [free[0][3][0]]
    want = serial_reference(ref_mod, model, prompts, stop_ids)
    # 64 MB of KV: every request fits, nobody is preempted
    got, loop, fake, metrics = serve(backend, ref_mod, model, cfg, weights, prompts, stop_ids,
                                     kv_cache_memory_mb=64)
    assert got == want
    assert metric(metrics, "nanoengine_preemptions_total") == 0
    assert metric(metrics, "nanoengine_generated_tokens_total") == sum(len(e) for e in want)
    assert loop._executor.num_active == 0 and len(fake.free) == fake.max_seqs
    assert loop._runner.allocator.num_free_blocks == backend.num_kv_blocks(model.config, settings(
        backend, kv_cache_memory_mb=64))
    if with_stop:
        assert want[0][-1][2] == "stop"
        assert metric(metrics, "nanoengine_finished_requests_total", {"finish_reason": "stop"}) >= 1
    # several tokens stream from one step, and the speculative counters follow the engine's
    assert metric(metrics, "nanoengine_speculative_accepted_tokens_total") == fake.accepted_total > 0
    assert fake.steps_run < sum(len(e) for e in want)


def test_preempted_requests_resume_with_the_same_outputs(ref, tiny) -> None:
    _, ref_mod, backend = ref
    cfg, weights, model, prompts = tiny
    want = serial_reference(ref_mod, model, prompts, ())
    # 1 MB of KV (32 blocks) admits four 112-token prompts (8 blocks each with the guess room),
    # which cannot all grow to 136 tokens
    got, loop, fake, metrics = serve(backend, ref_mod, model, cfg, weights, prompts, ())
    assert got == want
    assert metric(metrics, "nanoengine_preemptions_total") > 0
    # a preempted request is reloaded with its whole history as the prompt
    assert len(fake.loaded) > len(prompts)
    assert any(len(h) > PROMPT for h in fake.loaded)
    assert loop._runner.allocator.num_free_blocks == 32 and loop._executor.num_active == 0


def test_guess_room_account_covers_every_step(ref) -> None:
    """The host account reserves the step's guess room up front: never fewer blocks than the device
    reserves for the prompt plus the guesses a step can verify (speculative_generator.py:73-77)."""
    _, ref_mod, _ = ref
    batch_step = submodule("batch_step")
    cpu = torch.device("cpu")

    class _Exec:
        k = 4

        def slot_of(self, sequence):
            return None

        def release(self, sequence):
            pass

    inner = ref_mod.paged.PagedSlotAllocator(8, 16, cpu)
    acct = batch_step.GuessRoomAllocator(inner, _Exec())
    seq = ref_mod.seq.Sequence.from_request(ref_mod.iface.GenerationRequest(
        "a", list(range(30)), ref_mod.iface.SamplingParams(max_new_tokens=10)), cpu)
    acct.reserve(seq, seq.num_tokens)  # 30 + 4 guesses -> 3 blocks
    assert len(inner.block_table(seq)) == 3
    seq.token_ids.extend(range(8))  # 8 generated: 2 left, so 1 guess at most
    assert batch_step.guess_room(seq, 4) == 1
    acct.reserve(seq, seq.num_tokens)  # 38 + 1 -> 3 blocks
    assert len(inner.block_table(seq)) == 3
    assert acct.can_reserve(seq, 16 * 8 - 1) and not acct.can_reserve(seq, 16 * 8)
    acct.free(seq)
    assert inner.num_free_blocks == 8


def test_batch_loop_serves_draft_model_drafts(ref, tiny) -> None:
    """speculative=draft (DraftModelProposer, proposers.py:63-106): a one-layer draft of the same
    family; every request streams what the reference's serial generator with that draft emits."""
    make_golden, ref_mod, backend = ref
    cfg, weights, model, prompts = tiny
    pkg = package()
    draft_cfg = pkg.Qwen3Config(**{**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__}, "num_hidden_layers": 1})
    draft_weights = pkg.make_weights(draft_cfg, seed=1)
    draft_model = make_golden.build_model(ref_mod, draft_cfg, draft_weights, torch.float32)
    want = serial_reference(ref_mod, model, prompts, (), draft_model=draft_model)
    got, loop, fake, metrics = serve(backend, ref_mod, model, cfg, weights, prompts, (),
                                     draft=(draft_cfg, draft_weights, draft_model), speculative="draft",
                                     kv_cache_memory_mb=64)
    assert got == want
    assert metric(metrics, "nanoengine_speculative_proposed_tokens_total") > 0
    with pytest.raises(ValueError, match="draft model"):
        backend.create_b200_engine(model, frozenset(), settings(backend, speculative="draft"),
                                   ref_mod.metrics.EngineMetrics())
