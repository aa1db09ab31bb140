"""The B200 speculative step as a backend of nanoengine's own batched engine.

Importing this module imports the reference package (``nanoengine``): it is the part of the B200
backend a nanoengine deployment loads, next to its runtime.

* ``B200EngineSettings``: the reference's ``EngineSettings`` (config.py:23-102) plus
  ``speculative_backend`` (``NANOENGINE_SPECULATIVE_BACKEND``, ``torch`` | ``b200``). The
  reference's validator (config.py:81-99) refuses speculative decoding under a batch scheduler
  (:91-97); with the b200 backend that one rule is replaced by the backend's own (continuous
  scheduler, paged KV in 16-token blocks, no prefix cache, no chunked prefill, bfloat16, n-gram or
  draft-model drafts), and every other check of the reference's validator still runs.
* ``SpeculativeBatchEngineLoop``: the reference's ``BatchEngineLoop`` (engine/scheduling/
  batch_engine_loop.py:35-176) with ``_execute_plan`` (:114-130) running each plan as one batched
  speculative step (``batch_step.SpeculativeBatchExecutor``). The loop's admission, streaming,
  cancellation, finish handling and metrics are the reference's, unchanged; a step simply hands
  back up to k + 1 tokens per sequence, which ``_emit_token`` streams one by one.
* ``create_b200_engine``: ``runtime.create_engine`` (engine/runtime.py:132-187) for the b200
  backend: the reference's ``ContinuousBatchScheduler`` over its ``PagedSlotAllocator`` sized from
  ``kv_cache_memory_mb`` as the reference sizes it (``count_slots_for_budget``), the allocator
  wrapped so that reservations include each request's guess room.
"""

from __future__ import annotations

from typing import Literal

import torch
from nanoengine.config import EngineSettings
from nanoengine.constants import (
    KV_CACHE_PAGED,
    SCHEDULER_CONTINUOUS,
    SPECULATIVE_DRAFT,
    SPECULATIVE_NGRAM,
    SPECULATIVE_NONE,
)
from nanoengine.engine.memory.kv_cache_pool import count_slots_for_budget
from nanoengine.engine.memory.paged_allocator import PagedSlotAllocator
from nanoengine.engine.metrics import EngineMetrics
from nanoengine.engine.scheduling.batch_engine_loop import BatchEngineLoop
from nanoengine.engine.scheduling.batch_scheduler import ContinuousBatchScheduler, StepPlan
from pydantic import model_validator

from .batch_step import GuessRoomAllocator, SpeculativeBatchExecutor
from .config import BACKEND_B200, BACKEND_TORCH, Qwen3Config

B200_BLOCK_SIZE = 16


class B200EngineSettings(EngineSettings):
    speculative_backend: Literal["torch", "b200"] = BACKEND_TORCH

    @model_validator(mode="after")
    def check_batching_has_a_kv_cache(self) -> "B200EngineSettings":
        if self.speculative_backend != BACKEND_B200 or self.speculative == SPECULATIVE_NONE:
            return EngineSettings.check_batching_has_a_kv_cache(self)
        # every other rule of the reference's validator, checked on the same settings without
        # the speculative mode (the one rule the b200 backend replaces)
        EngineSettings.check_batching_has_a_kv_cache(self.model_copy(update={"speculative": SPECULATIVE_NONE}))
        problems = []
        if self.scheduler != SCHEDULER_CONTINUOUS:
            problems.append("scheduler=continuous")
        if self.kv_cache != KV_CACHE_PAGED or self.kv_block_size != B200_BLOCK_SIZE:
            problems.append(f"kv_cache=paged with kv_block_size={B200_BLOCK_SIZE}")
        if self.prefix_cache or self.chunked_prefill:
            problems.append("no prefix_cache and no chunked_prefill")
        if self.dtype != "bfloat16":
            problems.append("dtype=bfloat16")
        if self.speculative not in (SPECULATIVE_NGRAM, SPECULATIVE_DRAFT):
            problems.append("speculative=ngram or draft")
        if problems:
            raise ValueError("speculative_backend=b200 needs " + ", ".join(problems))
        return self


class SpeculativeBatchEngineLoop(BatchEngineLoop):
    """``BatchEngineLoop`` whose steps are batched speculative steps (see the module docstring)."""

    def __init__(self, executor: SpeculativeBatchExecutor, allocator: GuessRoomAllocator,
                 scheduler: ContinuousBatchScheduler, metrics: EngineMetrics, stop_token_ids: frozenset[int],
                 max_waiting_requests: int, device: torch.device) -> None:
        self._executor = executor
        super().__init__(_LoopRunner(allocator), scheduler, metrics, stop_token_ids, max_waiting_requests, device)

    def _execute_plan(self, plan: StepPlan) -> list:
        engine = self._executor.engine
        proposed, accepted = getattr(engine, "proposed_total", 0), getattr(engine, "accepted_total", 0)
        new_tokens = self._executor.execute(plan)
        # the speculative counters of the reference's metrics (speculative_generator.py:84-85)
        self._metrics.speculative_proposed_tokens.inc(getattr(engine, "proposed_total", 0) - proposed)
        self._metrics.speculative_accepted_tokens.inc(getattr(engine, "accepted_total", 0) - accepted)
        return new_tokens


class _LoopRunner:
    """What ``BatchEngineLoop`` reads of its runner besides ``run_step``: the allocator."""

    def __init__(self, allocator: GuessRoomAllocator) -> None:
        self.allocator = allocator

    def run_step(self, sequences, chunk_sizes=None):
        raise RuntimeError("the speculative batch loop runs its plans through the B200 executor")


def b200_config(reference_config) -> Qwen3Config:
    """The reference model's ``Qwen3Config`` (models/qwen3.py:13-28) as this package's."""
    names = Qwen3Config.__dataclass_fields__
    return Qwen3Config(**{name: getattr(reference_config, name) for name in names})


def num_kv_blocks(model_config, settings: EngineSettings) -> int:
    """Blocks of the KV budget, counted as the reference counts them (runtime.py:54-95,
    kv_cache_pool.py:27-31)."""
    slots = count_slots_for_budget(model_config, torch.bfloat16, settings.kv_cache_memory_mb,
                                   settings.is_int8_kv_cache)
    return slots // B200_BLOCK_SIZE


def create_b200_engine(model, stop_token_ids: frozenset[int], settings: B200EngineSettings,
                       metrics: EngineMetrics, draft_model=None, *, engine=None) -> SpeculativeBatchEngineLoop:
    """The b200 branch of ``runtime.create_engine``: ``model`` is the reference's
    ``Qwen3ForCausalLM`` whose weights the B200 model takes; ``draft_model`` (speculative=draft) the
    reference's draft model, loaded as ``runtime.create_proposer`` loads it (runtime.py:115-129),
    whose weights a second B200 model takes with its own KV pool of as many blocks (``engine``: a
    prebuilt ``B200SpeculativeEngine``, or any object with its request API)."""
    if settings.speculative_backend != BACKEND_B200:
        raise ValueError("create_b200_engine serves speculative_backend=b200")
    device = torch.device(settings.device)
    num_blocks = num_kv_blocks(model.config, settings)
    if engine is None:
        from .engine import B200SpeculativeEngine
        from .model import B200Model

        k = settings.num_speculative_tokens

        def device_model(ref_model, int8: bool):
            weights = {name: t.detach() for name, t in ref_model.state_dict().items()}
            return B200Model(b200_config(ref_model.config), weights, num_slots=num_blocks * B200_BLOCK_SIZE,
                             device=device, max_positions=settings.max_model_len + k + 1,
                             kv_int8=int8 and settings.is_int8_kv_cache,
                             max_rows=max(settings.max_num_seqs * (k + 1), settings.max_prefill_tokens),
                             max_seqs=settings.max_num_seqs, weight_int8=int8 and settings.quantization == "int8")

        draft = None
        if settings.speculative == SPECULATIVE_DRAFT:
            if draft_model is None:
                raise ValueError("speculative=draft needs the draft model (runtime.create_proposer loads it)")
            draft = device_model(draft_model, int8=False)
        engine = B200SpeculativeEngine(device_model(model, int8=True), k=k, max_ngram=settings.ngram_max_size,
                                       max_seqs=settings.max_num_seqs, max_model_len=settings.max_model_len,
                                       num_blocks=num_blocks, stop_token_ids=tuple(sorted(stop_token_ids)),
                                       cuda_graphs=settings.cuda_graphs, max_prefill_rows=settings.max_prefill_tokens,
                                       sampling=True, draft_model=draft, draft_num_blocks=num_blocks)
        if settings.cuda_graphs:
            engine.capture_all_buckets()
    executor = SpeculativeBatchExecutor(engine, stop_token_ids)
    allocator = GuessRoomAllocator(PagedSlotAllocator(num_blocks, B200_BLOCK_SIZE, device), executor)
    scheduler = ContinuousBatchScheduler(allocator, settings.max_num_seqs, settings.max_prefill_tokens)
    return SpeculativeBatchEngineLoop(executor, allocator, scheduler, metrics, stop_token_ids,
                                      settings.max_waiting_requests, device)
