"""The reference's serial speculative classes, restated for the GPU box (TEST INFRASTRUCTURE).

The reference (nanoengine, pure Python) is not installed where the ``-m gpu`` tests run, so the
GPU tests drive the B200 runner and proposers through this restatement of its serial seam. Each
class keeps the reference's names, arguments and behaviour (paths relative to
``nanoengine/src/nanoengine``):

* ``SamplingParams`` / ``GenerationRequest`` / ``TokenEvent``   engine/interface.py
* ``Sequence``                   engine/sequence_state.py:12-57 (a ``torch.Generator`` per request)
* ``PagedSlotAllocator``         engine/memory/paged_allocator.py:21-79 over the FIFO block list of
                                 engine/memory/block_allocator.py:8-33 (``oracle.speculative.PagedTables``)
* ``find_finish_reason``         engine/sampling.py:54-62
* ``SpeculativeGenerator``       engine/speculative/speculative_generator.py:21-90; ``verify`` is the
                                 ``verify_proposal`` it calls (the B200 device verify by default),
                                 and ``metrics`` records every step for the parity tests

``tests/test_reference_seam.py`` checks these against the reference itself where it is present
(same events, block tables and call sequence on the reference's own CPU runner).
"""

from __future__ import annotations

import importlib
from dataclasses import dataclass, field

import torch

from oracle.speculative import OutOfBlocks, PagedTables

PACKAGE = "inference-engine-from-scratch_b200"


@dataclass(frozen=True)
class SamplingParams:
    max_new_tokens: int
    temperature: float = 0.0
    top_p: float = 1.0
    seed: int | None = None
    ignore_eos: bool = False


@dataclass(frozen=True)
class GenerationRequest:
    request_id: str
    prompt_token_ids: list[int]
    sampling_params: SamplingParams


@dataclass(frozen=True)
class TokenEvent:
    request_id: str
    token_id: int
    is_finished: bool
    finish_reason: str | None


def new_generator(seed: int | None, device=None) -> torch.Generator:
    """A request's ``torch.Generator`` (engine/sampling.py:12-18), always on the CPU here: the B200
    path draws from the Philox stream keyed by its seed, never from the generator itself."""
    gen = torch.Generator()
    if seed is None:
        gen.seed()
    else:
        gen.manual_seed(seed)
    return gen


@dataclass(eq=False)
class Sequence:
    request: GenerationRequest
    sampling_generator: torch.Generator
    token_ids: list[int]
    num_prompt_tokens: int
    num_cached_tokens: int = 0

    @classmethod
    def from_request(cls, request: GenerationRequest, device=None) -> "Sequence":
        return cls(request, new_generator(request.sampling_params.seed, device), list(request.prompt_token_ids),
                   len(request.prompt_token_ids))

    request_id = property(lambda self: self.request.request_id)
    sampling_params = property(lambda self: self.request.sampling_params)
    num_tokens = property(lambda self: len(self.token_ids))
    num_generated_tokens = property(lambda self: len(self.token_ids) - self.num_prompt_tokens)
    num_uncached_tokens = property(lambda self: len(self.token_ids) - self.num_cached_tokens)

    def forget_cache(self) -> None:
        self.num_cached_tokens = 0


class PagedSlotAllocator:
    """Block tables per request id over a FIFO free list; ``reserve`` raises when blocks run out."""

    def __init__(self, num_blocks: int, block_size: int = 16, device=None) -> None:
        self.block_size = block_size
        self._tables = PagedTables(num_blocks, block_size)

    @property
    def num_free_blocks(self) -> int:
        return len(self._tables.blocks.free_blocks)

    def block_table(self, sequence) -> list[int]:
        return list(self._tables.tables.get(sequence.request_id, []))

    def reserve(self, sequence, num_tokens: int) -> None:
        self._tables.reserve(sequence.request_id, num_tokens)

    def free(self, sequence) -> None:
        self._tables.free(sequence.request_id)

    def on_tokens_cached(self, sequence) -> None:
        return None


def find_finish_reason(token_id: int, num_generated: int, params: SamplingParams, stop_ids) -> str | None:
    if token_id in stop_ids and not params.ignore_eos:
        return "stop"
    return "length" if num_generated >= params.max_new_tokens else None


@dataclass
class StepRecords:
    """Counters the reference keeps in EngineMetrics, plus every step (for the parity tests):
    (draft, block table after the reservation, verify logits, emitted tokens)."""

    proposed: int = 0
    accepted: int = 0
    steps: list = field(default_factory=list)


def _device_verify(proposal, logits, params, generator):
    return importlib.import_module(f"{PACKAGE}.serial").verify_proposal(proposal, logits, params, generator)


class SpeculativeGenerator:
    def __init__(self, runner, proposer, num_speculative_tokens: int, stop_token_ids, device=None,
                 metrics: StepRecords | None = None, verify=_device_verify) -> None:
        self._runner, self._proposer = runner, proposer
        self._k = num_speculative_tokens
        self._stop_ids = frozenset(stop_token_ids)
        self._device = device
        self._metrics = metrics
        self._verify = verify

    @property
    def vocab_size(self) -> int:
        return self._runner.vocab_size

    def generate(self, request: GenerationRequest):
        sequence = Sequence.from_request(request, self._device)
        try:
            yield from self._generate(sequence)
        finally:
            self._runner.allocator.free(sequence)
            self._proposer.release(sequence)
            importlib.import_module(f"{PACKAGE}.serial").release_stream(sequence.sampling_generator)

    def _generate(self, sequence: Sequence):
        # the first call prefills the prompt; every later call verifies guesses
        self._runner.allocator.reserve(sequence, sequence.num_tokens)
        tokens = self._runner.run_step([sequence])
        while True:
            for token in tokens:
                sequence.token_ids.append(token)
                reason = find_finish_reason(token, sequence.num_generated_tokens, sequence.sampling_params,
                                            self._stop_ids)
                yield TokenEvent(sequence.request_id, token, reason is not None, reason)
                if reason is not None:
                    return
            tokens = self._step(sequence)

    def _step(self, sequence: Sequence) -> list[int]:
        left = sequence.sampling_params.max_new_tokens - sequence.num_generated_tokens
        guesses = max(0, min(self._k, left - 1))
        proposal = self._proposer.propose(sequence, guesses) if guesses else _empty_proposal()
        before = sequence.num_tokens
        sequence.token_ids.extend(proposal.token_ids)
        self._runner.allocator.reserve(sequence, sequence.num_tokens)
        table = self._runner.allocator.block_table(sequence) if self._metrics is not None else None
        logits = self._runner.score_tokens(sequence, 1 + len(proposal.token_ids))
        new = self._verify(proposal, logits, sequence.sampling_params, sequence.sampling_generator)
        kept = len(new) - 1
        del sequence.token_ids[before:]
        sequence.num_cached_tokens = before + kept
        if self._metrics is not None:
            self._metrics.proposed += len(proposal.token_ids)
            self._metrics.accepted += kept
            self._metrics.steps.append((list(proposal.token_ids), table, logits, list(new)))
        return new


def _empty_proposal():
    return importlib.import_module(f"{PACKAGE}.serial").Proposal([])


__all__ = ["GenerationRequest", "OutOfBlocks", "PagedSlotAllocator", "SamplingParams", "Sequence",
           "SpeculativeGenerator", "StepRecords", "TokenEvent", "find_finish_reason"]
