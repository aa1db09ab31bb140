"""The reference's serial speculative API on the B200 kernels (one request at a time).

Same names, arguments and semantics as the reference (paths relative to nanoengine/src/nanoengine):

* ``SamplingParams`` / ``GenerationRequest`` / ``TokenEvent``  engine/interface.py:9-30
* ``Sequence``                 engine/sequence_state.py:12-57
* ``BlockAllocator``           engine/memory/block_allocator.py:8-33 (FIFO free list)
* ``PagedSlotAllocator``       engine/memory/paged_allocator.py:21-79
* ``B200ModelRunner``          engine/generation/model_runner.py:14-80 (``run_step``, ``score_tokens``)
* ``NgramProposer``            engine/speculative/proposers.py:39-60 (the suffix match runs on the GPU)
* ``create_sampling_generator`` engine/sampling.py:12-18 (a Philox4x32-10 stream instead of torch's)
* ``verify_proposal``          engine/speculative/verifier.py:27-60 (greedy: kernel argmax per row;
  sampled: ``ne_verify_logits``, rejection sampling on the request's Philox stream)
* ``SpeculativeGenerator``     engine/speculative/speculative_generator.py:21-90

so that a reference user can swap the runner (and proposer) of the serial speculative path. The
batched path (``engine.B200SpeculativeEngine``) runs the same step for many requests at once.
"""

from __future__ import annotations

import ctypes
import math
import os
from collections import deque
from collections.abc import Iterator
from dataclasses import dataclass, field

import torch

from . import _lib
from .model import B200Model
from .state import DeviceBatchState
from .state import seed_as_int64 as _seed_as_int64

GREEDY_TEMPERATURE = 0.0
PADDING_TOKEN_ID = 0


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


class PhiloxGenerator:
    """A request's random stream: uniform i = (Philox4x32-10(counter=i, key=seed) word 0 >> 8) * 2^-24.

    Stands where the reference keeps a ``torch.Generator`` (create_sampling_generator,
    engine/sampling.py:12-18): a fixed seed always gives the same tokens, no seed draws one from
    the OS. ``draws`` counts the uniforms consumed (the kernels advance it)."""

    def __init__(self, seed: int | None = None) -> None:
        self.seed = int(seed) if seed is not None else int.from_bytes(os.urandom(8), "little")
        self.draws = 0


def create_sampling_generator(seed: int | None, device=None) -> PhiloxGenerator:
    """engine/sampling.py:12-18."""
    return PhiloxGenerator(seed)


@dataclass(eq=False)
class Sequence:
    request: GenerationRequest
    token_ids: list[int]
    num_prompt_tokens: int
    num_cached_tokens: int = 0
    sampling_generator: PhiloxGenerator | None = None

    @classmethod
    def from_request(cls, request: GenerationRequest, device=None) -> "Sequence":
        return cls(request=request, token_ids=list(request.prompt_token_ids),
                   num_prompt_tokens=len(request.prompt_token_ids),
                   sampling_generator=create_sampling_generator(request.sampling_params.seed, device))

    @property
    def request_id(self) -> str:
        return self.request.request_id

    @property
    def sampling_params(self) -> SamplingParams:
        return self.request.sampling_params

    @property
    def num_tokens(self) -> int:
        return len(self.token_ids)

    @property
    def num_generated_tokens(self) -> int:
        return len(self.token_ids) - self.num_prompt_tokens

    @property
    def num_uncached_tokens(self) -> int:
        return len(self.token_ids) - self.num_cached_tokens


class OutOfKVMemoryError(Exception):
    """No free block is left in the KV cache pool (engine/memory/slot_allocator.py:10-11)."""


class BlockAllocator:
    def __init__(self, num_blocks: int) -> None:
        self.num_blocks = num_blocks
        self._free_blocks: deque[int] = deque(range(num_blocks))
        self._used_blocks: set[int] = set()

    @property
    def num_free_blocks(self) -> int:
        return len(self._free_blocks)

    @property
    def num_used_blocks(self) -> int:
        return len(self._used_blocks)

    def allocate(self) -> int:
        if not self._free_blocks:
            raise OutOfKVMemoryError("no free KV blocks")
        block = self._free_blocks.popleft()
        self._used_blocks.add(block)
        return block

    def free(self, block: int) -> None:
        if block not in self._used_blocks:
            raise ValueError(f"block {block} is not allocated")
        self._used_blocks.remove(block)
        self._free_blocks.append(block)


class PagedSlotAllocator:
    def __init__(self, num_blocks: int, block_size: int = 16) -> None:
        self.block_size = block_size
        self._blocks = BlockAllocator(num_blocks)
        self._block_tables: dict[str, list[int]] = {}

    @property
    def num_total_slots(self) -> int:
        return self._blocks.num_blocks * self.block_size

    @property
    def num_reserved_slots(self) -> int:
        return self._blocks.num_used_blocks * self.block_size

    @property
    def num_free_blocks(self) -> int:
        return self._blocks.num_free_blocks

    def block_table(self, sequence) -> list[int]:
        return list(self._block_tables.get(sequence.request_id, []))

    def count_missing_blocks(self, sequence, num_tokens: int) -> int:
        owned = len(self._block_tables.get(sequence.request_id, []))
        return max(0, math.ceil(num_tokens / self.block_size) - owned)

    def can_reserve(self, sequence, num_tokens: int) -> bool:
        return self.count_missing_blocks(sequence, num_tokens) <= self._blocks.num_free_blocks

    def reserve(self, sequence, num_tokens: int) -> None:
        if not self.can_reserve(sequence, num_tokens):
            raise OutOfKVMemoryError(f"no blocks for {num_tokens} tokens of {sequence.request_id}")
        table = self._block_tables.setdefault(sequence.request_id, [])
        for _ in range(self.count_missing_blocks(sequence, num_tokens)):
            table.append(self._blocks.allocate())

    def free(self, sequence) -> None:
        for block in self._block_tables.pop(sequence.request_id, []):
            self._blocks.free(block)

    @property
    def num_prefix_hit_tokens(self) -> int:
        return 0

    def on_tokens_cached(self, sequence) -> None:
        return None


class _HostRows:
    """Device buffers for one host-planned step of ``ne_forward`` (the serial path)."""

    def __init__(self, max_rows: int, table_stride: int, device) -> None:
        i32 = dict(dtype=torch.int32, device=device)
        self.max_rows = max_rows
        self.table_stride = table_stride
        self.ints = torch.zeros(4 * max_rows + 4 + table_stride, **i32)
        self.host = torch.zeros(self.ints.numel(), dtype=torch.int32).pin_memory()

    def fill(self, tokens, positions, slots, start, count, table, lm_rows) -> _lib.Rows:
        R, T = self.max_rows, self.table_stride
        h = self.host
        n, nl = len(tokens), len(lm_rows)
        h.zero_()
        h[0:n] = torch.tensor(tokens, dtype=torch.int32)
        h[R:R + n] = torch.tensor(positions, dtype=torch.int32)
        h[2 * R:2 * R + n] = torch.tensor(slots, dtype=torch.int32)
        h[3 * R:3 * R + nl] = torch.tensor(lm_rows, dtype=torch.int32)
        meta = 4 * R
        h[meta:meta + 4] = torch.tensor([n, nl, start, count], dtype=torch.int32)
        h[meta + 4:meta + 4 + len(table)] = torch.tensor(table, dtype=torch.int32)
        self.ints.copy_(h, non_blocking=True)
        base = self.ints.data_ptr()
        return _lib.Rows(
            max_rows=max(n, 1), num_seqs=1, num_rows=base + 4 * meta, token_ids=base, positions=base + 4 * R,
            slot_mapping=base + 8 * R, q_start=base + 4 * (meta + 2), q_len=base + 4 * (meta + 3),
            block_tables=base + 4 * (meta + 4), table_index=None, block_table_stride=T, max_context=T * 16,
            max_q_len=max(n, 1), lm_rows=base + 12 * R, lm_count=base + 4 * (meta + 1), lm_max=max(nl, 1),
        )


class B200ModelRunner:
    """ModelRunner (engine/generation/model_runner.py:14-80) whose step is ``ne_forward``."""

    def __init__(self, model: B200Model, allocator: PagedSlotAllocator, device=None) -> None:
        self.lib = _lib.load()
        self._model = model
        self.allocator = allocator
        self._device = model.device
        self._rows = _HostRows(model.max_rows, math.ceil(model.max_positions / 16), model.device)
        self._argmax = torch.zeros(model.max_rows, dtype=torch.int32, device=model.device)
        self.last_argmax: list[int] = []

    @property
    def vocab_size(self) -> int:
        return self._model.cfg.vocab_size

    def _forward(self, sequence, count: int, lm_rows: list[int], logits: torch.Tensor | None) -> list[int]:
        start = sequence.num_cached_tokens
        table = self.allocator.block_table(sequence)
        bs = self.allocator.block_size
        positions = list(range(start, start + count))
        slots = [table[p // bs] * bs + p % bs for p in positions]
        tokens = sequence.token_ids[start:start + count]
        rows = self._rows.fill(tokens, positions, slots, 0, count, table, lm_rows)
        mode = _lib.NE_LM_LOGITS if logits is not None else _lib.NE_LM_ARGMAX
        _lib.check(self.lib.ne_forward(self._model.handle, ctypes.byref(rows), mode,
                                       _lib.ptr(logits), self._argmax.data_ptr(), _lib.stream_handle()),
                   "ne_forward")
        ids = self._argmax[: len(lm_rows)].tolist()
        self._model.raise_on_device_error()
        return ids

    def run_step(self, sequences, token_counts=None) -> list[int]:
        """Prefill (or continue) each sequence and return its next token: the argmax, or one draw
        from its target distribution when sampling (ModelRunner._sample, model_runner.py:72-80)."""
        out = []
        for i, seq in enumerate(sequences):
            count = token_counts[i] if token_counts else seq.num_uncached_tokens
            params = seq.sampling_params
            sampled = params.temperature != GREEDY_TEMPERATURE
            logits = None
            if sampled:
                logits = torch.empty((1, self.vocab_size), dtype=torch.bfloat16, device=self._device)
            ids = self._forward(seq, count, [count - 1], logits)
            seq.num_cached_tokens += count
            self.allocator.on_tokens_cached(seq)
            if sampled:
                ids = _logits_verifier(self._device).verify([], logits, params, seq.sampling_generator)
            out.append(ids[0])
        return out

    def score_tokens(self, sequence, token_count: int) -> torch.Tensor:
        """Logits ``[token_count, vocab]`` (bf16, on the GPU) after each of the next tokens."""
        logits = torch.empty((token_count, self.vocab_size), dtype=torch.bfloat16, device=self._device)
        self.last_argmax = self._forward(sequence, token_count, list(range(token_count)), logits)
        sequence.num_cached_tokens += token_count
        self.allocator.on_tokens_cached(sequence)
        return logits


@dataclass(frozen=True)
class Proposal:
    token_ids: list[int]
    probabilities: torch.Tensor | None = None
    # a sampled draft model's logits rows of its guesses (bf16 [len(token_ids), vocab] on the GPU):
    # the verify kernel takes their softmax / top-p as the draft distributions
    draft_logits: torch.Tensor | None = None


class NgramProposer:
    """Prompt lookup on the GPU (``ne_ngram_propose``); same answers as proposers.py:44-57."""

    def __init__(self, max_ngram: int, min_ngram: int = 1, max_model_len: int = 4096, device="cuda") -> None:
        self.lib = _lib.load()
        self._max_ngram = max_ngram
        self._min_ngram = min_ngram
        self._state = DeviceBatchState(1, max_model_len, 16, 1, device=device)
        self._slot = torch.zeros(1, dtype=torch.int32, device=device)
        self._draft_len = torch.zeros(1, dtype=torch.int32, device=device)
        self._status = torch.zeros(1, dtype=torch.int32, device=device)

    def propose(self, sequence, num_tokens: int) -> Proposal:
        history = list(sequence.token_ids)
        if num_tokens <= 0:
            return Proposal([])
        if num_tokens > self._state.k:
            raise ValueError(f"at most {self._state.k} guesses per call")
        self._state.load(0, history, max_new_tokens=num_tokens + 1)
        _lib.check(self.lib.ne_ngram_propose(self._state.ref, self._slot.data_ptr(), 1, num_tokens,
                                             self._max_ngram, self._min_ngram, self._draft_len.data_ptr(),
                                             self._status.data_ptr(), _lib.stream_handle()), "ne_ngram_propose")
        g = int(self._draft_len.item())
        if int(self._status.item()):
            raise _lib.NativeError(_lib.describe_device_status(int(self._status.item())))
        L = len(history)
        return Proposal(self._state.history[0, L:L + g].tolist() if g > 0 else [])

    def release(self, sequence) -> None:
        return None


class DraftModelProposer:
    """DraftModelProposer (engine/speculative/proposers.py:63-106) on the GPU: ``runner`` is a
    ``B200ModelRunner`` over the draft model and its own paged allocator; each proposal syncs the
    draft sequence with the target (common-prefix cache kept, ``_sync_draft``) and runs
    ``num_tokens`` draft steps, the first catching up on the target's new tokens. Greedy requests:
    the guesses are the draft's argmax ids, returned as one-hot drafts (``probabilities`` None,
    which ``verify_proposal`` reads as one-hot rows, the distributions the reference stacks for a
    greedy draft). Sampled requests: each guess is drawn from the draft's distribution on the
    request's generator (one uniform, as ``sample_from_probabilities``), and the draft's logits rows
    go with the proposal (``draft_logits``) for verification against them."""

    def __init__(self, runner: B200ModelRunner, device=None) -> None:
        self._runner = runner
        self._device = device
        self._draft_sequences: dict[str, Sequence] = {}

    def propose(self, sequence, num_tokens: int) -> Proposal:
        params = sequence.sampling_params
        sampled = params.temperature != GREEDY_TEMPERATURE
        draft = self._sync_draft(sequence)
        guesses: list[int] = []
        rows: list[torch.Tensor] = []
        for _ in range(num_tokens):
            self._runner.allocator.reserve(draft, draft.num_tokens)
            if not sampled:
                guess = self._runner.run_step([draft])[0]  # the argmax after the draft's uncached tokens
            else:
                row = self._runner.score_tokens(draft, draft.num_uncached_tokens)[-1:]
                guess = _logits_verifier(row.device).verify([], row, params, sequence.sampling_generator)[0]
                rows.append(row)
            draft.token_ids.append(guess)
            guesses.append(guess)
        return Proposal(guesses, draft_logits=torch.cat(rows) if rows else None)

    def release(self, sequence) -> None:
        draft = self._draft_sequences.pop(sequence.request_id, None)
        if draft is not None:
            self._runner.allocator.free(draft)

    def _sync_draft(self, sequence) -> Sequence:
        draft = self._draft_sequences.get(sequence.request_id)
        if draft is None:
            draft = Sequence.from_request(sequence.request, self._device)
            self._draft_sequences[sequence.request_id] = draft
        common = 0
        for draft_token, target_token in zip(draft.token_ids, sequence.token_ids):
            if draft_token != target_token:
                break
            common += 1
        draft.token_ids = list(sequence.token_ids)
        draft.num_cached_tokens = min(draft.num_cached_tokens, common)
        return draft


class _LogitsVerifier:
    """``ne_verify_logits`` for one proposal at a time: a one-slot device state holds the guesses,
    the request's sampling parameters and its Philox position."""

    MAX_GUESSES = 16

    def __init__(self, device) -> None:
        self.lib = _lib.load()
        self.device = torch.device(device)
        k = self.MAX_GUESSES
        self.state = DeviceBatchState(1, 8, k, 1, device=self.device)
        self.state.flags.fill_(_lib.NE_SEQ_IGNORE_EOS)
        i32 = dict(dtype=torch.int32, device=self.device)
        self.slot = torch.zeros(1, **i32)
        self.lm_start = torch.zeros(1, **i32)
        self.draft_len = torch.zeros(1, **i32)
        self.scratch = torch.zeros((2 * k + 1) * 32, dtype=torch.uint8, device=self.device)
        self.out = torch.zeros(k + 1 + 4, **i32)
        base = self.out.data_ptr()
        self.out_struct = _lib.StepOutputs(tokens=base, count=base + 4 * (k + 1), finish=base + 4 * (k + 2),
                                           proposed=base + 4 * (k + 3), accepted=base + 4 * (k + 4))
        self.status = torch.zeros(1, **i32)

    def verify(self, guesses: list[int], logits: torch.Tensor, params: SamplingParams,
               generator: PhiloxGenerator | None, draft_logits: torch.Tensor | None = None) -> list[int]:
        g = len(guesses)
        if g > self.MAX_GUESSES:
            raise ValueError(f"at most {self.MAX_GUESSES} guesses per proposal")
        if logits.dim() != 2 or logits.shape[0] < g + 1 or logits.dtype != torch.bfloat16 or not logits.is_cuda:
            raise ValueError("target logits must be a CUDA bf16 tensor of [len(guesses) + 1, vocab]")
        sampled = params.temperature != GREEDY_TEMPERATURE
        if sampled and generator is None:
            raise ValueError("sampled verification needs the request's generator")
        st = self.state
        hist = torch.zeros(st.history_stride, dtype=torch.int32)
        hist[:g] = torch.tensor(guesses, dtype=torch.int32)
        st.history[0].copy_(hist)
        st.seq_len.zero_()
        st.num_cached.zero_()
        st.num_prompt.zero_()
        st.max_new_tokens.fill_(1 << 30)
        st.temperature.fill_(float(params.temperature))
        st.top_p.fill_(float(params.top_p))
        if sampled:
            st.rng_seed.fill_(_seed_as_int64(generator.seed))
            st.rng_draws.fill_(generator.draws)
        self.draft_len.fill_(g)
        logits = logits.contiguous()
        if draft_logits is not None and sampled and g > 0:
            if draft_logits.shape != (g, logits.shape[1]) or draft_logits.dtype != torch.bfloat16:
                raise ValueError("draft logits must be bf16 [len(guesses), vocab]")
            draft_logits = draft_logits.contiguous()
            _lib.check(self.lib.ne_verify_logits_drafted(
                st.ref, self.slot.data_ptr(), 1, self.MAX_GUESSES, self.draft_len.data_ptr(),
                self.lm_start.data_ptr(), logits.data_ptr(), logits.shape[1], g + 1, draft_logits.data_ptr(),
                self.lm_start.data_ptr(), g, self.scratch.data_ptr(), self.scratch.numel(),
                ctypes.byref(self.out_struct), self.status.data_ptr(), _lib.stream_handle()),
                "ne_verify_logits_drafted")
        else:
            _lib.check(self.lib.ne_verify_logits(
                st.ref, self.slot.data_ptr(), 1, self.MAX_GUESSES, self.draft_len.data_ptr(),
                self.lm_start.data_ptr(), logits.data_ptr(), logits.shape[1], g + 1, self.scratch.data_ptr(),
                self.scratch.numel(), ctypes.byref(self.out_struct), self.status.data_ptr(), _lib.stream_handle()),
                "ne_verify_logits")
        out = self.out.tolist()
        count = out[self.MAX_GUESSES + 1]
        word = int(self.status.item())
        if word:
            self.status.zero_()
            raise _lib.NativeError(f"device reported: {_lib.describe_device_status(word)} (0x{word:x})")
        if sampled:
            generator.draws = int(st.rng_draws[0].item())
        return out[:count]


_VERIFIERS: dict[str, _LogitsVerifier] = {}


def _logits_verifier(device) -> _LogitsVerifier:
    key = str(torch.device(device))
    if key not in _VERIFIERS:
        _VERIFIERS[key] = _LogitsVerifier(device)
    return _VERIFIERS[key]


def verify_proposal(proposal: Proposal, target_logits: torch.Tensor, params: SamplingParams, generator=None,
                    target_argmax: list[int] | None = None) -> list[int]:
    """verifier.py:27-60 with one-hot drafts (n-gram, greedy draft model) or a sampled draft model's
    rows (``proposal.draft_logits``): kept guesses + one target token.

    Greedy: ``target_argmax`` (the kernel's per-row argmax ids, lowest index on ties) are compared
    on the host; without them the verify kernel takes the argmax itself. Sampled: rejection
    sampling on the GPU with ``generator`` (the request's ``PhiloxGenerator``), which advances.
    """
    if proposal.probabilities is not None:
        raise ValueError("the B200 verify takes one-hot drafts or a draft model's logits rows (draft_logits)")
    if params.temperature != GREEDY_TEMPERATURE or target_argmax is None:
        return _logits_verifier(target_logits.device).verify(list(proposal.token_ids), target_logits, params,
                                                             generator, draft_logits=proposal.draft_logits)
    kept: list[int] = []
    for index, guess in enumerate(proposal.token_ids):
        if guess == target_argmax[index]:
            kept.append(guess)
            continue
        return [*kept, target_argmax[index]]
    return [*kept, target_argmax[len(proposal.token_ids)]]


def find_finish_reason(token_id: int, num_generated_tokens: int, params: SamplingParams,
                       stop_token_ids: frozenset[int]) -> str | None:
    """engine/sampling.py:54-62."""
    if not params.ignore_eos and token_id in stop_token_ids:
        return "stop"
    if num_generated_tokens >= params.max_new_tokens:
        return "length"
    return None


@dataclass
class SpeculativeCounters:
    proposed: int = 0
    accepted: int = 0
    steps: list = field(default_factory=list)


class SpeculativeGenerator:
    """engine/speculative/speculative_generator.py:21-90 over ``B200ModelRunner``."""

    def __init__(self, runner: B200ModelRunner, proposer: "NgramProposer | DraftModelProposer", num_speculative_tokens: int,
                 stop_token_ids: frozenset[int], device=None, metrics: SpeculativeCounters | None = None) -> None:
        self._runner = runner
        self._proposer = proposer
        self._num_speculative_tokens = num_speculative_tokens
        self._stop_token_ids = stop_token_ids
        self._metrics = metrics

    @property
    def vocab_size(self) -> int:
        return self._runner.vocab_size

    def generate(self, request: GenerationRequest) -> Iterator[TokenEvent]:
        sequence = Sequence.from_request(request)
        try:
            yield from self._generate(sequence)
        finally:
            self._runner.allocator.free(sequence)
            self._proposer.release(sequence)

    def _generate(self, sequence: Sequence) -> Iterator[TokenEvent]:
        self._runner.allocator.reserve(sequence, sequence.num_tokens)
        new_tokens = self._runner.run_step([sequence])
        while True:
            for token_id in new_tokens:
                sequence.token_ids.append(token_id)
                reason = find_finish_reason(token_id, sequence.num_generated_tokens, sequence.sampling_params,
                                            self._stop_token_ids)
                yield TokenEvent(sequence.request_id, token_id, reason is not None, reason)
                if reason is not None:
                    return
            new_tokens = self._run_speculative_step(sequence)

    def _run_speculative_step(self, sequence: Sequence) -> list[int]:
        remaining = sequence.sampling_params.max_new_tokens - sequence.num_generated_tokens
        num_guesses = max(0, min(self._num_speculative_tokens, remaining - 1))
        proposal = self._proposer.propose(sequence, num_guesses) if num_guesses else Proposal([])
        length_before = sequence.num_tokens
        sequence.token_ids.extend(proposal.token_ids)
        self._runner.allocator.reserve(sequence, sequence.num_tokens)
        table = self._runner.allocator.block_table(sequence)
        target_logits = self._runner.score_tokens(sequence, 1 + len(proposal.token_ids))
        sampled = sequence.sampling_params.temperature != GREEDY_TEMPERATURE
        new_tokens = verify_proposal(proposal, target_logits, sequence.sampling_params, sequence.sampling_generator,
                                     target_argmax=None if sampled else self._runner.last_argmax)
        num_kept = len(new_tokens) - 1
        del sequence.token_ids[length_before:]
        sequence.num_cached_tokens = length_before + num_kept
        if self._metrics is not None:
            self._metrics.proposed += len(proposal.token_ids)
            self._metrics.accepted += num_kept
            self._metrics.steps.append((list(proposal.token_ids), table, target_logits, list(new_tokens)))
        return new_tokens
