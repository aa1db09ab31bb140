"""The B200 parts of the reference's serial speculative API (one request at a time).

These plug into the reference's own serial classes (paths relative to nanoengine/src/nanoengine):
the reference's ``SpeculativeGenerator`` (engine/speculative/speculative_generator.py:21-90) drives
them with its own ``Sequence`` (engine/sequence_state.py:12-57) and ``PagedSlotAllocator``
(engine/memory/paged_allocator.py:21-79), exactly as ``runtime.create_engine`` wires its
``ModelRunner`` and proposer (engine/runtime.py:162-171). Built here:

* ``B200ModelRunner``          ModelRunner (engine/generation/model_runner.py:14-80): ``run_step`` and
                               ``score_tokens`` over ``ne_forward``; it reads the sequence's
                               ``token_ids`` / ``num_cached_tokens`` and the allocator's
                               ``block_table`` / ``block_size``, and calls ``on_tokens_cached``
* ``NgramProposer``            engine/speculative/proposers.py:39-60 (the suffix match runs on the GPU)
* ``DraftModelProposer``       engine/speculative/proposers.py:63-106 over a ``B200ModelRunner``
* ``PhiloxGenerator`` / ``create_sampling_generator``
                               a request's random stream (Philox4x32-10) where the reference keeps a
                               ``torch.Generator`` (engine/sampling.py:12-18)
* ``verify_proposal``          engine/speculative/verifier.py:27-60 on the GPU (greedy: the kernel's
                               per-row argmax; sampled: ``ne_verify_logits``, rejection sampling on the
                               request's Philox stream)

The reference's own ``verify_proposal`` also works on the bf16 logits ``score_tokens`` returns (it
is plain torch); this module's ``verify_proposal`` is the device path, whose sampled decisions are
bit-comparable with the reference's when both draw from the same Philox stream. A reference
``Sequence`` carries a ``torch.Generator``: sampled first tokens (``run_step``) then draw from a
Philox stream keyed by that generator's seed (``initial_seed()``), one stream per generator.
The batched path (``engine.B200SpeculativeEngine``) runs the same step for many requests at once.
"""

from __future__ import annotations

import ctypes
import math
import os
from collections import OrderedDict
from dataclasses import dataclass

import torch

from . import _lib
from .model import B200Model
from .state import DeviceBatchState
from .state import seed_as_int64 as _seed_as_int64

GREEDY_TEMPERATURE = 0.0


class PhiloxGenerator:
    """A request's random stream: uniform i = (Philox4x32-10(counter=i, key=seed) word 0 >> 8) * 2^-24.

    Stands where the reference keeps a ``torch.Generator`` (create_sampling_generator,
    engine/sampling.py:12-18): a fixed seed always gives the same tokens, no seed draws one from
    the OS. ``draws`` counts the uniforms consumed (the kernels advance it)."""

    def __init__(self, seed: int | None = None) -> None:
        self.seed = int(seed) if seed is not None else int.from_bytes(os.urandom(8), "little")
        self.draws = 0


def create_sampling_generator(seed: int | None, device=None) -> PhiloxGenerator:
    """engine/sampling.py:12-18, with a Philox stream in place of the ``torch.Generator``."""
    return PhiloxGenerator(seed)


# torch.Generator objects take no weak references: the streams of reference generators are held
# by object id (with the generator, so a recycled id is noticed) until ``release_stream``, and at
# most _MAX_TORCH_STREAMS of them (the least recently used is dropped; the serial path serves one
# request at a time)
_MAX_TORCH_STREAMS = 1024
_TORCH_STREAMS: "OrderedDict[int, tuple[object, PhiloxGenerator]]" = OrderedDict()


def philox_stream(generator) -> PhiloxGenerator:
    """The Philox stream a request draws from: its own ``PhiloxGenerator``, or for the reference's
    ``torch.Generator`` one stream per generator object, keyed by its ``initial_seed()``."""
    if isinstance(generator, PhiloxGenerator):
        return generator
    if generator is None:
        raise ValueError("sampled decoding needs the request's generator")
    held = _TORCH_STREAMS.get(id(generator))
    if held is None or held[0] is not generator:
        held = (generator, PhiloxGenerator(int(generator.initial_seed())))
        _TORCH_STREAMS[id(generator)] = held
        while len(_TORCH_STREAMS) > _MAX_TORCH_STREAMS:
            _TORCH_STREAMS.popitem(last=False)
    _TORCH_STREAMS.move_to_end(id(generator))
    return held[1]


def release_stream(generator) -> None:
    """Forget the Philox stream of a finished request's ``torch.Generator``."""
    _TORCH_STREAMS.pop(id(generator), None)


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
    """ModelRunner (engine/generation/model_runner.py:14-80) whose step is ``ne_forward``.

    ``allocator`` is the reference's ``PagedSlotAllocator`` (or any object with ``block_size``,
    ``block_table(sequence)`` and ``on_tokens_cached(sequence)``); sequences are the reference's
    ``Sequence`` (``token_ids``, ``num_cached_tokens``, ``sampling_params``, ``sampling_generator``)."""

    def __init__(self, model: B200Model, allocator, device=None) -> None:
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
            self._cached(seq)
            if sampled:
                ids = _logits_verifier(self._device).verify([], logits, params, philox_stream(seq.sampling_generator))
            out.append(ids[0])
        return out

    def score_tokens(self, sequence, token_count: int) -> torch.Tensor:
        """Logits ``[token_count, vocab]`` (bf16, on the GPU) after each of the next tokens."""
        logits = torch.empty((token_count, self.vocab_size), dtype=torch.bfloat16, device=self._device)
        self.last_argmax = self._forward(sequence, token_count, list(range(token_count)), logits)
        sequence.num_cached_tokens += token_count
        self._cached(sequence)
        return logits

    def _cached(self, sequence) -> None:
        hook = getattr(self.allocator, "on_tokens_cached", None)  # (the prefix-cache hook)
        if hook is not None:
            hook(sequence)


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
        self._draft_sequences: dict = {}

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
                guess = _logits_verifier(row.device).verify([], row, params, philox_stream(sequence.sampling_generator))[0]
                rows.append(row)
            draft.token_ids.append(guess)
            guesses.append(guess)
        return Proposal(guesses, draft_logits=torch.cat(rows) if rows else None)

    def release(self, sequence) -> None:
        draft = self._draft_sequences.pop(sequence.request_id, None)
        if draft is not None:
            self._runner.allocator.free(draft)

    def _sync_draft(self, sequence):
        draft = self._draft_sequences.get(sequence.request_id)
        if draft is None:
            # a sequence of the caller's own class (the reference's Sequence) for the draft model
            draft = type(sequence).from_request(sequence.request, self._device)
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

    def verify(self, guesses: list[int], logits: torch.Tensor, params, generator: PhiloxGenerator | None,
               draft_logits: torch.Tensor | None = None) -> list[int]:
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


def verify_proposal(proposal, target_logits: torch.Tensor, params, generator=None,
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
        stream = philox_stream(generator) if params.temperature != GREEDY_TEMPERATURE else None
        return _logits_verifier(target_logits.device).verify(list(proposal.token_ids), target_logits, params,
                                                             stream, draft_logits=getattr(proposal, "draft_logits", None))
    kept: list[int] = []
    for index, guess in enumerate(proposal.token_ids):
        if guess == target_argmax[index]:
            kept.append(guess)
            continue
        return [*kept, target_argmax[index]]
    return [*kept, target_argmax[len(proposal.token_ids)]]
