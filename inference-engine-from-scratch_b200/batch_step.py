"""The batched speculative step behind a batch scheduler's step plans.

The reference's batch loop (engine/scheduling/batch_engine_loop.py:114-130, ``_execute_plan``)
asks its runner for one token per sequence per step; its scheduler (batch_scheduler.py:30-85)
admits, reserves KV memory and preempts. Here the same plans run through
``B200SpeculativeEngine``: a prefill plan loads the admitted sequences into engine slots and
prefills them (one first token each), a decode plan runs one speculative step for every running
sequence (draft, verify, accept and KV commit on the device), which emits 1 to k + 1 tokens per
sequence, already cut at a stop token or the length limit as ``find_finish_reason``
(engine/sampling.py:54-62) would cut them.

Sequences are the reference's ``Sequence`` objects (engine/sequence_state.py:12-57), read by
attribute only: ``request_id``, ``token_ids``, ``num_prompt_tokens``, ``num_generated_tokens``,
``num_cached_tokens``, ``sampling_params`` and ``sampling_generator``. This module imports nothing
from the reference; ``nanoengine_backend`` binds it to the reference's loop and settings.

KV memory: the engine keeps its own device block FIFO; the scheduler's allocator is the host
account the scheduler admits and preempts by. ``GuessRoomAllocator`` makes that account reserve,
for every request it sees, room for the request's next step's guesses as well
(``min(k, remaining - 1)``, the cap of speculative_generator.py:73-74), so the host account is
never below what the device reserves and the device FIFO never runs dry while the scheduler
believes there is room.
"""

from __future__ import annotations


def guess_room(sequence, k: int) -> int:
    """The most guesses the sequence's next speculative step can verify (speculative_generator.py:73-74)."""
    remaining = sequence.sampling_params.max_new_tokens - sequence.num_generated_tokens
    return max(0, min(k, remaining - 1))


def request_seed(sequence) -> int:
    """The Philox key of a request: the seed its ``torch.Generator`` was made with
    (``create_sampling_generator``, engine/sampling.py:11-18; a random one when the request gave none)."""
    generator = getattr(sequence, "sampling_generator", None)
    if generator is not None:
        return int(generator.initial_seed())
    seed = sequence.sampling_params.seed
    return int(seed) if seed is not None else 0


class SpeculativeBatchExecutor:
    """Runs step plans through a ``B200SpeculativeEngine`` (or any object with its request API:
    ``k``, ``add_requests``, ``prefill``, ``step``, ``release``, ``draws_used``)."""

    def __init__(self, engine, stop_token_ids=()) -> None:
        self.engine = engine
        self.k = engine.k
        self.stop_token_ids = frozenset(stop_token_ids)
        self._slots: dict[str, int] = {}   # request id -> engine slot
        self._draws: dict[str, int] = {}   # request id -> Philox draws used before it was preempted

    @property
    def num_active(self) -> int:
        return len(self._slots)

    def slot_of(self, sequence) -> int | None:
        return self._slots.get(sequence.request_id)

    def _load(self, sequences: list) -> list[int]:
        """Load sequences into free engine slots: the whole history as the prompt (a preempted
        sequence is recomputed from its tokens, as the reference's ``forget_cache`` asks), the
        remaining new-token budget, and the request's sampling parameters; one ``add_requests``
        call per distinct parameter set, in plan order within each."""
        groups: dict[tuple, list[int]] = {}
        for i, seq in enumerate(sequences):
            if seq.request_id in self._slots:
                raise RuntimeError(f"request {seq.request_id} is already loaded")
            p = seq.sampling_params
            groups.setdefault((bool(p.ignore_eos), float(p.temperature), float(p.top_p)), []).append(i)
        slots: list[int] = [0] * len(sequences)
        for (ignore_eos, temperature, top_p), members in groups.items():
            seqs = [sequences[i] for i in members]
            got = self.engine.add_requests(
                [list(s.token_ids) for s in seqs],
                [s.sampling_params.max_new_tokens - s.num_generated_tokens for s in seqs],
                ignore_eos=ignore_eos, temperature=temperature, top_p=top_p,
                seeds=[request_seed(s) for s in seqs], draws=[self._draws.pop(s.request_id, 0) for s in seqs])
            for i, slot in zip(members, got):
                slots[i] = slot
                self._slots[sequences[i].request_id] = slot
        return slots

    def prefill(self, sequences: list) -> list[tuple[object, int]]:
        """A prefill plan: every sequence caches all its tokens and yields its next token."""
        if not sequences:
            return []
        slots = self._load(sequences)
        # prompts longer than one prefill call take several (chunked within the plan)
        res = self.engine.prefill(slots, chunk=getattr(self.engine, "max_prefill_rows", None))
        out = []
        for seq, slot in zip(sequences, slots):
            tokens = res.tokens[slot]
            if len(tokens) != 1:
                raise RuntimeError(f"prefill of {seq.request_id} returned {len(tokens)} tokens")
            seq.num_cached_tokens = len(seq.token_ids)
            out.append((seq, tokens[0]))
        return out

    def step(self, sequences: list) -> list[tuple[object, int]]:
        """A decode plan: one speculative step per sequence; its emitted tokens in order, sequence
        by sequence (``num_cached_tokens`` set to what the step leaves cached: every token but the
        last emitted one)."""
        if not sequences:
            return []
        missing = [s.request_id for s in sequences if s.request_id not in self._slots]
        if missing:
            raise RuntimeError(f"decode plan lists requests that were never prefilled: {missing}")
        slots = [self._slots[s.request_id] for s in sequences]
        res = self.engine.step(slots)
        out = []
        for seq, slot in zip(sequences, slots):
            tokens = res.tokens[slot]
            seq.num_cached_tokens = len(seq.token_ids) + len(tokens) - 1
            out.extend((seq, t) for t in tokens)
        return out

    def execute(self, plan) -> list[tuple[object, int]]:
        """A scheduler's ``StepPlan`` (batch_scheduler.py:19-27): prefill plans and decode plans;
        prompt chunks are a chunked-prefill scheduler's and are refused."""
        if getattr(plan, "prefill_chunks", None):
            raise ValueError("the speculative batch step serves whole prefills (no chunked-prefill scheduler)")
        return self.prefill(list(plan.sequences)) if plan.is_prefill else self.step(list(plan.sequences))

    def release(self, sequence) -> None:
        """Free the sequence's engine slot (finished, failed or preempted); a sampled request keeps
        the count of uniforms it drew, so that it resumes its Philox stream where it stopped."""
        slot = self._slots.pop(sequence.request_id, None)
        if slot is None:
            return
        if sequence.sampling_params.temperature > 0.0 and not self._finished(sequence):
            self._draws[sequence.request_id] = int(self.engine.draws_used(slot))
        self.engine.release([slot])

    def _finished(self, sequence) -> bool:
        """Whether the sequence's last token finished it (``find_finish_reason``, engine/sampling.py:54-62)."""
        params = sequence.sampling_params
        if sequence.num_generated_tokens >= params.max_new_tokens:
            return True
        return (sequence.num_generated_tokens > 0 and not params.ignore_eos
                and sequence.token_ids[-1] in self.stop_token_ids)


class GuessRoomAllocator:
    """A scheduler's slot allocator (the reference's ``SlotAllocator`` protocol,
    engine/memory/slot_allocator.py) whose reservations include the request's guess room, and
    whose ``free`` also frees the request's engine slot. Everything else is the wrapped
    allocator's."""

    def __init__(self, inner, executor: SpeculativeBatchExecutor) -> None:
        self._inner = inner
        self._executor = executor

    def _need(self, sequence, num_tokens: int) -> int:
        return num_tokens + guess_room(sequence, self._executor.k)

    def can_reserve(self, sequence, num_tokens: int) -> bool:
        return self._inner.can_reserve(sequence, self._need(sequence, num_tokens))

    def reserve(self, sequence, num_tokens: int) -> None:
        self._inner.reserve(sequence, self._need(sequence, num_tokens))

    def free(self, sequence) -> None:
        self._executor.release(sequence)
        self._inner.free(sequence)

    def __getattr__(self, name):
        return getattr(self._inner, name)
