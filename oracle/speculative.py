"""Serial speculative generation over a paged KV cache, restated (TEST INFRASTRUCTURE).

Follows (paths relative to ``nanoengine/src/nanoengine``):

* ``BlockAllocator``                     engine/memory/block_allocator.py:8-33   FIFO free list
* ``PagedSlotAllocator``                 engine/memory/paged_allocator.py:21-79  block tables
* ``build_step_inputs``                  engine/generation/batch_builder.py:22-65
* ``ModelRunner.run_step`` / ``score_tokens`` / ``_sample``
                                         engine/generation/model_runner.py:33-80
* ``SpeculativeGenerator._generate`` / ``_run_speculative_step``
                                         engine/speculative/speculative_generator.py:50-85
* ``find_finish_reason``                 engine/sampling.py:54-62
* ``DraftModelProposer``                 engine/speculative/proposers.py:63-106 (``DraftProposer``)

Every step is recorded (draft, block table after the reservation, verify logits, emitted tokens,
``num_cached_tokens`` after the rollback), which is what the parity tests compare.
The random draws come from an injected uniform iterator (see ``oracle/verify.py``).
"""

from __future__ import annotations

import math
from collections import deque
from dataclasses import dataclass, field

import torch

from . import ngram, qwen3, verify

PADDING_TOKEN_ID = 0


class OutOfBlocks(Exception):
    pass


class BlockFIFO:
    """engine/memory/block_allocator.py:8-33."""

    def __init__(self, num_blocks: int) -> None:
        self.num_blocks = num_blocks
        self.free_blocks: deque[int] = deque(range(num_blocks))
        self.used: set[int] = set()

    def allocate(self) -> int:
        if not self.free_blocks:
            raise OutOfBlocks("no free KV blocks")
        block = self.free_blocks.popleft()
        self.used.add(block)
        return block

    def free(self, block: int) -> None:
        if block not in self.used:
            raise ValueError(f"block {block} is not allocated")
        self.used.remove(block)
        self.free_blocks.append(block)


class PagedTables:
    """engine/memory/paged_allocator.py:21-79."""

    def __init__(self, num_blocks: int, block_size: int) -> None:
        self.block_size = block_size
        self.blocks = BlockFIFO(num_blocks)
        self.tables: dict[str, list[int]] = {}

    def missing(self, rid: str, num_tokens: int) -> int:
        return max(0, math.ceil(num_tokens / self.block_size) - len(self.tables.get(rid, [])))

    def reserve(self, rid: str, num_tokens: int) -> None:
        if self.missing(rid, num_tokens) > len(self.blocks.free_blocks):
            raise OutOfBlocks(f"no blocks for {num_tokens} tokens of {rid}")
        table = self.tables.setdefault(rid, [])
        for _ in range(self.missing(rid, num_tokens)):
            table.append(self.blocks.allocate())

    def free(self, rid: str) -> None:
        for block in self.tables.pop(rid, []):
            self.blocks.free(block)

    def context_slots(self, rids: list[str], context_length: int) -> torch.Tensor:
        per_row = math.ceil(context_length / self.block_size)
        rows = []
        for rid in rids:
            table = self.tables[rid][:per_row]
            rows.append(table + [0] * (per_row - len(table)))
        tables = torch.tensor(rows, dtype=torch.int64)
        positions = torch.arange(context_length)
        return tables[:, positions // self.block_size] * self.block_size + positions % self.block_size


@dataclass
class Seq:
    """engine/sequence_state.py:12-57 (the fields the speculative path reads)."""

    request_id: str
    token_ids: list[int]
    num_prompt_tokens: int
    max_new_tokens: int
    temperature: float = 0.0
    top_p: float = 1.0
    ignore_eos: bool = False
    num_cached_tokens: int = 0

    @property
    def num_tokens(self) -> int:
        return len(self.token_ids)

    @property
    def num_generated_tokens(self) -> int:
        return len(self.token_ids) - self.num_prompt_tokens


def finish_reason(token_id: int, seq: Seq, stop_token_ids: frozenset[int]) -> str | None:
    """engine/sampling.py:54-62."""
    if not seq.ignore_eos and token_id in stop_token_ids:
        return "stop"
    if seq.num_generated_tokens >= seq.max_new_tokens:
        return "length"
    return None


class OracleRunner:
    """engine/generation/model_runner.py:14-80 over ``oracle.qwen3`` and ``PagedTables``."""

    def __init__(self, weights, cfg, num_blocks: int, block_size: int, dtype, int8_kv=False):
        self.weights = weights
        self.cfg = cfg
        self.tables = PagedTables(num_blocks, block_size)
        self.pool = qwen3.KVPool.create(cfg, num_blocks * block_size, dtype, int8_kv)

    def step_inputs(self, seqs: list[Seq], counts: list[int]):
        """engine/generation/batch_builder.py:22-65."""
        ends = [s.num_cached_tokens + c for s, c in zip(seqs, counts)]
        q_len, c_len = max(counts), max(ends)
        token_rows, position_rows = [], []
        for s, end in zip(seqs, ends):
            start = s.num_cached_tokens
            pad = [PADDING_TOKEN_ID] * (q_len - (end - start))
            token_rows.append(s.token_ids[start:end] + pad)
            position_rows.append(list(range(start, end)) + pad)
        token_ids = torch.tensor(token_rows, dtype=torch.int64)
        positions = torch.tensor(position_rows, dtype=torch.int64)
        real = torch.arange(q_len)[None, :] < torch.tensor(counts)[:, None]
        context_slots = self.tables.context_slots([s.request_id for s in seqs], c_len)
        slot_mapping = context_slots.gather(1, positions).masked_fill(~real, self.pool.scratch_slot)
        mask = qwen3.attention_mask(positions, torch.tensor(ends), c_len)
        return token_ids, qwen3.StepContext(positions, slot_mapping, context_slots, mask)

    @torch.inference_mode()
    def forward_rows(self, seqs: list[Seq], counts: list[int]) -> torch.Tensor:
        """Cache ``counts[i]`` tokens of each sequence; final hidden states ``[b, q, H]``."""
        token_ids, ctx = self.step_inputs(seqs, counts)
        hidden = qwen3.forward(self.weights, self.cfg, token_ids, ctx, self.pool)
        for s, c in zip(seqs, counts):
            s.num_cached_tokens += c
        return hidden

    @torch.inference_mode()
    def run_step(self, seqs: list[Seq], uniforms_by_seq=None, stable: bool = False) -> tuple[list[int], torch.Tensor]:
        """model_runner.py:33-50,64-80: prefill all uncached tokens, sample one token each."""
        counts = [s.num_tokens - s.num_cached_tokens for s in seqs]
        hidden = self.forward_rows(seqs, counts)
        last = hidden[torch.arange(len(seqs)), torch.tensor(counts) - 1]
        logits = qwen3.compute_logits(self.weights, self.cfg, last)
        tokens = torch.argmax(logits, dim=-1).tolist()
        for row, s in enumerate(seqs):
            if s.temperature != verify.GREEDY_TEMPERATURE:
                probs = verify.token_probabilities(logits[row], s.temperature, s.top_p, stable)
                tokens[row] = verify.inverse_cdf(probs, next(uniforms_by_seq[row]))
        return tokens, logits

    @torch.inference_mode()
    def score_tokens(self, seq: Seq, count: int) -> torch.Tensor:
        """model_runner.py:52-62: logits after each of the next ``count`` tokens."""
        hidden = self.forward_rows([seq], [count])
        return qwen3.compute_logits(self.weights, self.cfg, hidden[0, :count])


class DraftProposer:
    """engine/speculative/proposers.py:63-106: a draft model of the same family runs
    ``num_tokens`` steps ahead of the target on its own paged cache (``runner``); the first step
    catches up on the tokens the target added. Greedy drafts are the draft's argmax; sampled ones
    are drawn from the request's uniform stream (the same stream verification reads)."""

    def __init__(self, runner: OracleRunner, stable: bool = False) -> None:
        self.runner = runner
        self.stable = stable
        self.drafts: dict[str, Seq] = {}

    def propose(self, seq: Seq, num_tokens: int, uniforms) -> tuple[list[int], torch.Tensor | None]:
        draft = self._sync(seq)
        guesses: list[int] = []
        distributions = []
        for _ in range(num_tokens):
            self.runner.tables.reserve(draft.request_id, draft.num_tokens)
            logits = self.runner.score_tokens(draft, draft.num_tokens - draft.num_cached_tokens)[-1]
            probabilities = verify.token_probabilities(logits, seq.temperature, seq.top_p, self.stable)
            if seq.temperature == verify.GREEDY_TEMPERATURE:
                guess = int(torch.argmax(probabilities).item())
            else:
                guess = verify.inverse_cdf(probabilities, next(uniforms))
            draft.token_ids.append(guess)
            guesses.append(guess)
            distributions.append(probabilities)
        return guesses, torch.stack(distributions) if distributions else None

    def release(self, seq: Seq) -> None:
        if self.drafts.pop(seq.request_id, None) is not None:
            self.runner.tables.free(seq.request_id)

    def _sync(self, seq: Seq) -> Seq:
        """proposers.py:93-106: the draft's tokens become the target's; its cache is kept for
        the common prefix."""
        draft = self.drafts.get(seq.request_id)
        if draft is None:
            draft = Seq(seq.request_id, list(seq.token_ids[: seq.num_prompt_tokens]), seq.num_prompt_tokens,
                        seq.max_new_tokens, seq.temperature, seq.top_p, seq.ignore_eos)
            self.drafts[seq.request_id] = draft
        common = 0
        for a, b in zip(draft.token_ids, seq.token_ids):
            if a != b:
                break
            common += 1
        draft.token_ids = list(seq.token_ids)
        draft.num_cached_tokens = min(draft.num_cached_tokens, common)
        return draft


@dataclass
class StepRecord:
    draft: list[int]
    block_table: list[int]
    logits: torch.Tensor
    new_tokens: list[int]
    num_cached_tokens: int
    uniforms_used: int = 0


@dataclass
class Generation:
    tokens: list[int] = field(default_factory=list)
    finish_reason: str | None = None
    prefill_block_table: list[int] = field(default_factory=list)
    prefill_logits: torch.Tensor | None = None
    steps: list[StepRecord] = field(default_factory=list)
    proposed: int = 0
    accepted: int = 0


class _CountingStream:
    def __init__(self, inner) -> None:
        self.inner = inner
        self.count = 0

    def __iter__(self):
        return self

    def __next__(self) -> float:
        self.count += 1
        return next(self.inner)


def generate(
    runner: OracleRunner,
    seq: Seq,
    num_speculative_tokens: int,
    max_ngram: int,
    stop_token_ids: frozenset[int] = frozenset(),
    uniforms=None,
    keep_logits: bool = True,
    free_at_end: bool = True,
    stable: bool = False,
    proposer: DraftProposer | None = None,
) -> Generation:
    """engine/speculative/speculative_generator.py:42-85 with ``NgramProposer`` drafts, or the
    draft model's (``proposer``) (``stable``: top-p ties by ascending id, as
    ``verify.apply_top_p`` documents)."""
    stream = _CountingStream(uniforms if uniforms is not None else iter(()))
    out = Generation()
    try:
        runner.tables.reserve(seq.request_id, seq.num_tokens)
        out.prefill_block_table = list(runner.tables.tables[seq.request_id])
        new_tokens, logits = runner.run_step([seq], [stream], stable)
        out.prefill_logits = logits[0] if keep_logits else None
        while True:
            for token in new_tokens:
                seq.token_ids.append(token)
                out.tokens.append(token)
                reason = finish_reason(token, seq, stop_token_ids)
                if reason is not None:
                    out.finish_reason = reason
                    return out
            before = stream.count
            remaining = seq.max_new_tokens - seq.num_generated_tokens
            num_guesses = max(0, min(num_speculative_tokens, remaining - 1))
            draft_probabilities = None
            if proposer is not None:
                draft, draft_probabilities = proposer.propose(seq, num_guesses, stream) if num_guesses else ([], None)
            else:
                draft = ngram.propose(seq.token_ids, num_guesses, max_ngram) if num_guesses else []
            length_before = seq.num_tokens
            seq.token_ids.extend(draft)
            runner.tables.reserve(seq.request_id, seq.num_tokens)
            table = list(runner.tables.tables[seq.request_id])
            target_logits = runner.score_tokens(seq, 1 + len(draft))
            new_tokens = verify.verify_proposal(
                draft, draft_probabilities, target_logits, seq.temperature, seq.top_p, stream, stable
            )
            kept = len(new_tokens) - 1
            del seq.token_ids[length_before:]
            seq.num_cached_tokens = length_before + kept
            out.proposed += len(draft)
            out.accepted += kept
            out.steps.append(
                StepRecord(
                    draft=list(draft),
                    block_table=table,
                    logits=target_logits if keep_logits else torch.empty(0),
                    new_tokens=list(new_tokens),
                    num_cached_tokens=seq.num_cached_tokens,
                    uniforms_used=stream.count - before,
                )
            )
    finally:
        if free_at_end:
            runner.tables.free(seq.request_id)
        if proposer is not None:
            proposer.release(seq)
