"""A CPU stand-in for ``B200SpeculativeEngine``'s request API, for host-side tests of the code that
drives the engine (the batch executor and the nanoengine loop binding).

Test infrastructure only: each request's whole speculative generation is computed up front by the
CPU oracle (``oracle.speculative.generate``, the reference's serial speculative path restated) and
then handed out one step at a time, as the engine's ``prefill`` / ``step`` would hand it out: the
first token at prefill, then each step's kept guesses plus one, cut at a stop token or the length
limit. A request that is released and loaded again (a preemption) is generated again from its
whole history, which is what the engine does with a reloaded request.
"""

from __future__ import annotations

import torch

from oracle import speculative as oracle_spec
from tests.conftest import submodule


class OracleSpecEngine:
    def __init__(self, weights, cfg, k: int, max_ngram: int, max_seqs: int, stop_token_ids=(),
                 max_prefill_rows: int = 4096, draft=None) -> None:
        """``draft``: (config, weights) of a draft model whose greedy guesses replace the n-gram
        lookup (DraftModelProposer)."""
        self.weights, self.cfg, self.draft = weights, cfg, draft
        self.k, self.max_ngram, self.max_seqs = k, max_ngram, max_seqs
        self.stop = frozenset(stop_token_ids)
        self.max_prefill_rows = max_prefill_rows
        self.free = list(range(max_seqs))
        self.chunks: dict[int, list[tuple[list[int], str | None, int]]] = {}
        self.loaded: list[list[int]] = []  # every history loaded, in order
        self.proposed_total = self.accepted_total = 0
        self.steps_run = 0

    def add_requests(self, prompts, max_new_tokens, *, ignore_eos=False, temperature=0.0, top_p=1.0, seeds=None,
                     draws=None, prefix=None):
        if temperature != 0.0:
            raise ValueError("the oracle stand-in serves greedy requests")
        if len(prompts) > len(self.free):
            raise RuntimeError("no free sequence slot")
        slots = []
        for prompt, new in zip(prompts, max_new_tokens):
            slot = self.free.pop(0)
            runner = oracle_spec.OracleRunner(self.weights, self.cfg, 512, 16, torch.float32)
            seq = oracle_spec.Seq(f"slot{slot}", list(prompt), len(prompt), new, ignore_eos=ignore_eos)
            proposer = None
            if self.draft is not None:
                draft_cfg, draft_weights = self.draft
                proposer = oracle_spec.DraftProposer(
                    oracle_spec.OracleRunner(draft_weights, draft_cfg, 512, 16, torch.float32))
            gen = oracle_spec.generate(runner, seq, self.k, self.max_ngram, self.stop, keep_logits=False,
                                       proposer=proposer)
            pieces = [([gen.tokens[0]], 0)] + [(list(s.new_tokens), len(s.draft)) for s in gen.steps]
            chunks, emitted = [], 0
            for piece, proposed in pieces:  # cut at the generation's end (a stop inside a step's kept run)
                take = piece[: len(gen.tokens) - emitted]
                if not take:
                    break
                emitted += len(take)
                chunks.append((take, gen.finish_reason if emitted == len(gen.tokens) else None, proposed))
            self.chunks[slot] = chunks
            self.loaded.append(list(prompt))
            slots.append(slot)
        return slots

    def _serve(self, slots):
        res = submodule("engine").StepResult()
        for slot in slots:
            tokens, finish, proposed = self.chunks[slot].pop(0)
            res.tokens[slot] = tokens
            res.finish[slot] = finish
            res.proposed += proposed
            res.accepted += len(tokens) - 1 if proposed else 0
        self.proposed_total += res.proposed
        self.accepted_total += res.accepted
        self.steps_run += 1
        return res

    def prefill(self, slots, prompt_lengths=None, chunk=None):
        return self._serve(slots)

    def step(self, slots):
        return self._serve(slots)

    def draws_used(self, slot: int) -> int:
        return 0

    def release(self, slots) -> None:
        for slot in slots:
            self.chunks.pop(slot, None)
            self.free.append(slot)
