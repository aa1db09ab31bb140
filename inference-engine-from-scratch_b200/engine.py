"""Batched speculative decoding on the B200 kernels: the drop-in for the runner's speculative step.

``B200SpeculativeEngine.step(slots)`` runs, for every listed sequence slot and entirely on the GPU,
what ``SpeculativeGenerator._run_speculative_step`` does for one sequence
(engine/speculative/speculative_generator.py:70-85): n-gram draft with the guess cap
``min(k, remaining - 1)``, block reservation for the guesses, one (k+1)-token verify forward,
acceptance (greedy, or rejection sampling on each request's Philox stream where temperature > 0),
and the commit ``num_cached = len_before + kept``; then the emission / finish loop of
``_generate`` (:54-67). Per-sequence results equal the serial reference's, since batching changes
no per-request arithmetic. With ``cuda_graphs`` every batch bucket (engine/generation/
cuda_graph_runner.py:26 buckets) is captured once and replayed.

Each step copies the step's batch-slot list host->device and reads the packed results
device->host (tokens, counts, finish reasons, proposed / accepted) in one copy.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import _lib
from .model import B200Model
from .state import DeviceBatchState

BATCH_SIZE_BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256)
FINISH_REASONS = {_lib.NE_FINISH_STOP: "stop", _lib.NE_FINISH_LENGTH: "length"}


def build_buckets(largest: int, candidates=BATCH_SIZE_BUCKETS) -> list[int]:
    """engine/generation/cuda_graph_runner.py:35-36."""
    return sorted({v for v in candidates if v < largest} | {largest})


def round_up_to_bucket(value: int, buckets: list[int]) -> int:
    return next(b for b in buckets if b >= value)


@dataclass
class StepResult:
    """Per listed slot: emitted tokens, finish reason (None while running), guesses proposed / kept."""

    tokens: dict[int, list[int]] = field(default_factory=dict)
    finish: dict[int, str | None] = field(default_factory=dict)
    proposed: int = 0
    accepted: int = 0


class _Outputs:
    """One flat int32 buffer: tokens [B, k+1] | count [B] | finish [B] | proposed [B] | accepted [B]."""

    def __init__(self, max_seqs: int, k: int, device) -> None:
        self.k = k
        self.max_seqs = max_seqs
        w = k + 1
        self.buf = torch.zeros(max_seqs * (w + 4), dtype=torch.int32, device=device)
        self.host = torch.zeros_like(self.buf, device="cpu").pin_memory()
        n = max_seqs
        base = self.buf.data_ptr()
        self.struct = _lib.StepOutputs(
            tokens=base, count=base + 4 * n * w, finish=base + 4 * n * (w + 1),
            proposed=base + 4 * n * (w + 2), accepted=base + 4 * n * (w + 3),
        )

    def start_fetch(self) -> None:
        """Enqueue the device->host copy of the results and an event after it (no host wait)."""
        self.host.copy_(self.buf, non_blocking=True)
        self.event = torch.cuda.Event()
        self.event.record()

    def fetch(self, num: int):
        """Copy the whole buffer device->host (unless start_fetch did) and split it (one D2H per step)."""
        if getattr(self, "event", None) is None:
            self.start_fetch()
        self.event.synchronize()
        self.event = None
        n, w = self.max_seqs, self.k + 1
        h = self.host
        tokens = h[: n * w].view(n, w)[:num]
        count = h[n * w: n * (w + 1)][:num]
        finish = h[n * (w + 1): n * (w + 2)][:num]
        proposed = h[n * (w + 2): n * (w + 3)][:num]
        accepted = h[n * (w + 3): n * (w + 4)][:num]
        return tokens, count, finish, proposed, accepted


class B200SpeculativeEngine:
    def __init__(
        self,
        model: B200Model,
        k: int = 4,
        max_ngram: int = 3,
        max_seqs: int = 64,
        max_model_len: int = 4096,
        num_blocks: int | None = None,
        stop_token_ids=(),
        cuda_graphs: bool = True,
        max_prefill_rows: int | None = None,
        sampling: bool = False,
        draft_model: B200Model | None = None,
        draft_num_blocks: int | None = None,
    ) -> None:
        """``draft_model``: drafts come from this smaller model of the same family
        (DraftModelProposer, engine/speculative/proposers.py:63-106; greedy requests) instead of
        n-gram lookup; it keeps its own batch state and KV pool (``draft_num_blocks`` blocks)."""
        self.lib = _lib.load()
        self.model = model
        self.k = k
        self.max_ngram = max_ngram
        self.max_seqs = max_seqs
        if model.max_seqs < max_seqs or model.max_rows < max_seqs * (k + 1):
            raise ValueError("the model workspace is smaller than max_seqs x (k + 1) rows")
        if max_model_len + k + 1 > model.max_positions:
            raise ValueError("max_model_len + k exceeds the RoPE table")
        blocks = num_blocks if num_blocks is not None else model.num_slots // 16
        if blocks * 16 > model.num_slots:
            raise ValueError("more blocks than the KV pool holds")
        self.state = DeviceBatchState(max_seqs, max_model_len, k, blocks, 16, stop_token_ids, model.device)
        # two result buffers: generate() reads step i's results while step i + 1 runs
        self._outs = [_Outputs(max_seqs, k, model.device), _Outputs(max_seqs, k, model.device)]
        self.outputs = self._outs[0]
        self.max_prefill_rows = min(max_prefill_rows or model.max_rows, model.max_rows)
        self.buckets = build_buckets(max_seqs)
        self.cuda_graphs = cuda_graphs
        self._slots_dev = torch.full((max_seqs,), -1, dtype=torch.int32, device=model.device)
        self._dev_slots_key = None  # (slots, bucket) the device slot list holds
        self._slots_hosts = [torch.full((max_seqs,), -1, dtype=torch.int32).pin_memory() for _ in range(2)]
        self._slots_host = self._slots_hosts[0]
        self._graphs: dict[tuple[int, int], torch.cuda.CUDAGraph] = {}
        # sampled requests (temperature > 0) need every lm row's logits: bind a sampling buffer
        # (bound to the model before each eager launch or capture, since engines may share a model)
        self.sampling = sampling
        self._sample_rows = max_seqs * (k + 1)
        self._sample_buf = None
        if sampling:
            nbytes = int(self.lib.ne_sampling_buffer_bytes(model.handle, self._sample_rows))
            self._sample_buf = torch.empty(nbytes, dtype=torch.uint8, device=model.device)
        # draft model: its own batch state (same slots and history stride) and result buffer
        self.draft_model = draft_model
        self.draft_state = None
        if draft_model is not None:
            if draft_model is model:
                raise ValueError("the draft model needs a model object (and KV pool) of its own")
            if draft_model.cfg.vocab_size != model.cfg.vocab_size:
                raise ValueError("the draft model needs the target's vocabulary")
            if draft_model.max_seqs < max_seqs or draft_model.max_rows < max_seqs * (k + 1):
                raise ValueError("the draft model workspace is smaller than max_seqs x (k + 1) rows")
            if max_model_len + k + 1 > draft_model.max_positions:
                raise ValueError("max_model_len + k exceeds the draft model's RoPE table")
            dblocks = draft_num_blocks if draft_num_blocks is not None else draft_model.num_slots // 16
            if dblocks * 16 > draft_model.num_slots:
                raise ValueError("more draft blocks than the draft KV pool holds")
            self.draft_state = DeviceBatchState(max_seqs, max_model_len, k, dblocks, 16, (), model.device)
            self._draft_outs = _Outputs(max_seqs, k, model.device)
            self.max_prefill_rows = min(self.max_prefill_rows, draft_model.max_rows)
            self._draft_rows = None
            if sampling:
                # sampled drafts: each of the k draft steps keeps its rows (one per entry) in its own
                # region of one buffer, regions a whole number of vocabulary rows apart, for the
                # verification against the draft's distributions
                row_bytes = 2 * draft_model.cfg.vocab_size
                need = int(self.lib.ne_sampling_buffer_bytes(draft_model.handle, max_seqs))
                self._region_rows = -(-need // row_bytes)
                self._region_bytes = self._region_rows * row_bytes
                self._draft_regions = torch.empty(k * self._region_bytes, dtype=torch.uint8, device=model.device)
                self._draft_stats = torch.empty(k * self._region_rows * 32, dtype=torch.uint8, device=model.device)
        self._uncached: dict[int, int] = {}       # slot -> prompt tokens still to prefill
        self._prefixes: dict[int, list] = {}      # holder slot -> [tokens, shared blocks, users, copies]
        self._prefix_of: dict[int, int] = {}      # slot -> holder slot of its shared prefix
        self._shared_count: dict[int, int] = {}   # slot -> blocks it shares with its prefix holder
        self.proposed_total = 0
        self.accepted_total = 0
        self.h2d_bytes = 0  # host->device bytes copied for requests and steps
        self.d2h_bytes = 0  # device->host bytes read back (step results)
        self.steps_run = 0  # prefill and speculative steps whose results were read
        self.preemptions = 0  # sequences generate() preempted to free KV blocks

    # ------------------------------------------------------------------ request lifecycle
    def add_request(self, prompt: list[int], max_new_tokens: int, *, ignore_eos: bool = False,
                    temperature: float = 0.0, top_p: float = 1.0, seed: int = 0, prefix: int | None = None,
                    draws: int = 0) -> int:
        """Load a request into a free slot. ``seed`` keys the request's Philox stream (``draws``:
        the uniforms it already used, for a preempted request that resumes); ``prefix`` (from
        ``add_prefix``) shares the KV blocks of a prompt prefix the request starts with."""
        return self.add_requests([prompt], [max_new_tokens], ignore_eos=ignore_eos, temperature=temperature,
                                 top_p=top_p, seeds=[seed], prefix=prefix, draws=[draws])[0]

    def add_requests(self, prompts: list[list[int]], max_new_tokens: list[int], *, ignore_eos: bool = False,
                     temperature: float = 0.0, top_p: float = 1.0, seeds: list[int] | None = None,
                     prefix: int | None = None, draws: list[int] | None = None) -> list[int]:
        """``add_request`` for many requests at once, in order: one host->device copy per field
        for all of them, and one block-sharing launch per shared-block count."""
        n = len(prompts)
        seeds = list(seeds) if seeds is not None else [0] * n
        draws = list(draws) if draws is not None else [0] * n
        if len(max_new_tokens) != n or len(seeds) != n or len(draws) != n:
            raise ValueError("one max_new_tokens, seed and draws value per prompt")
        if temperature != 0.0 and not self.sampling:
            raise ValueError("temperature > 0 needs an engine built with sampling=True")
        if self.draft_state is not None and prefix is not None:
            raise ValueError("draft-model drafts serve requests without shared prefixes")
        if prefix is not None:
            tokens = self._prefixes[prefix][0]
            if any(p[: len(tokens)] != tokens for p in prompts):
                raise ValueError("the prompt does not start with the shared prefix")
        if n > len(self.state.free_slots):
            raise RuntimeError("no free sequence slot")
        for prompt, new in zip(prompts, max_new_tokens):  # (checked before any slot is taken)
            if len(prompt) == 0 or len(prompt) + new > self.state.max_model_len:
                raise ValueError(f"prompt of {len(prompt)} + {new} new tokens exceeds max_model_len")
        slots = [self.state.acquire() for _ in range(n)]
        self.state.load_many(slots, prompts, list(max_new_tokens), ignore_eos=[ignore_eos] * n,
                             temperature=[temperature] * n, top_p=[top_p] * n, seed=seeds, draws=draws)
        per_request = 5 * 4 + 4 + 4 + 8 + 8
        self.h2d_bytes += sum(4 * len(p) + per_request for p in prompts)
        groups: dict[int, list[int]] = {}
        for slot, prompt in zip(slots, prompts):
            shared = 0
            if prefix is not None:
                # whole blocks only, and at least one prompt token left to prefill (it yields the first token)
                blocks = min(self._prefixes[prefix][1], (len(prompt) - 1) // 16)
                groups.setdefault(blocks, []).append(slot)
                self._prefixes[prefix][2] += 1
                self._prefix_of[slot] = prefix
                self._shared_count[slot] = blocks
                shared = blocks * 16
            self._uncached[slot] = len(prompt) - shared
        for blocks, group in groups.items():
            self.state.share_blocks(prefix, group, blocks)
        if self.draft_state is not None:
            # the draft sequence never finishes on its own: it follows the target (ne_draft_sync)
            self.draft_state.load_many(slots, prompts, [self.state.max_model_len - len(p) for p in prompts],
                                       ignore_eos=[True] * n, temperature=[temperature] * n, top_p=[top_p] * n,
                                       seed=seeds, draws=draws)
            self.draft_state.max_new_tokens[torch.tensor(slots, device=self.model.device)] = 1 << 30
            self.h2d_bytes += sum(4 * len(p) + per_request for p in prompts)
        return slots

    def add_prefix(self, tokens: list[int]) -> int:
        """Prefill a prompt prefix once (its own slot holds the blocks); requests that start with it
        pass the returned handle as ``prefix`` and reuse its full 16-token blocks."""
        holder = self.add_request(tokens, 1, ignore_eos=True)
        self.prefill([holder])
        blocks = len(tokens) // 16
        # int8 KV: dequantise the shared blocks once (the attention reads the copies)
        first = self.model.take_kv_copies(blocks) if blocks else None
        if first is not None:
            _lib.check(self.lib.ne_kv_shadow_fill(self.model.handle, self.state.ref, holder, blocks, first,
                                                  _lib.stream_handle()), "ne_kv_shadow_fill")
        self._prefixes[holder] = [list(tokens), blocks, 0, first]
        return holder

    def drop_prefix(self, prefix: int) -> None:
        if self._prefixes[prefix][2]:
            raise RuntimeError("requests still share this prefix")
        _, blocks, _, first = self._prefixes.pop(prefix)
        if first is not None:  # unmap before the holder's blocks return to the pool
            _lib.check(self.lib.ne_kv_shadow_clear(self.model.handle, self.state.ref, prefix, blocks,
                                                   _lib.stream_handle()), "ne_kv_shadow_clear")
            self.model.return_kv_copies(first, blocks)
        self.state.release([prefix])

    def _bind_sampler(self) -> None:
        buf = self._sample_buf
        _lib.check(self.lib.ne_model_set_sampling_buffer(
            self.model.handle, _lib.ptr(buf), 0 if buf is None else buf.numel(), self._sample_rows),
            "ne_model_set_sampling_buffer")

    def sampled_logits(self, rows: int) -> torch.Tensor:
        """The last sampled step's target logits ``[rows, vocab]`` (bf16, lm-row order)."""
        if self._sample_buf is None:
            raise ValueError("the engine was built without sampling")
        vocab = self.model.cfg.vocab_size
        return self._sample_buf[: rows * vocab * 2].view(torch.bfloat16).view(rows, vocab)

    def draft_logits(self, num_entries: int) -> tuple[torch.Tensor, list[int]]:
        """The last sampled draft-model step's draft rows: ``[k, rows, vocab]`` bf16 (draft step j
        in region j) and, per batch entry, its row in every region."""
        if self.draft_state is None or not self.sampling:
            raise ValueError("the engine has no sampled draft model")
        vocab = self.draft_model.cfg.vocab_size
        regions = self._draft_regions.view(torch.bfloat16).view(self.k, -1)[:, : self._region_rows * vocab]
        start = _lib.device_int32(self.lib.ne_model_lm_start(self.draft_model.handle), num_entries, self.model.device)
        return regions.reshape(self.k, self._region_rows, vocab), start.cpu().tolist()

    def draws_used(self, slot: int) -> int:
        """Uniforms the request in ``slot`` has drawn from its Philox stream so far (one device read)."""
        return int(self.state.rng_draws[slot].item())

    def release(self, slots: list[int]) -> None:
        self.state.release(slots)
        if self.draft_state is not None:
            self.draft_state.release(slots)
        for s in slots:
            self._uncached.pop(s, None)
            self._shared_count.pop(s, None)
            holder = self._prefix_of.pop(s, None)
            if holder is not None:
                self._prefixes[holder][2] -= 1

    def _set_slots(self, slots: list[int], bucket: int, host: int = 0) -> None:
        # consecutive steps usually list the same slots: the device copy is then already current
        key = (tuple(slots), bucket)
        if key == self._dev_slots_key:
            return
        # the pinned source of an asynchronous copy must not change before the copy runs: the two
        # in-flight steps of generate() use two host buffers
        h = self._slots_hosts[host]
        h.fill_(-1)
        h[: len(slots)] = torch.tensor(slots, dtype=torch.int32)
        self._slots_dev[:bucket].copy_(h[:bucket], non_blocking=True)
        self._dev_slots_key = key
        self.h2d_bytes += 4 * bucket

    def _collect(self, slots: list[int], outs: _Outputs | None = None) -> StepResult:
        outs = outs or self.outputs
        tokens, count, finish, proposed, accepted = outs.fetch(len(slots))
        self.d2h_bytes += outs.buf.numel() * 4
        self.steps_run += 1
        result = StepResult()
        # one host conversion per field (per-slot tensor slicing costs more than the step's GPU time)
        rows, counts, fins = tokens.tolist(), count.tolist(), finish.tolist()
        for i, slot in enumerate(slots):
            result.tokens[slot] = rows[i][: counts[i]]
            result.finish[slot] = FINISH_REASONS.get(fins[i])
        result.proposed = sum(proposed.tolist())
        result.accepted = sum(accepted.tolist())
        self.proposed_total += result.proposed
        self.accepted_total += result.accepted
        return result

    # ------------------------------------------------------------------ prefill
    def prefill(self, slots: list[int], prompt_lengths: list[int] | None = None,
                chunk: int | None = None) -> StepResult:
        """Prefill the newly added slots: calls of at most ``max_prefill_rows`` rows; with ``chunk``,
        at most ``chunk`` prompt tokens per sequence per call (chunked prefill), the first token
        arriving with a sequence's last chunk. (``prompt_lengths`` is accepted for the older call
        form; the uncached counts are known from ``add_request``.)"""
        merged = StepResult()
        remaining = {s: self._uncached.get(s, 0) for s in slots}
        pending = list(slots)
        while pending:
            group, rows, take = [], 0, {}
            for s in pending:
                r = min(remaining[s], chunk) if chunk else remaining[s]
                if group and rows + r > self.max_prefill_rows:
                    break
                group.append(s)
                take[s] = r
                rows += r
            if rows > self.max_prefill_rows:
                raise ValueError(f"a prefill call of {rows} rows exceeds the workspace; use chunk=")
            # (without chunking, the group's longest take bounds every sequence's rows the same way)
            res = self._prefill_call(group, rows, chunk or max(take.values()))
            for s in group:
                remaining[s] -= take[s]
                if remaining[s] == 0:
                    merged.tokens[s] = res.tokens[s]
                    merged.finish[s] = res.finish[s]
                    self._uncached[s] = 0
            pending = [s for s in pending if remaining[s] > 0]
        return merged

    def _prefill_call(self, slots: list[int], rows: int, chunk: int) -> StepResult:
        self._set_slots(slots, len(slots))
        self._bind_sampler()
        _lib.check(self.lib.ne_prefill(self.model.handle, self.state.ref, self._slots_dev.data_ptr(), len(slots),
                                       max(rows, 1), self.k, chunk, ctypes.byref(self.outputs.struct),
                                       _lib.stream_handle()), "ne_prefill")
        if self.draft_state is not None:
            # the draft model prefills the same prompt tokens into its own cache (its own first
            # token is replaced by the target's at the next ne_draft_sync)
            self._bind_draft_region(0)
            _lib.check(self.lib.ne_prefill(self.draft_model.handle, self.draft_state.ref, self._slots_dev.data_ptr(),
                                           len(slots), max(rows, 1), self.k, chunk,
                                           ctypes.byref(self._draft_outs.struct), _lib.stream_handle()),
                       "ne_prefill (draft)")
        res = self._collect(slots)
        self.model.raise_on_device_error()
        if self.draft_model is not None:
            self.draft_model.raise_on_device_error()
        return res

    # ------------------------------------------------------------------ speculative step
    def _launch_step(self, bucket: int, buf: int = 0) -> None:
        self._bind_sampler()
        if self.draft_state is None:
            _lib.check(self.lib.ne_spec_step(self.model.handle, self.state.ref, self._slots_dev.data_ptr(), bucket,
                                             self.k, self.max_ngram, ctypes.byref(self._outs[buf].struct),
                                             _lib.stream_handle()), "ne_spec_step")
            return
        # draft model: sync with the target, k greedy draft steps (the first catches up), verify
        stream, slots = _lib.stream_handle(), self._slots_dev.data_ptr()
        _lib.check(self.lib.ne_draft_sync(self.state.ref, self.draft_state.ref, slots, bucket, self.k, stream),
                   "ne_draft_sync")
        for j in range(self.k):
            self._bind_draft_region(j)  # (sampled drafts: step j's rows stay in region j)
            _lib.check(self.lib.ne_prefill(self.draft_model.handle, self.draft_state.ref, slots, bucket,
                                           bucket * (self.k + 1), self.k, 0, ctypes.byref(self._draft_outs.struct),
                                           stream), "ne_prefill (draft step)")
        rows = None
        if self.sampling:
            rows = _lib.DraftRows(logits=self._draft_regions.data_ptr(),
                                  start=self.lib.ne_model_lm_start(self.draft_model.handle),
                                  stride=self._region_rows, rows=self.k * self._region_rows,
                                  stats=self._draft_stats.data_ptr())
        _lib.check(self.lib.ne_spec_step_drafted(self.model.handle, self.state.ref, self.draft_state.ref, slots, bucket,
                                                 self.k, ctypes.byref(self._outs[buf].struct), stream,
                                                 ctypes.byref(rows) if rows is not None else None),
                   "ne_spec_step_drafted")

    def _bind_draft_region(self, j: int) -> None:
        if self.draft_state is None or not self.sampling:
            return
        _lib.check(self.lib.ne_model_set_sampling_buffer(
            self.draft_model.handle, self._draft_regions.data_ptr() + j * self._region_bytes, self._region_bytes,
            self.max_seqs), "ne_model_set_sampling_buffer (draft)")

    def launch(self, slots: list[int], buf: int = 0) -> int:
        """Enqueue one step for ``slots`` (no host sync) writing result buffer ``buf``; returns the
        bucket used."""
        bucket = round_up_to_bucket(len(slots), self.buckets)
        self._set_slots(slots, bucket, buf)
        if not self.cuda_graphs:
            self._launch_step(bucket, buf)
            return bucket
        graph = self._graphs.get((bucket, buf))
        if graph is None:
            for b in (0, 1):  # both result buffers at once: generate() alternates them
                self._capture(bucket, b)
            graph = self._graphs[(bucket, buf)]
        graph.replay()
        return bucket

    def step(self, slots: list[int]) -> StepResult:
        self.launch(slots)
        return self._collect(slots)

    def capture_all_buckets(self) -> int:
        """Capture every batch bucket's step up front (both result buffers), largest first, so
        that no step waits for a capture while requests are served: the reference's
        DecodeGraphRunner.capture_all_buckets (engine/generation/cuda_graph_runner.py:93-104),
        which its runtime calls at start-up (engine/runtime.py:160). Returns the graphs held."""
        if self.cuda_graphs:
            for bucket in reversed(self.buckets):
                for buf in (0, 1):
                    if (bucket, buf) not in self._graphs:
                        self._capture(bucket, buf)
        return len(self._graphs)

    def _capture(self, bucket: int, buf: int = 0) -> torch.cuda.CUDAGraph:
        """Capture one bucket's step. The capture itself changes no state: every slot in the
        bucket is idle (-1) while capturing, so the captured kernels find no work."""
        saved = self._slots_dev.clone()
        self._slots_dev.fill_(-1)  # (restored below, so the slot list key stays valid)
        torch.cuda.synchronize()
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            self._launch_step(bucket, buf)  # warm-up outside capture (idle slots: no state change)
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._launch_step(bucket, buf)
        torch.cuda.synchronize()
        self._slots_dev.copy_(saved)
        self._graphs[(bucket, buf)] = graph
        return graph

    # ------------------------------------------------------------------ whole requests
    def generate(self, prompts: list[list[int]], max_new_tokens: int, ignore_eos: bool = True, *,
                 temperature: float = 0.0, top_p: float = 1.0, seeds: list[int] | None = None,
                 shared_prefix: int = 0, prefill_chunk: int | None = None) -> list[list[int]]:
        """Serve every prompt with continuous batching (up to ``max_seqs`` at a time); request i
        samples with ``seeds[i]`` (default i) when ``temperature`` > 0. ``shared_prefix`` > 0: the
        prompts' common first tokens are prefilled once and their KV blocks shared (one slot holds
        them); ``prefill_chunk``: chunked prefill.

        KV blocks: before each step the host bounds every running sequence's blocks (its length
        plus the guesses a step may reserve) and, when the next step could exhaust the pool,
        preempts the newest sequences as the reference's ContinuousBatchScheduler does
        (engine/scheduling/batch_scheduler.py:67-85): their blocks are freed and they return to the
        front of the queue with their tokens so far, to be prefilled again (recompute) and
        continued on the same random stream."""
        outputs: list[list[int]] = [[] for _ in prompts]
        pending = list(range(len(prompts)))
        running: dict[int, int] = {}  # slot -> request index
        order: dict[int, int] = {}    # slot -> admission number (the newest is preempted first)
        resume: dict[int, tuple[list[int], int, int]] = {}  # index -> (tokens, new tokens left, draws)
        prefix = self.add_prefix(prompts[0][:shared_prefix]) if shared_prefix else None
        prefix_blocks = -(-(shared_prefix + 1) // 16) if prefix is not None else 0
        k, bs = self.k, 16
        admitted_total = [0]

        def tokens_of(index: int) -> list[int]:
            return resume[index][0] if index in resume else prompts[index]

        def length(slot: int) -> int:  # prompt + tokens emitted so far (read back)
            index = running[slot]
            return len(prompts[index]) + len(outputs[index])

        def blocks_bound(extra: int) -> int:
            """Blocks the running sequences may hold after ``extra`` more tokens each (their
            rejected guesses stay reserved, so k more), shared prefix blocks counted once."""
            used = prefix_blocks
            for slot in running:
                used += max(0, -(-(length(slot) + extra + k) // bs) - self._shared_count.get(slot, 0))
            return used

        def preempt(slot: int) -> None:
            index = running.pop(slot)
            order.pop(slot, None)
            left = max_new_tokens - len(outputs[index])
            draws = int(self.state.rng_draws[slot].item())
            self.release([slot])
            resume[index] = (prompts[index] + outputs[index], left, draws)
            pending.insert(0, index)
            self.preemptions += 1

        def admit() -> None:
            batch: list[int] = []
            added = 0  # blocks the batch's sequences may hold, counted as blocks_bound(k + 1) does
            free = len(self.state.free_slots)
            while pending and len(batch) < free:
                index = pending[0]
                tokens = tokens_of(index)
                # the new prefill's blocks and one step of growth for everyone must fit the pool
                need = -(-(len(tokens) + 1 + k) // bs)
                if (running or batch) and blocks_bound(k + 1) + added + need > self.state.num_blocks:
                    break
                pending.pop(0)
                batch.append(index)
                shared = min(self._prefixes[prefix][1], (len(tokens) - 1) // 16) if prefix is not None else 0
                added += max(0, -(-(len(tokens) + (k + 1) + k) // bs) - shared)
            if not batch:
                return
            slots = self.add_requests(
                [tokens_of(i) for i in batch], [resume[i][1] if i in resume else max_new_tokens for i in batch],
                ignore_eos=ignore_eos, temperature=temperature, top_p=top_p,
                seeds=[seeds[i] if seeds is not None else i for i in batch], prefix=prefix,
                draws=[resume[i][2] if i in resume else 0 for i in batch])
            for slot, index in zip(slots, batch):
                running[slot] = index
                order[slot] = admitted_total[0]
                admitted_total[0] += 1
            res = self.prefill(slots, chunk=prefill_chunk)
            self._absorb(res, running, outputs)

        def make_room(extra: int) -> None:
            while len(running) > 1 and blocks_bound(extra) > self.state.num_blocks:
                preempt(max(running, key=lambda s: order.get(s, -1)))

        # Steps run one ahead of the host: step i + 1 is enqueued before step i's results are
        # read, so the host work of a step overlaps the next one on the GPU. A sequence that
        # finished at step i is still listed in step i + 1, where the device treats it as idle
        # (finished flag); its slot is released after step i's results arrive.
        inflight = None  # (slots, result buffer) of the step on the GPU
        buf = 0
        while pending or running or inflight:
            if inflight is None:
                admit()
                make_room(k + 1)
                if running:
                    slots = sorted(running)
                    self.launch(slots, buf)
                    self._outs[buf].start_fetch()
                    inflight = (slots, buf)
                    buf ^= 1
                continue
            if running and blocks_bound(2 * (k + 1)) > self.state.num_blocks:
                # the pool is tight: read the step in flight first (exact lengths), then decide
                res = self._collect(inflight[0], self._outs[inflight[1]])
                self._absorb(res, running, outputs)
                inflight = None
                continue
            nxt = None
            if running:
                slots = sorted(running)
                self.launch(slots, buf)
                self._outs[buf].start_fetch()
                nxt = (slots, buf)
                buf ^= 1
            res = self._collect(inflight[0], self._outs[inflight[1]])
            self._absorb(res, running, outputs)
            inflight = nxt
            if pending and self.state.free_slots and inflight is not None:
                # admission needs a prefill: read the step in flight first (its slots are current)
                res = self._collect(inflight[0], self._outs[inflight[1]])
                self._absorb(res, running, outputs)
                inflight = None
        if prefix is not None:
            self.drop_prefix(prefix)
        return outputs

    def _absorb(self, res: StepResult, running: dict[int, int], outputs: list[list[int]]) -> None:
        done = []
        for slot, toks in res.tokens.items():
            if slot not in running:  # finished at the previous step (idle in this one)
                continue
            outputs[running[slot]].extend(toks)
            if res.finish.get(slot) is not None:
                done.append(slot)
        for slot in done:
            del running[slot]
        self.release(done)
