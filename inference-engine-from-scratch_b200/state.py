"""Device-resident per-sequence state of the batched speculative step (``ne_batch_state``).

Replaces, for this path, the host-side ``Sequence`` fields the step touches
(engine/sequence_state.py:12-57: ``token_ids``, ``num_cached_tokens``, sampling params) and the paged
allocator's block tables (engine/memory/paged_allocator.py:21-79) with device tensors, so one
step needs no host round trip. The free-block FIFO reproduces engine/memory/block_allocator.py:8-33:
blocks are popped from the head in batch order and freed blocks appended at the tail, so a serial
(one-request-at-a-time) run hands out exactly the reference's block ids.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib


def check_sampling(temperature: float, top_p: float) -> None:
    """The request API's bounds (api/schemas.py: temperature >= 0, 0 < top_p <= 1)."""
    if not temperature >= 0.0:
        raise ValueError(f"temperature must be >= 0, got {temperature}")
    if not 0.0 < top_p <= 1.0:
        raise ValueError(f"top_p must be in (0, 1], got {top_p}")


def seed_as_int64(seed: int) -> int:
    """A 64-bit Philox key as the signed value an int64 tensor holds (same bits)."""
    seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    return seed - (1 << 64) if seed >= 1 << 63 else seed


class DeviceBatchState:
    def __init__(
        self,
        max_seqs: int,
        max_model_len: int,
        k: int,
        num_blocks: int,
        block_size: int = 16,
        stop_token_ids=(),
        device: torch.device | str = "cuda",
    ) -> None:
        self.lib = _lib.load()
        dev = torch.device(device)
        self.device = dev
        self.max_seqs = max_seqs
        self.max_model_len = max_model_len
        self.k = k
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.history_stride = max_model_len + k + 1
        self.block_table_stride = math.ceil(self.history_stride / block_size)
        i32 = dict(dtype=torch.int32, device=dev)
        self.history = torch.zeros((max_seqs, self.history_stride), **i32)
        self.seq_len = torch.zeros(max_seqs, **i32)
        self.num_cached = torch.zeros(max_seqs, **i32)
        self.num_prompt = torch.zeros(max_seqs, **i32)
        self.max_new_tokens = torch.zeros(max_seqs, **i32)
        self.flags = torch.full((max_seqs,), _lib.NE_SEQ_FINISHED, **i32)
        self.temperature = torch.zeros(max_seqs, dtype=torch.float32, device=dev)
        self.top_p = torch.ones(max_seqs, dtype=torch.float32, device=dev)
        self.rng_seed = torch.zeros(max_seqs, dtype=torch.int64, device=dev)
        self.rng_draws = torch.zeros(max_seqs, dtype=torch.int64, device=dev)
        self.block_tables = torch.full((max_seqs, self.block_table_stride), -1, **i32)
        self.num_blocks_used = torch.zeros(max_seqs, **i32)
        self.num_shared_blocks = torch.zeros(max_seqs, **i32)
        self.free_ring = torch.zeros(num_blocks, **i32)
        self.ring_head_tail = torch.zeros(2, dtype=torch.int64, device=dev)
        stops = list(stop_token_ids) or [-1]
        self.stop_ids = torch.tensor(stops, **i32)
        self.struct = _lib.BatchState(
            max_seqs=max_seqs, history_stride=self.history_stride, block_table_stride=self.block_table_stride,
            num_blocks=num_blocks, history=self.history.data_ptr(), seq_len=self.seq_len.data_ptr(),
            num_cached=self.num_cached.data_ptr(), num_prompt=self.num_prompt.data_ptr(),
            max_new_tokens=self.max_new_tokens.data_ptr(), flags=self.flags.data_ptr(),
            temperature=self.temperature.data_ptr(), top_p=self.top_p.data_ptr(),
            rng_seed=self.rng_seed.data_ptr(), rng_draws=self.rng_draws.data_ptr(),
            block_tables=self.block_tables.data_ptr(), num_blocks_used=self.num_blocks_used.data_ptr(),
            num_shared_blocks=self.num_shared_blocks.data_ptr(),
            free_ring=self.free_ring.data_ptr(), ring_head_tail=self.ring_head_tail.data_ptr(),
            stop_ids=self.stop_ids.data_ptr(), num_stop_ids=len(stop_token_ids),
        )
        self.free_slots: list[int] = list(range(max_seqs))
        self.reset_blocks()

    @property
    def ref(self):
        return ctypes.byref(self.struct)

    def reset_blocks(self) -> None:
        """BlockAllocator.__init__: the FIFO holds 0 .. num_blocks - 1."""
        _lib.check(self.lib.ne_state_reset_blocks(self.ref, _lib.stream_handle()), "ne_state_reset_blocks")

    def load(self, slot: int, prompt: list[int], max_new_tokens: int, *, ignore_eos: bool = False,
             temperature: float = 0.0, top_p: float = 1.0, seed: int = 0, draws: int = 0) -> None:
        """Copy one request into sequence slot ``slot`` (Sequence.from_request)."""
        self.load_many([slot], [prompt], [max_new_tokens], ignore_eos=[ignore_eos], temperature=[temperature],
                       top_p=[top_p], seed=[seed], draws=[draws])

    def load_many(self, slots: list[int], prompts: list[list[int]], max_new_tokens: list[int], *,
                  ignore_eos: list[bool], temperature: list[float], top_p: list[float], seed: list[int],
                  draws: list[int]) -> None:
        """Copy requests into their slots (Sequence.from_request for each): the prompts as one
        padded block and every per-sequence field as one vector, each a single host->device copy
        from pinned memory scattered by slot index."""
        n = len(slots)
        for prompt, new in zip(prompts, max_new_tokens):
            if len(prompt) == 0 or len(prompt) + new > self.max_model_len:
                raise ValueError(f"prompt of {len(prompt)} + {new} new tokens exceeds max_model_len")
        for t, p in zip(temperature, top_p):
            check_sampling(t, p)
        width = max(len(p) for p in prompts)
        block = torch.zeros((n, width), dtype=torch.int32, pin_memory=True)
        for i, prompt in enumerate(prompts):
            block[i, : len(prompt)] = torch.tensor(prompt, dtype=torch.int32)
        lens = [len(p) for p in prompts]
        ints = torch.tensor([lens, [0] * n, lens, list(max_new_tokens),
                             [_lib.NE_SEQ_IGNORE_EOS if e else 0 for e in ignore_eos]], dtype=torch.int32).pin_memory()
        floats = torch.tensor([list(temperature), list(top_p)], dtype=torch.float32).pin_memory()
        longs = torch.tensor([[seed_as_int64(v) for v in seed], [int(v) for v in draws]], dtype=torch.int64).pin_memory()
        idx = torch.tensor(slots, dtype=torch.long).pin_memory().to(self.device, non_blocking=True)
        dev_block = block.to(self.device, non_blocking=True)
        self.history[idx, :width] = dev_block
        i_dev = ints.to(self.device, non_blocking=True)
        self.seq_len[idx] = i_dev[0]
        self.num_cached[idx] = i_dev[1]
        self.num_prompt[idx] = i_dev[2]
        self.max_new_tokens[idx] = i_dev[3]
        self.flags[idx] = i_dev[4]
        f_dev = floats.to(self.device, non_blocking=True)
        self.temperature[idx] = f_dev[0]
        self.top_p[idx] = f_dev[1]
        l_dev = longs.to(self.device, non_blocking=True)
        self.rng_seed[idx] = l_dev[0]
        self.rng_draws[idx] = l_dev[1]
        # the pinned sources must outlive the asynchronous copies
        self._pinned = (block, ints, floats, longs)

    def acquire(self) -> int:
        if not self.free_slots:
            raise RuntimeError("no free sequence slot")
        return self.free_slots.pop(0)

    def release(self, slots: list[int]) -> None:
        """PagedSlotAllocator.free for each slot, in order; the slots become reusable."""
        if not slots:
            return
        ids = torch.tensor(slots, dtype=torch.int32).to(self.device)
        _lib.check(self.lib.ne_state_free_slots(self.ref, ids.data_ptr(), len(slots), _lib.stream_handle()),
                   "ne_state_free_slots")
        self.flags[ids.long()] = _lib.NE_SEQ_FINISHED
        for s in slots:
            if s not in self.free_slots:
                self.free_slots.append(s)
        self._keepalive = ids

    def share_blocks(self, src_slot: int, dst_slots: list[int], num_blocks: int) -> None:
        """The first ``num_blocks`` table entries of ``src_slot`` become shared, cached blocks of
        each slot in ``dst_slots`` (ne_state_share_blocks)."""
        if not dst_slots or num_blocks <= 0:
            return
        ids = torch.tensor(dst_slots, dtype=torch.int32).to(self.device)
        status = torch.zeros(1, dtype=torch.int32, device=self.device)
        _lib.check(self.lib.ne_state_share_blocks(self.ref, src_slot, ids.data_ptr(), len(dst_slots), num_blocks,
                                                  status.data_ptr(), _lib.stream_handle()), "ne_state_share_blocks")
        word = int(status.item())
        if word:
            raise _lib.NativeError(f"device reported: {_lib.describe_device_status(word)} (0x{word:x})")

    # ------------------------------------------------------------------ inspection (host copies)
    def block_table(self, slot: int) -> list[int]:
        n = int(self.num_blocks_used[slot].item())
        return self.block_tables[slot, :n].tolist()

    def tokens(self, slot: int) -> list[int]:
        n = int(self.seq_len[slot].item())
        return self.history[slot, :n].tolist()

    def num_free_blocks(self) -> int:
        head, tail = self.ring_head_tail.tolist()
        return int(tail - head)
