"""The attention entry point that allocates nothing, against the scratch-taking entry point.

``ne_paged_attention_static_scratch`` serves callers that may not allocate device memory (their
host framework owns the device's memory through its own allocator, or they must not call
cudaMalloc once running): its split-KV partials live in a fixed 4 MiB array inside the library.
Its results must match ``ne_paged_attention`` (caller-provided scratch) within the tolerance of the
attention tests, on two calls in a row, and a request for more splits than the array holds must be
refused without launching anything. This file sorts last so that a run stopping at the first
failure has already run every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from tests.conftest import submodule

pytestmark = pytest.mark.gpu

NE_ERR_WORKSPACE = 5


def _case(seed: int, q_lens, ctx, nh=16, nkv=8, num_blocks=96, device="cuda:0"):
    g = torch.Generator().manual_seed(seed)
    shape = (num_blocks * 16 + 1, nkv, 128)
    k_cache = torch.randn(shape, generator=g).to(torch.bfloat16).to(device)
    v_cache = torch.randn(shape, generator=g).to(torch.bfloat16).to(device)
    perm = torch.randperm(num_blocks, generator=g).tolist()
    tables, q_start, positions, row = [], [], [], 0
    for ql, c in zip(q_lens, ctx):
        nb = (c + 15) // 16
        tables.append(perm[:nb])
        perm = perm[nb:]
        q_start.append(row)
        positions += list(range(c - ql, c))
        row += ql
    stride = max(len(t) for t in tables)
    table = torch.full((len(q_lens), stride), -1, dtype=torch.int32)
    for b, t in enumerate(tables):
        table[b, : len(t)] = torch.tensor(t)
    keep = {
        "q": torch.randn(row, nh, 128, generator=g).to(torch.bfloat16).to(device),
        "k": k_cache, "v": v_cache,
        "qs": torch.tensor(q_start, dtype=torch.int32, device=device),
        "ql": torch.tensor(q_lens, dtype=torch.int32, device=device),
        "pos": torch.tensor(positions, dtype=torch.int32, device=device),
        "tab": table.to(device),
    }
    rows = submodule("_lib").Rows(
        max_rows=row, num_seqs=len(q_lens), num_rows=None, token_ids=None, positions=keep["pos"].data_ptr(),
        slot_mapping=None, q_start=keep["qs"].data_ptr(), q_len=keep["ql"].data_ptr(),
        block_tables=keep["tab"].data_ptr(), table_index=None, block_table_stride=stride, max_context=stride * 16,
        max_q_len=max(q_lens), lm_rows=None, lm_count=None, lm_max=0,
    )
    return keep, rows, row, nh, nkv, num_blocks * 16 + 1


def test_static_scratch_attention_matches_the_scratch_entry_on_two_calls() -> None:
    if not torch.cuda.is_available():
        pytest.fail("needs a CUDA device")
    submodule("build").build()
    lib = submodule("_lib").load()
    stream = torch.cuda.current_stream().cuda_stream
    scratch = torch.empty(16 << 20, dtype=torch.uint8, device="cuda:0")
    status = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    # two calls in a row with different shapes and split counts: the second must not see the first's partials
    for seed, q_lens, ctx, splits in ((1, [5, 1, 3], [333, 40, 170], 8), (2, [5], [900], 24)):
        keep, rows, M, nh, nkv, slots = _case(seed, q_lens, ctx)
        want = torch.zeros(M, nh, 128, dtype=torch.bfloat16, device="cuda:0")
        got = torch.full((M, nh, 128), float("nan"), dtype=torch.bfloat16, device="cuda:0")
        rc = lib.ne_paged_attention(keep["q"].data_ptr(), want.data_ptr(), keep["k"].data_ptr(), keep["v"].data_ptr(),
                                    None, None, 0, ctypes.byref(rows), nh, nkv, 16, slots, scratch.data_ptr(),
                                    scratch.numel(), status.data_ptr(), stream)
        assert rc == 0
        rc = lib.ne_paged_attention_static_scratch(keep["q"].data_ptr(), got.data_ptr(), keep["k"].data_ptr(),
                                                   keep["v"].data_ptr(), None, None, 0, ctypes.byref(rows), nh, nkv,
                                                   16, slots, splits, status.data_ptr(), stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=2e-2)


def test_static_scratch_attention_refuses_more_splits_than_the_array_holds() -> None:
    if not torch.cuda.is_available():
        pytest.fail("needs a CUDA device")
    lib = submodule("_lib").load()
    keep, rows, M, nh, nkv, slots = _case(3, [5] * 64, [120] * 64, num_blocks=600)
    out = torch.zeros(M, nh, 128, dtype=torch.bfloat16, device="cuda:0")
    # 64 sequences x 8 heads x 32 splits x 10 vectors x 520 B = 85 MB > 4 MiB
    rc = lib.ne_paged_attention_static_scratch(keep["q"].data_ptr(), out.data_ptr(), keep["k"].data_ptr(),
                                               keep["v"].data_ptr(), None, None, 0, ctypes.byref(rows), nh, nkv, 16,
                                               slots, 32, None, torch.cuda.current_stream().cuda_stream)
    assert rc == NE_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0  # nothing was launched
