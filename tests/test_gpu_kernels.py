"""Kernel-level parity on the GPU: each kernel through the C ABI against a plain fp32 torch reference
(GEMM, RMSNorm, attention) or the CPU oracle (n-gram drafts, bit-exact)."""

from __future__ import annotations

import ctypes
import json

import pytest
import torch

from oracle import qwen3 as oq
from tests.conftest import GOLDEN, submodule

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    submodule("build").build()
    return submodule("_lib").load()


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize(
    "M,N,K",
    [(1, 128, 64), (5, 256, 1024), (16, 4096, 1024), (100, 1024, 2048), (128, 1024, 3072), (320, 6144, 1024),
     (330, 1024, 2048), (600, 384, 256), (2048, 512, 256)],
)
def test_gemm_matches_fp32_torch(lib, cuda_device, M, N, K) -> None:
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(cuda_device)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    rc = lib.ne_gemm_bf16(x.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, K, status.data_ptr(), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = (x.float() @ w.float().T)
    # fp32 accumulation in both; only the summation order differs -> within one bf16 rounding step
    torch.testing.assert_close(y.float(), ref, rtol=8e-3, atol=2e-3)


@pytest.mark.parametrize(
    "M,N,K",
    [(1, 128, 64), (7, 256, 1024), (64, 4096, 1024), (140, 1024, 2048), (140, 6144, 1024), (330, 1024, 3072),
     (600, 384, 256)],
)
def test_int8_weight_gemm_matches_the_dequantised_reference(lib, cuda_device, M, N, K) -> None:
    """Int8Linear.forward (models/int8_quantization.py:55-57): x . bf16(q * scale)^T."""
    model_mod = submodule("model")
    g = torch.Generator(device="cpu").manual_seed(M * 3 + N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    q, s = oq.quantize_vectors(w)
    dequant = q.to(torch.bfloat16) * s  # the reference's bf16 dequantisation
    y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    xd, qd, sd = x.to(cuda_device), q.to(cuda_device), s.reshape(-1).contiguous().to(cuda_device)
    rc = lib.ne_gemm_w8(xd.data_ptr(), qd.data_ptr(), sd.data_ptr(), y.data_ptr(), M, N, K, status.data_ptr(),
                        _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = x.float() @ dequant.float().T
    torch.testing.assert_close(y.float().cpu(), ref, rtol=8e-3, atol=2e-3)
    # and the same bits as the bf16 GEMM on the dequantised weights (same tiles, same order)
    y16 = torch.empty_like(y)
    dq = dequant.to(cuda_device)
    assert lib.ne_gemm_bf16(xd.data_ptr(), dq.data_ptr(), y16.data_ptr(), M, N, K, None, _stream()) == 0
    torch.cuda.synchronize()
    assert torch.equal(y, y16)
    # the model's own row quantisation equals the reference's, bit for bit
    q2, s2 = model_mod.quantize_rows(w)
    assert torch.equal(q2, q) and torch.equal(s2, s)


def test_gemm_is_deterministic(lib, cuda_device) -> None:
    x = torch.randn(320, 2048, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn(1024, 2048, device=cuda_device) * 0.02).to(torch.bfloat16)
    outs = []
    for _ in range(3):
        y = torch.empty(320, 1024, dtype=torch.bfloat16, device=cuda_device)
        assert lib.ne_gemm_bf16(x.data_ptr(), w.data_ptr(), y.data_ptr(), 320, 1024, 2048, None, _stream()) == 0
        outs.append(y)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


@pytest.mark.parametrize("rows,hidden", [(1, 1024), (37, 1024), (320, 256), (5, 4096)])
def test_rmsnorm_matches_reference_arithmetic(lib, cuda_device, rows, hidden) -> None:
    g = torch.Generator().manual_seed(rows * hidden)
    x = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    y = torch.empty(rows, hidden, dtype=torch.bfloat16, device=cuda_device)
    assert lib.ne_rmsnorm(x.to(cuda_device).data_ptr(), w.to(cuda_device).data_ptr(), y.data_ptr(), rows, hidden,
                          1e-6, _stream()) == 0
    want = oq.rms_norm(x, w, 1e-6)
    got = y.cpu()
    # the only freedom is the fp32 summation order of mean(x^2): bf16(x * r) at most one bf16 step
    # apart, which the rounded product with the weight can widen to two steps of the output
    torch.testing.assert_close(got.float(), want.float(), rtol=1.6e-2, atol=1e-3)
    assert (got == want).float().mean() > 0.99


def test_ngram_kernel_is_bit_exact_on_the_reference_cases(lib, cuda_device) -> None:
    cases = json.loads((GOLDEN / "ngram_cases.json").read_text())
    groups: dict[tuple[int, int], list[dict]] = {}
    for case in cases:
        groups.setdefault((case["k"], case["max_ngram"]), []).append(case)
    state_mod = submodule("state")
    for (k, max_ngram), group in groups.items():
        st = state_mod.DeviceBatchState(len(group), 256, k, 4, device=cuda_device)
        for slot, case in enumerate(group):
            st.load(slot, case["history"], max_new_tokens=k + 1)
        slots = torch.arange(len(group), dtype=torch.int32, device=cuda_device)
        draft_len = torch.zeros(len(group), dtype=torch.int32, device=cuda_device)
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        rc = lib.ne_ngram_propose(st.ref, slots.data_ptr(), len(group), k, max_ngram, 1, draft_len.data_ptr(),
                                  status.data_ptr(), _stream())
        assert rc == 0
        lens = draft_len.tolist()
        assert int(status.item()) == 0
        for slot, case in enumerate(group):
            L = len(case["history"])
            got = st.history[slot, L:L + lens[slot]].tolist() if lens[slot] > 0 else []
            assert got == case["expected"], case


def _attention_reference(q, k_cache, v_cache, tables, q_start, q_len, positions, nh, nkv, k_scale=None, v_scale=None):
    out = torch.zeros_like(q, dtype=torch.float32)
    G = nh // nkv
    for b in range(len(q_len)):
        for j in range(q_len[b]):
            row = q_start[b] + j
            pos = positions[row]
            slots = [tables[b][p // 16] * 16 + p % 16 for p in range(pos + 1)]
            if k_scale is None:
                keys, vals = k_cache[slots].float(), v_cache[slots].float()
            else:  # read_from_cache: int8 -> bf16 times the bf16 scale, in bf16
                keys = (k_cache[slots].to(torch.bfloat16) * k_scale[slots]).float()
                vals = (v_cache[slots].to(torch.bfloat16) * v_scale[slots]).float()
            for head in range(nh):
                kv = head // G
                s = (keys[:, kv, :] @ q[row, head].float()) / (128 ** 0.5)
                p = torch.softmax(s, dim=0)
                out[row, head] = p @ vals[:, kv, :]
    return out


ATTENTION_CASES = [
    # (nh, nkv, q_lens, contexts, scratch MB): speculative rows, prefill-like rows, split-KV
    (16, 8, [5, 1, 3], [69, 16, 200], 0),
    (16, 8, [5, 2], [333, 90], 8),
    (32, 8, [9, 2], [40, 17], 0),
    (32, 8, [5], [700], 8),
    (4, 2, [64], [64], 0),
    (16, 8, [40, 3], [40, 130], 0),
    # two query tiles per KV head (k = 8 drafts, G = 2): warp-split path, with and without split-KV
    (16, 8, [9, 3, 9], [700, 40, 300], 8),
    (16, 8, [9, 7], [1100, 160], 0),
    # enough (entry, KV head) pairs for the two-warp launch (one wave of five CTAs per SM)
    (16, 8, [9] * 60, [30 + (i * 37) % 350 for i in range(60)], 0),
    # prefill rows: eight-warp CTAs, one per query group of 128 vectors, with split-KV partials
    (16, 8, [300, 5], [600, 200], 32),
    # 19-55 entries (more than one CTA per SM, at most three): the four-warp tensor-load kernel, one and two tiles
    (16, 8, [3] * 30, [24 + (i * 53) % 300 for i in range(30)], 0),
    (16, 8, [9] * 24, [40 + (i * 71) % 400 for i in range(24)], 0),
    # contexts long enough for the planner to split the KV (32 blocks or more per split): one and two tiles
    (16, 8, [5], [2100], 8),
    (16, 8, [9, 3], [1500, 1300], 8),
]


@pytest.mark.parametrize("nh,nkv,q_lens,ctx,scratch_mb", ATTENTION_CASES)
@pytest.mark.parametrize("kv_int8", [False, True])
def test_paged_attention_matches_fp32_reference(lib, cuda_device, nh, nkv, q_lens, ctx, scratch_mb, kv_int8) -> None:
    g = torch.Generator().manual_seed(sum(ctx) + kv_int8)
    num_blocks = max(96, sum((c + 15) // 16 for c in ctx))
    shape = (num_blocks * 16 + 1, nkv, 128)
    k_cache = torch.randn(shape, generator=g).to(torch.bfloat16)
    v_cache = torch.randn(shape, generator=g).to(torch.bfloat16)
    k_scale = v_scale = None
    if kv_int8:
        k_cache, k_scale = oq.quantize_vectors(k_cache)
        v_cache, v_scale = oq.quantize_vectors(v_cache)
    perm = torch.randperm(num_blocks, generator=g).tolist()
    tables, q_start, positions = [], [], []
    row = 0
    for ql, c in zip(q_lens, ctx):
        nb = (c + 15) // 16
        tables.append(perm[:nb])
        perm = perm[nb:]
        q_start.append(row)
        positions += list(range(c - ql, c))
        row += ql
    M = row
    q = torch.randn(M, nh, 128, generator=g).to(torch.bfloat16)
    stride = max(len(t) for t in tables)
    table_t = torch.full((len(q_lens), stride), -1, dtype=torch.int32)
    for b, t in enumerate(tables):
        table_t[b, :len(t)] = torch.tensor(t)
    dev = cuda_device
    out = torch.zeros(M, nh, 128, dtype=torch.bfloat16, device=dev)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)  # noqa: E731
    t_qs, t_ql, t_pos, t_tab = i32(q_start), i32(q_lens), i32(positions), table_t.to(dev)
    rows = submodule("_lib").Rows(
        max_rows=M, num_seqs=len(q_lens), num_rows=None, token_ids=None, positions=t_pos.data_ptr(),
        slot_mapping=None, q_start=t_qs.data_ptr(), q_len=t_ql.data_ptr(), block_tables=t_tab.data_ptr(),
        table_index=None, block_table_stride=stride, max_context=stride * 16, max_q_len=max(q_lens), lm_rows=None,
        lm_count=None, lm_max=0,
    )
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    scratch = torch.empty(scratch_mb << 20, dtype=torch.uint8, device=dev) if scratch_mb else None
    dk, dv = k_cache.to(dev), v_cache.to(dev)
    dks = k_scale.squeeze(-1).contiguous().to(dev) if kv_int8 else None
    dvs = v_scale.squeeze(-1).contiguous().to(dev) if kv_int8 else None
    rc = lib.ne_paged_attention(q.to(dev).data_ptr(), out.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                dks.data_ptr() if kv_int8 else None, dvs.data_ptr() if kv_int8 else None,
                                int(kv_int8), ctypes.byref(rows), nh, nkv, 16, num_blocks * 16 + 1,
                                scratch.data_ptr() if scratch is not None else None, scratch_mb << 20,
                                status.data_ptr(), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    want = _attention_reference(q, k_cache, v_cache, tables, q_start, q_lens, positions, nh, nkv, k_scale, v_scale)
    # P is rounded to bf16 before the PV product (as flash attention does); outputs are bf16
    torch.testing.assert_close(out.cpu().float(), want, rtol=2e-2, atol=2e-2)


def test_cp_async_staging_matches_the_fp32_reference_too() -> None:
    """The speculative step's attention loads K / V with tensor loads (TMA) by default, bf16 and int8
    pools; with NE_ATTN_TMA=0 it stages them with cp.async: the same cases, that path, in a fresh
    process."""
    import os
    import subprocess
    import sys

    from tests.conftest import REPO

    env = dict(os.environ, NE_ATTN_TMA="0")
    proc = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", "tests/test_gpu_kernels.py", "-k",
         "paged_attention_matches_fp32_reference"], cwd=REPO, env=env, capture_output=True, text=True,
        timeout=900)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-2000:]
