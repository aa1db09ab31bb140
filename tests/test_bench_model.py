"""The byte model behind ``bench.py``'s roofline (CPU).

``roofline.achieved`` is the dominant kernel's algorithmic bytes per launch over its duration, and
``roofline.traffic`` comes from the committed ncu captures (``profiles/ncu_traffic.json``). These
tests pin the per-launch bytes of the Qwen3-0.6B verify step to the sizes of the tensors a launch
must move, and check that every committed capture read at least those bytes and at most a quarter
more, at the rows and context it was taken at (a capture that re-read weights or KV, or that
belongs to another shape, fails here).
"""

from __future__ import annotations

import importlib
import json
import sys

import pytest

from tests.conftest import REPO, package

sys.path.insert(0, str(REPO))
bench = importlib.import_module("bench")

KV_BF16 = 8 * 128 * 2 * 2  # bytes of K and V per token and layer: 8 KV heads x 128 dims, bf16


@pytest.fixture(scope="module")
def cfg():
    return package().QWEN3_0_6B


def test_projection_bytes_are_the_weights_plus_the_rows(cfg) -> None:
    H, I, q, kv = 1024, 3072, 16 * 128, 8 * 128
    ab = bench.algorithmic_bytes
    assert ab("gemm_qkv", cfg, 0, 0, KV_BF16) == (q + 2 * kv) * H * 2 == 8_388_608
    assert ab("gemm_o", cfg, 0, 0, KV_BF16) == H * q * 2 == 4_194_304
    assert ab("gemm_gateup", cfg, 0, 0, KV_BF16) == 2 * I * H * 2 == 12_582_912
    assert ab("gemm_down", cfg, 0, 0, KV_BF16) == H * I * 2 == 6_291_456
    assert ab("lm_head", cfg, 0, 0, KV_BF16) == 151_936 * H * 2 == 311_164_928
    # each row adds its activations in and out (QKV: x in; q, k, v out)
    M = 135
    assert ab("gemm_qkv", cfg, M, 0, KV_BF16) - ab("gemm_qkv", cfg, 0, 0, KV_BF16) == M * (H + q + 2 * kv) * 2
    # int8 weights: one byte per element and one bf16 scale per output row
    assert ab("gemm_qkv", cfg, 0, 0, KV_BF16, wb=1) == (q + 2 * kv) * (H + 2)


def test_step_weights_match_the_model(cfg) -> None:
    """28 layers of projections plus the LM head: the 1,192,099,840 weight bytes of a 0.6B step less
    the 131,072 bytes of RMSNorm weights (input, post-attention and q / k norms, the final norm)."""
    norms = 28 * (2 * 1024 + 2 * 128) * 2 + 1024 * 2
    assert norms == 131_072
    assert bench.algorithmic_bytes("step", cfg, 0, 0, KV_BF16) == 1_192_099_840 - norms


def test_attention_and_rmsnorm_bytes(cfg) -> None:
    ab = bench.algorithmic_bytes
    assert ab("attention", cfg, 0, 4_981, KV_BF16) == 4_981 * KV_BF16 == 20_402_176
    # q in and the output row out per verify row
    assert ab("attention", cfg, 10, 0, KV_BF16) == 10 * 2 * 16 * 128 * 2
    # eight fp32 partial slices and the residual row in, residual and normed rows out, the weights
    assert ab("rmsnorm", cfg, 135, 0, KV_BF16) == 8 * 135 * 1024 * 4 + 3 * 135 * 1024 * 2 + 1024 * 2


def test_committed_traffic_is_the_algorithmic_bytes_read_once(cfg) -> None:
    """DRAM reads of each captured launch lie between what must come from DRAM (the weights, or the
    KV the launch attends over: zero rows) and a quarter above the launch's algorithmic bytes at its
    rows (the activation rows in and out mostly stay in L2)."""
    traffic = json.loads((REPO / "profiles" / "ncu_traffic.json").read_text())
    assert traffic == bench.ncu_traffic()
    checked = 0
    for kind in ("gemm_qkv", "gemm_o", "gemm_gateup", "gemm_down", "lm_head", "attention"):
        rec = traffic[kind]
        ctx = rec.get("ctx_sum", 0)
        must = bench.algorithmic_bytes(kind, cfg, 0, ctx, KV_BF16)
        algorithmic = bench.algorithmic_bytes(kind, cfg, rec["rows"], ctx, KV_BF16)
        assert must <= rec["dram_bytes"] <= 1.25 * algorithmic, (kind, rec, must, algorithmic)
        checked += 1
    assert checked == 6
