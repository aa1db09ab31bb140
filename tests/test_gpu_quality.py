"""int8 quality reporting on the B200 path (benchmarks/quality.py:58-115 restated in
``quality.py``): perplexity under the full-precision and the configured model, greedy agreement."""

from __future__ import annotations

import math

import pytest
import torch

from tests.conftest import package, submodule

pytestmark = pytest.mark.gpu


def test_int8_kv_keeps_greedy_agreement_and_the_report_is_consistent() -> None:
    """The reference's bar for an int8 KV cache (tests/engine/test_quantization_and_cuda_graphs.py:
    104-120): at least 90% of greedy tokens agree with full precision; perplexities are finite."""
    submodule("build").build()
    quality = submodule("quality")
    cfg = package().SMALL_TEST
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (quality.NUM_PROMPTS * quality.PROMPT_TOKENS,), generator=g).tolist()
    for weight_int8 in (False, True):
        full, configured = quality.build_pair(cfg, 0, "cuda:0", weight_int8=weight_int8, kv_int8=True)
        report = quality.evaluate_quality(full, configured, ids)
        assert report.num_completions == quality.NUM_PROMPTS
        assert 0 <= report.identical_completions <= report.num_completions
        assert all(math.isfinite(p) and p > 1.0 for p in (report.perplexity_full_precision,
                                                          report.perplexity_configured))
        if not weight_int8:
            assert report.greedy_token_agreement >= 0.9
        # the full-precision model against itself: identical
        same = quality.evaluate_quality(full, full, ids, num_prompts=2)
        assert same.greedy_token_agreement == 1.0 and same.identical_completions == 2
        assert same.perplexity_full_precision == same.perplexity_configured
        full.close()
        configured.close()
