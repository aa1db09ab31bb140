"""The CPU oracle reproduces the reference's own outputs (fixtures made by tests/golden/make_golden.py).

This is what pins the oracle: every fixture came from the unmodified reference run on the CPU.
"""

from __future__ import annotations

import json

import pytest
import torch

from oracle import ngram, philox, qwen3, speculative, verify
from tests.conftest import GOLDEN, load_golden, package

FP32_LOGITS_ATOL = 1e-4
BF16_LOGITS_ATOL = 2e-2


def test_ngram_known_answers_and_random_histories() -> None:
    cases = json.loads((GOLDEN / "ngram_cases.json").read_text())
    assert cases[0]["expected"] == [3, 4, 5] and cases[1]["expected"] == []
    for case in cases:
        got = ngram.propose(case["history"], case["k"], case["max_ngram"])
        fast = ngram.propose_numpy(case["history"], case["k"], case["max_ngram"])
        assert got == case["expected"] == fast, case


def test_philox_matches_the_published_known_answer() -> None:
    # Random123 known-answer vectors for philox4x32-10 (zero, all-ones and pi-digit inputs)
    assert philox.philox4x32_10((0, 0, 0, 0), (0, 0)) == (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)
    ones = 0xFFFFFFFF
    assert philox.philox4x32_10((ones,) * 4, (ones, ones)) == (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)
    pi = philox.philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0))
    assert pi == (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)


def test_verify_proposal_with_injected_uniforms() -> None:
    data = load_golden("verify_cases.pt")
    assert data["cases"][0]["expected"] == [2, 4, 1, 5] and data["cases"][1]["expected"] == [2, 4]
    for case in data["cases"]:
        stream = philox.UniformStream(case["seed"])
        got = verify.verify_proposal(
            case["guesses"], None, case["logits"], case["temperature"], case["top_p"], stream
        )
        assert got == case["expected"], case["seed"]
        assert stream.index == case["draws"], case["seed"]


def test_top_p_keeps_the_same_tokens() -> None:
    for case in load_golden("top_p_cases.pt")["cases"]:
        probs = verify.token_probabilities(case["logits"], case["temperature"], case["top_p"])
        assert torch.equal(probs > 0, case["kept"])
        torch.testing.assert_close(probs, case["probs"], atol=1e-6, rtol=1e-5)


def test_stable_top_p_differs_from_the_reference_only_inside_a_split_tie_group() -> None:
    """The kernels' convention (ties at the cut kept lowest id first) keeps as many tokens as the
    reference, with the same normaliser; only which members of an equal-probability group that
    straddles the cut survive may differ."""
    g = torch.Generator().manual_seed(21)
    rows = [case["logits"] for case in load_golden("top_p_cases.pt")["cases"]]
    rows += [(torch.randn(4, 4096, generator=g) * 0.7).to(torch.bfloat16) for _ in range(8)]
    for logits in rows:
        for temperature, top_p in ((0.8, 0.95), (1.0, 0.5)):
            ref = verify.token_probabilities(logits, temperature, top_p)
            ours = verify.token_probabilities(logits, temperature, top_p, stable=True)
            assert torch.equal((ref > 0).sum(-1), (ours > 0).sum(-1))
            plain = torch.softmax(logits.float() / temperature, dim=-1)
            differ = (ref > 0) != (ours > 0)
            for r in range(logits.shape[0]):
                if differ[r].any():  # every differing token shares the cut-off probability
                    tau = plain[r][ours[r] > 0].min()
                    assert torch.all(plain[r][differ[r]] == tau)
                else:
                    torch.testing.assert_close(ours[r], ref[r], atol=0, rtol=0)


def test_quantize_vectors_is_bit_exact() -> None:
    for case in load_golden("quant_cases.pt")["cases"]:
        q, s = qwen3.quantize_vectors(case["values"])
        assert torch.equal(q, case["quantized"]) and torch.equal(s, case["scales"])
        if case["values"].dtype == torch.float32:  # the reference's own bound (fp32 scales)
            back = q.float() * s.float()
            assert torch.all((back - case["values"]).abs() <= s / 2 + 1e-6)


def _check_run(golden, cfg, weights, dtype, atol, draft=None):
    int8 = golden["int8"]
    w = {k: v.to(dtype) for k, v in weights.items()}
    if int8:
        w = qwen3.quantize_weights(w)
    runner = speculative.OracleRunner(w, cfg, golden["num_blocks"], 16, dtype, int8_kv=int8)
    proposer = None
    if draft is not None:  # (config, weights) of the draft model, its own cache
        draft_cfg, draft_weights = draft
        proposer = speculative.DraftProposer(speculative.OracleRunner(
            {k: v.to(dtype) for k, v in draft_weights.items()}, draft_cfg, golden["num_blocks"], 16, dtype))
    ids = golden["digest_ids"]
    for index, record in enumerate(golden["records"]):
        seq = speculative.Seq(
            f"r{index}", list(record["prompt"]), len(record["prompt"]), golden["max_new"],
            temperature=golden["temperature"], top_p=golden["top_p"], ignore_eos=True,
        )
        seed = record["seed"]
        stream = philox.UniformStream(0 if seed is None else seed)
        out = speculative.generate(runner, seq, golden["k"], golden["max_ngram"], uniforms=stream, proposer=proposer)
        assert out.prefill_block_table == record["prefill_block_table"]
        assert len(out.steps) == len(record["steps"])
        for mine, ref in zip(out.steps, record["steps"]):
            assert mine.draft == ref["draft"]
            assert mine.block_table == ref["block_table"]
            assert mine.new_tokens == ref["new_tokens"]
            # (a sampled draft model draws one uniform per guess before verification does)
            draft_draws = len(ref["draft"]) if draft is not None and golden["temperature"] > 0 else 0
            assert mine.uniforms_used == ref["draws"] + draft_draws
            d = ref["logits"]
            assert torch.equal(torch.argmax(mine.logits, dim=-1).to(torch.int32), d["argmax"])
            torch.testing.assert_close(mine.logits.float()[:, ids], d["at_ids"], atol=atol, rtol=0)
        assert out.tokens == record["tokens"]
        assert len(runner.tables.blocks.free_blocks) == record["free_blocks_after"]


@pytest.mark.parametrize(
    "mode,dtype,atol",
    [
        ("fp32", torch.float32, FP32_LOGITS_ATOL),
        ("bf16", torch.bfloat16, BF16_LOGITS_ATOL),
        ("int8", torch.bfloat16, BF16_LOGITS_ATOL),
        ("sampled", torch.bfloat16, BF16_LOGITS_ATOL),
    ],
)
def test_serial_speculation_small_model(mode, dtype, atol) -> None:
    pkg = package()
    golden = load_golden(f"spec_small_{mode}.pt")
    _check_run(golden, pkg.SMALL_TEST, pkg.make_weights(pkg.SMALL_TEST, seed=0), dtype, atol)


def test_serial_speculation_config1_qwen3_0_6b_fp32() -> None:
    """BASELINE config 1 exactly: 63 guesses proposed, 62 kept, 128 tokens, 12 blocks."""
    pkg = package()
    golden = load_golden("spec_config1_fp32.pt")
    assert golden["proposed"] == 63 and golden["accepted"] == 62
    _check_run(golden, pkg.QWEN3_0_6B, pkg.make_weights(pkg.QWEN3_0_6B, seed=0), torch.float32,
               FP32_LOGITS_ATOL)


@pytest.mark.parametrize("fixture", ["spec_small_draft_bf16.pt", "spec_small_draft_same_bf16.pt",
                                     "spec_small_draft_sampled.pt"])
def test_serial_speculation_with_a_draft_model(fixture) -> None:
    """DraftModelProposer (proposers.py:63-106): a one-layer draft of the same family (greedy and
    sampled: drafts drawn from the draft's distribution, rejection sampling against its rows), and
    the target as its own draft (every guess kept)."""
    pkg = package()
    cfg = pkg.SMALL_TEST
    golden = load_golden(fixture)
    assert golden["proposer"] == "draft"
    if "same" in fixture:
        draft = (cfg, pkg.make_weights(cfg, seed=0))
        assert golden["accepted"] == golden["proposed"] > 0
    else:
        draft_cfg = pkg.Qwen3Config(**{**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__}, "num_hidden_layers": 1})
        draft = (draft_cfg, pkg.make_weights(draft_cfg, seed=1))
    _check_run(golden, cfg, pkg.make_weights(cfg, seed=0), torch.bfloat16, BF16_LOGITS_ATOL, draft=draft)
