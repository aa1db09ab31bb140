"""What int8 costs in quality on the B200 path (the reference's ``benchmarks/quality.py:58-115``
restated over this package): perplexity of one token sequence under the full-precision (bf16)
model and under the configured one (int8 weights and / or int8 KV), and how many greedy tokens of
``NUM_PROMPTS`` continuations stay the same.

    python -m inference-engine-from-scratch_b200.quality [--model qwen3-0.6b|small] [--output-dir results]

Differences from the reference's script, all forced by this build's inputs: the weights are the
seeded random init (no checkpoint download) and the text is a seeded token-id sequence (no
tokenizer); the greedy continuations come from the speculative engine, whose greedy outputs are
the plain greedy decoder's (the reference uses its cached generator). Perplexity reads the logits
of every position from one forward (``ne_forward`` with all rows' logits) and takes the
cross-entropy on the host copy, as the reference does with torch.
"""

from __future__ import annotations

import argparse
import json
import math
from dataclasses import asdict, dataclass
from pathlib import Path

import torch
from torch.nn import functional

from .config import QWEN3_0_6B, SMALL_TEST, Qwen3Config
from .engine import B200SpeculativeEngine
from .model import B200Model
from .serial import B200ModelRunner
from .weights import make_weights

NUM_PROMPTS = 8
PROMPT_TOKENS = 24
GENERATED_TOKENS = 32
QUALITY_FILE_STEM = "quality-int8"


@dataclass(frozen=True)
class QualityReport:
    perplexity_full_precision: float
    perplexity_configured: float
    greedy_token_agreement: float
    identical_completions: int
    num_completions: int
    settings: str


@dataclass
class _Tokens:
    """The fields of a sequence ``B200ModelRunner.score_tokens`` reads (and advances)."""

    token_ids: list[int]
    num_cached_tokens: int = 0


class _WholePool:
    """A block table over the first blocks of the pool, for one scoring pass."""

    block_size = 16

    def __init__(self, num_tokens: int) -> None:
        self._table = list(range(math.ceil(num_tokens / self.block_size)))

    def block_table(self, sequence) -> list[int]:
        return list(self._table)


def compute_perplexity(model: B200Model, token_ids: list[int]) -> float:
    """exp(mean cross-entropy of token i + 1 given tokens 0..i), one forward over the sequence."""
    if math.ceil(len(token_ids) / 16) * 16 > model.num_slots:
        raise ValueError("the sequence does not fit the model's KV pool")
    runner = B200ModelRunner(model, _WholePool(len(token_ids)))
    logits = runner.score_tokens(_Tokens(list(token_ids)), len(token_ids))
    loss = functional.cross_entropy(logits[:-1].float(), torch.tensor(token_ids[1:], device=logits.device))
    return math.exp(loss.item())


def generate_greedy(model: B200Model, prompts: list[list[int]], max_new: int) -> list[list[int]]:
    blocks_per = math.ceil((max(len(p) for p in prompts) + max_new + 8) / 16)
    engine = B200SpeculativeEngine(model, k=4, max_seqs=len(prompts), max_model_len=blocks_per * 16,
                                   num_blocks=len(prompts) * blocks_per, cuda_graphs=False)
    outs = engine.generate(prompts, max_new, ignore_eos=True)
    model.raise_on_device_error()
    return outs


def evaluate_quality(full_model: B200Model, configured_model: B200Model, token_ids: list[int],
                     num_prompts: int = NUM_PROMPTS, prompt_tokens: int = PROMPT_TOKENS,
                     generated: int = GENERATED_TOKENS) -> QualityReport:
    prompts = [token_ids[i * prompt_tokens:(i + 1) * prompt_tokens] for i in range(num_prompts)]
    if any(len(p) < prompt_tokens for p in prompts):
        raise ValueError(f"need {num_prompts * prompt_tokens} token ids for the prompts")
    expected = generate_greedy(full_model, prompts, generated)
    actual = generate_greedy(configured_model, prompts, generated)
    matches = sum(a == b for e, c in zip(expected, actual) for a, b in zip(e, c))
    identical = sum(e == c for e, c in zip(expected, actual))
    settings = (f"weights={'int8' if configured_model.weight_int8 else 'bf16'}, "
                f"kv_cache={'int8' if configured_model.kv_int8 else 'bf16'}")
    return QualityReport(
        perplexity_full_precision=compute_perplexity(full_model, token_ids),
        perplexity_configured=compute_perplexity(configured_model, token_ids),
        greedy_token_agreement=matches / (num_prompts * generated),
        identical_completions=identical,
        num_completions=num_prompts,
        settings=settings,
    )


def render_quality_markdown(report: QualityReport) -> str:
    return "\n".join([
        f"# int8 quality ({report.settings})",
        "",
        "| Metric | Full precision | Configured |",
        "|---|---|---|",
        f"| Perplexity on the fixed token sequence | {report.perplexity_full_precision:.3f} "
        f"| {report.perplexity_configured:.3f} |",
        f"| Greedy token agreement | 100% | {report.greedy_token_agreement:.1%} |",
        f"| Identical completions | {report.num_completions} | {report.identical_completions} |",
        "",
    ])


def build_pair(cfg: Qwen3Config, seed: int, device, weight_int8: bool, kv_int8: bool) -> tuple[B200Model, B200Model]:
    weights = make_weights(cfg, seed=seed)
    slots = 64 * 16 * 16
    full = B200Model(cfg, weights, num_slots=slots, device=device, max_positions=1024, max_rows=1024,
                     max_seqs=NUM_PROMPTS)
    configured = B200Model(cfg, weights, num_slots=slots, device=device, max_positions=1024, max_rows=1024,
                           max_seqs=NUM_PROMPTS, weight_int8=weight_int8, kv_int8=kv_int8)
    return full, configured


def main(arguments: list[str] | None = None) -> None:
    parser = argparse.ArgumentParser(prog="quality")
    parser.add_argument("--model", choices=("qwen3-0.6b", "small"), default="qwen3-0.6b")
    parser.add_argument("--weights", choices=("int8", "bf16"), default="int8")
    parser.add_argument("--kv-cache", choices=("int8", "bf16"), default="int8")
    parser.add_argument("--output-dir", type=Path, default=Path("results"))
    parsed = parser.parse_args(arguments)
    cfg = QWEN3_0_6B if parsed.model == "qwen3-0.6b" else SMALL_TEST
    full, configured = build_pair(cfg, 0, "cuda", parsed.weights == "int8", parsed.kv_cache == "int8")
    g = torch.Generator().manual_seed(0)
    token_ids = torch.randint(0, cfg.vocab_size, (NUM_PROMPTS * PROMPT_TOKENS,), generator=g).tolist()
    report = evaluate_quality(full, configured, token_ids)
    parsed.output_dir.mkdir(parents=True, exist_ok=True)
    stem = parsed.output_dir / QUALITY_FILE_STEM
    stem.with_suffix(".md").write_text(render_quality_markdown(report), encoding="utf-8")
    stem.with_suffix(".json").write_text(json.dumps(asdict(report), indent=2) + "\n")
    full.close()
    configured.close()


if __name__ == "__main__":
    main()
