"""Draft-model drafts (DraftModelProposer, engine/speculative/proposers.py:63-106) on the GPU, against
the reference's own runs (tests/golden/spec_small_draft*_bf16.pt): a one-layer draft of the same
family (seed 1), and the target as its own draft (every guess kept).

* the serial drop-in (B200ModelRunner + DraftModelProposer + SpeculativeGenerator) reproduces the
  reference's drafts, block tables and emitted tokens step by step; a draft whose top-2 logits
  are within the bf16 tolerance may pick the other token (the steps diverge from there, the
  emitted tokens may not);
* the batched device-resident engine (ne_draft_sync, k draft ne_prefill steps,
  ne_spec_step_drafted) emits the same tokens, eagerly and through CUDA graphs, serially and with
  continuous batching.
"""

from __future__ import annotations

import pytest
import torch

from tests import reference_seam as seam
from tests.conftest import load_golden, package, submodule

pytestmark = pytest.mark.gpu

DRAFT_TIE_TOL = 2e-2  # bf16 logits


def _draft_cfg(cfg, same: bool):
    pkg = package()
    if same:
        return cfg
    return pkg.Qwen3Config(**{**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__}, "num_hidden_layers": 1})


@pytest.fixture(scope="module")
def models():
    submodule("build").build()
    pkg = package()
    cfg = pkg.SMALL_TEST
    mk = submodule("model").B200Model
    target = mk(cfg, pkg.make_weights(cfg, seed=0), num_slots=64 * 16, device="cuda:0", max_positions=512,
                max_rows=512, max_seqs=8)
    dcfg = _draft_cfg(cfg, same=False)
    draft = mk(dcfg, pkg.make_weights(dcfg, seed=1), num_slots=64 * 16, device="cuda:0", max_positions=512,
               max_rows=512, max_seqs=8)
    # the target's weights as a draft of its own: a second model (its own KV pool)
    twin = mk(cfg, pkg.make_weights(cfg, seed=0), num_slots=64 * 16, device="cuda:0", max_positions=512,
              max_rows=512, max_seqs=8)
    return cfg, target, draft, twin


@pytest.mark.parametrize("same", [False, True])
def test_serial_drop_in_with_a_draft_model(models, same) -> None:
    cfg, target, draft, twin = models
    draft_model = twin if same else draft
    serial = submodule("serial")
    golden = load_golden("spec_small_draft_same_bf16.pt" if same else "spec_small_draft_bf16.pt")
    allocator = seam.PagedSlotAllocator(golden["num_blocks"], 16)
    runner = serial.B200ModelRunner(target, allocator)
    draft_runner = serial.B200ModelRunner(draft_model, seam.PagedSlotAllocator(golden["num_blocks"], 16))
    proposer = serial.DraftModelProposer(draft_runner, "cuda:0")
    excused = 0
    for index, record in enumerate(golden["records"]):
        counters = seam.StepRecords()
        gen = seam.SpeculativeGenerator(runner, proposer, golden["k"], frozenset(), metrics=counters)
        params = seam.SamplingParams(max_new_tokens=golden["max_new"], ignore_eos=True)
        events = list(gen.generate(seam.GenerationRequest(f"r{index}", record["prompt"], params)))
        # greedy speculation emits the target's own greedy tokens, whatever the drafts
        assert [e.token_id for e in events] == record["tokens"]
        for (draft_ids, table, _, new_tokens), ref in zip(counters.steps, record["steps"]):
            if draft_ids != ref["draft"]:
                top2 = ref["draft_top2"]
                assert len(top2) and float((top2[:, 0] - top2[:, 1]).min()) < DRAFT_TIE_TOL, (draft_ids, ref["draft"])
                excused += 1
                break
            assert table == ref["block_table"]
            assert new_tokens == ref["new_tokens"]
        else:
            assert len(counters.steps) == len(record["steps"])
        if same:
            assert counters.accepted == counters.proposed > 0
    assert excused <= 1
    target.raise_on_device_error()
    draft_model.raise_on_device_error()


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("same", [False, True])
def test_batched_engine_with_a_draft_model(models, graphs, same) -> None:
    cfg, target, draft, twin = models
    golden = load_golden("spec_small_draft_same_bf16.pt" if same else "spec_small_draft_bf16.pt")
    prompts = [r["prompt"] for r in golden["records"]]
    expected = [r["tokens"] for r in golden["records"]]
    for max_seqs in (1, 3):  # one request at a time, then continuous batching
        eng = submodule("engine").B200SpeculativeEngine(
            target, k=golden["k"], max_ngram=3, max_seqs=max_seqs, max_model_len=256, num_blocks=64,
            cuda_graphs=graphs, draft_model=twin if same else draft, draft_num_blocks=64)
        outs = eng.generate(prompts, golden["max_new"])
        assert outs == expected
        if same:
            assert eng.accepted_total == eng.proposed_total > 0
        else:
            assert 0 <= eng.accepted_total <= eng.proposed_total
        assert eng.state.num_free_blocks() == 64 and eng.draft_state.num_free_blocks() == 64
        target.raise_on_device_error()
        (twin if same else draft).raise_on_device_error()


def test_draft_engine_refuses_shared_prefixes_and_a_shared_kv_pool(models) -> None:
    _, target, draft, _ = models
    engine = submodule("engine")
    eng = engine.B200SpeculativeEngine(target, k=4, max_seqs=2, max_model_len=256, num_blocks=64,
                                       cuda_graphs=False, draft_model=draft)
    holder = eng.add_prefix(list(range(1, 40)))
    with pytest.raises(ValueError):
        eng.add_request(list(range(1, 50)), 4, prefix=holder)
    with pytest.raises(ValueError):  # the draft needs a KV pool of its own
        engine.B200SpeculativeEngine(target, k=4, max_seqs=2, max_model_len=256, num_blocks=64,
                                     cuda_graphs=False, draft_model=target)
