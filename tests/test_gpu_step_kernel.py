"""The persistent verify-step kernel (``NE_STEP_KERNEL=1``, csrc/step_kernel.cu) against the
per-projection launches it replaces, on the same KV state: greedy argmax ids of verify rows at the
benchmarked Qwen3-0.6B shape (1, 2 and 5 rows) and with fewer layers, and whole batched generations
of the small model (eager and CUDA graphs) token for token against the reference's fixtures."""

from __future__ import annotations

import os

import pytest
import torch

from tests import reference_seam as seam
from tests.conftest import load_golden, package, submodule

pytestmark = pytest.mark.gpu


@pytest.fixture()
def step_kernel_on():
    before = os.environ.get("NE_STEP_KERNEL")
    os.environ["NE_STEP_KERNEL"] = "1"
    yield
    if before is None:
        os.environ.pop("NE_STEP_KERNEL", None)
    else:
        os.environ["NE_STEP_KERNEL"] = before


@pytest.fixture(scope="module")
def full_weights():
    pkg = package()
    return pkg.make_weights(pkg.QWEN3_0_6B, seed=0)


@pytest.mark.parametrize("layers", [1, 28])
def test_verify_rows_take_the_per_projection_argmax(full_weights, layers) -> None:
    submodule("build").build()
    pkg = package()
    serial = submodule("serial")
    cfg = pkg.Qwen3Config(**{**{f: getattr(pkg.QWEN3_0_6B, f) for f in pkg.QWEN3_0_6B.__dataclass_fields__},
                             "num_hidden_layers": layers})
    weights = {k: v for k, v in full_weights.items()
               if not k.startswith("model.layers.") or int(k.split(".")[2]) < layers}
    model = submodule("model").B200Model(cfg, weights, num_slots=64 * 16, device="cuda:0", max_positions=512,
                                         max_rows=512, max_seqs=8)
    try:
        allocator = seam.PagedSlotAllocator(64, 16)
        runner = serial.B200ModelRunner(model, allocator)
        prompt = pkg.make_prompt(cfg.vocab_size, 64, 0, True)
        seq = seam.Sequence.from_request(seam.GenerationRequest("p", prompt, seam.SamplingParams(64)))
        allocator.reserve(seq, seq.num_tokens + 8)
        first = runner.run_step([seq])[0]
        g = torch.Generator().manual_seed(1)
        for count in (1, 2, 5):
            seq.token_ids = prompt + [first] + torch.randint(0, cfg.vocab_size, (count - 1,), generator=g).tolist()
            seq.num_cached_tokens = len(prompt)
            logits = torch.empty((count, cfg.vocab_size), dtype=torch.bfloat16, device="cuda:0")
            runner._forward(seq, count, list(range(count)), logits)  # per-projection path, all logits
            os.environ["NE_STEP_KERNEL"] = "1"
            try:
                ids = runner._forward(seq, count, list(range(count)), None)
            finally:
                os.environ.pop("NE_STEP_KERNEL", None)
            chosen = logits.float().gather(1, torch.tensor(ids, device="cuda:0")[:, None])[:, 0]
            top = logits.float().max(dim=-1).values
            # a row maximum of the per-projection logits, up to the summation-order differences of two
            # bf16 forwards (split-K partition, RMSNorm statistics): within 2e-2 of the top logit
            assert ((top - chosen) <= 2e-2).all(), (count, ids, (top - chosen).tolist())
        model.raise_on_device_error()
    finally:
        model.close()


@pytest.mark.parametrize("graphs", [False, True])
def test_batched_generation_serves_the_reference_outputs(step_kernel_on, graphs) -> None:
    submodule("build").build()
    pkg = package()
    cfg = pkg.SMALL_TEST
    model = submodule("model").B200Model(cfg, pkg.make_weights(cfg, seed=0), num_slots=64 * 16, device="cuda:0",
                                         max_positions=512, max_rows=512, max_seqs=8)
    try:
        golden = load_golden("spec_small_bf16.pt")
        eng = submodule("engine").B200SpeculativeEngine(model, k=4, max_ngram=3, max_seqs=3, max_model_len=256,
                                                        num_blocks=64, cuda_graphs=graphs)
        before = model.lib.ne_model_launch_count(model.handle)
        outs = eng.generate([r["prompt"] for r in golden["records"]], golden["max_new"])
        assert outs == [r["tokens"] for r in golden["records"]]
        model.raise_on_device_error()
        assert model.lib.ne_model_launch_count(model.handle) > before
    finally:
        model.close()
