"""The serial seam: the B200 classes fit the reference's own serial API, and the test seam the GPU
tests drive them with (``tests/reference_seam.py``) behaves like the reference's classes.

Where the reference's sources are present (``NANOENGINE_REFERENCE_SRC``, or a ``reference``
checkout beside this repository), the reference's own ``SpeculativeGenerator`` and the seam's run
the same requests over the reference's own CPU ``ModelRunner`` and ``NgramProposer`` and must emit
the same events, reserve the same block tables and make the same calls. These tests need no GPU.
"""

from __future__ import annotations

import importlib
import inspect
import sys

import pytest
import torch

from tests import reference_seam as seam
from tests.conftest import REPO, load_golden, package, reference_src, submodule


@pytest.fixture(scope="module")
def ref():
    src = reference_src()
    if src is None:
        pytest.skip("the reference's sources are not present on this host")
    sys.path.insert(0, str(REPO / "tests" / "golden"))
    try:
        make_golden = importlib.import_module("make_golden")
    finally:
        sys.path.remove(str(REPO / "tests" / "golden"))
    return make_golden, make_golden.Ref(str(src))


def summary(value):
    """A comparable picture of a call argument (sequences by their state, tensors by their values)."""
    if isinstance(value, (list, tuple)):
        return [summary(v) for v in value]
    if isinstance(value, dict):
        return {k: summary(v) for k, v in value.items()}
    if hasattr(value, "token_ids") and hasattr(value, "num_cached_tokens"):
        return ("sequence", value.request_id, tuple(value.token_ids), value.num_cached_tokens)
    if hasattr(value, "token_ids"):
        return ("proposal", tuple(value.token_ids))
    if torch.is_tensor(value):
        return ("tensor", tuple(value.shape), value.float().sum().item())
    return value


class Recorder:
    """Wraps a runner / proposer / allocator and logs every call the generator makes."""

    def __init__(self, inner, log: list, name: str) -> None:
        self._inner, self._log, self._name = inner, log, name

    def __getattr__(self, attr):
        value = getattr(self._inner, attr)
        if attr == "allocator":
            return Recorder(value, self._log, f"{self._name}.allocator")
        if not callable(value):
            return value
        log, name = self._log, self._name

        def call(*args, **kwargs):
            log.append((f"{name}.{attr}", summary(args), summary(kwargs)))
            out = value(*args, **kwargs)
            log.append(("->", summary(out)))
            return out

        return call


def run_generator(generator_cls, ref_mod, model, cfg, prompts, stop_ids, *, seam_side: bool):
    cpu = torch.device("cpu")
    pool = ref_mod.pool.KVCachePool(model.config, 64 * 16, cpu, torch.float32)
    # the reference's CPU runner builds its context slots from the reference's allocator (the
    # seam's own allocator is compared with it separately)
    allocator = ref_mod.paged.PagedSlotAllocator(64, 16, cpu)
    log: list = []
    runner = ref_mod.runner.ModelRunner(model, pool, allocator, cpu)
    proposer = ref_mod.proposers.NgramProposer(3)
    kwargs = dict(verify=ref_mod.verifier.verify_proposal) if seam_side else {}
    gen = generator_cls(Recorder(runner, log, "runner"), Recorder(proposer, log, "proposer"), 4, frozenset(stop_ids),
                        cpu, None, **kwargs)
    request_cls = seam.GenerationRequest if seam_side else ref_mod.iface.GenerationRequest
    params_cls = seam.SamplingParams if seam_side else ref_mod.iface.SamplingParams
    events = []
    for index, prompt in enumerate(prompts):
        params = params_cls(max_new_tokens=24, ignore_eos=not stop_ids)
        events.append([(e.token_id, e.is_finished, e.finish_reason)
                       for e in gen.generate(request_cls(f"r{index}", list(prompt), params))])
    return events, log, allocator.num_free_blocks


@pytest.mark.parametrize("with_stop", [False, True])
def test_seam_generator_behaves_like_the_reference_generator(ref, with_stop) -> None:
    make_golden, ref_mod = ref
    pkg = package()
    cfg = pkg.Qwen3Config(**{**{f: getattr(pkg.SMALL_TEST, f) for f in pkg.SMALL_TEST.__dataclass_fields__},
                             "num_hidden_layers": 1})
    model = make_golden.build_model(ref_mod, cfg, pkg.make_weights(cfg, seed=0), torch.float32)
    prompts = [pkg.make_prompt(cfg.vocab_size, 40, 0, True), pkg.make_prompt(cfg.vocab_size, 21, 1, False)]
    stop_ids: list[int] = []
    if with_stop:
        free, _, _ = run_generator(ref_mod.specgen.SpeculativeGenerator, ref_mod, model, cfg, prompts, (),
                                   seam_side=False)
        stop_ids = [free[0][3][0]]
    want = run_generator(ref_mod.specgen.SpeculativeGenerator, ref_mod, model, cfg, prompts, stop_ids,
                         seam_side=False)
    got = run_generator(seam.SpeculativeGenerator, ref_mod, model, cfg, prompts, stop_ids, seam_side=True)
    assert got[0] == want[0]
    assert got[1] == want[1]  # the same calls, in the same order, with the same arguments
    assert got[2] == want[2]
    if with_stop:
        assert want[0][0][-1][2] == "stop"


def test_seam_allocator_reserves_like_the_reference(ref) -> None:
    _, ref_mod = ref
    cpu = torch.device("cpu")
    mine, theirs = seam.PagedSlotAllocator(8, 16), ref_mod.paged.PagedSlotAllocator(8, 16, cpu)
    seqs = {}
    for rid, n in [("a", 5), ("b", 40), ("a", 17), ("c", 16), ("b", 41), ("a", 33)]:
        for alloc, side in ((mine, "m"), (theirs, "t")):
            key = (side, rid)
            if key not in seqs:
                mod = seam if side == "m" else ref_mod.iface
                seq_cls = seam.Sequence if side == "m" else ref_mod.seq.Sequence
                seqs[key] = seq_cls.from_request(mod.GenerationRequest(rid, [1], mod.SamplingParams(4)), cpu)
            alloc.reserve(seqs[key], n)
        assert mine.block_table(seqs[("m", rid)]) == theirs.block_table(seqs[("t", rid)])
    with pytest.raises(seam.OutOfBlocks):
        mine.reserve(seqs[("m", "c")], 16 * 8)
    with pytest.raises(Exception, match="free|KV|block"):
        theirs.reserve(seqs[("t", "c")], 16 * 8)
    for rid in "abc":
        mine.free(seqs[("m", rid)])
        theirs.free(seqs[("t", rid)])
    assert mine.num_free_blocks == theirs.num_free_blocks == 8


def test_finish_reasons_follow_the_reference(ref) -> None:
    _, ref_mod = ref
    for token, generated, ignore, stops in [(5, 1, False, {5}), (5, 1, True, {5}), (6, 4, False, {5}),
                                            (6, 3, False, {5}), (5, 4, False, {5})]:
        mine = seam.find_finish_reason(token, generated, seam.SamplingParams(4, ignore_eos=ignore), frozenset(stops))
        theirs = ref_mod.sampling.find_finish_reason(token, generated,
                                                     ref_mod.iface.SamplingParams(max_new_tokens=4, ignore_eos=ignore),
                                                     frozenset(stops))
        assert mine == theirs


def test_b200_classes_take_the_calls_the_reference_generator_makes(ref) -> None:
    """Same method names and parameters as the reference's ModelRunner and proposers, so the
    reference's SpeculativeGenerator can hold them (runtime.create_engine, engine/runtime.py:162-171)."""
    _, ref_mod = ref
    serial = submodule("serial")
    pairs = [(serial.B200ModelRunner, ref_mod.runner.ModelRunner, ("run_step", "score_tokens")),
             (serial.NgramProposer, ref_mod.proposers.NgramProposer, ("propose", "release")),
             (serial.DraftModelProposer, ref_mod.proposers.DraftModelProposer, ("propose", "release"))]
    for mine, theirs, methods in pairs:
        for name in methods:
            a = list(inspect.signature(getattr(mine, name)).parameters)
            b = list(inspect.signature(getattr(theirs, name)).parameters)
            assert a == b, (mine.__name__, name, a, b)
    assert isinstance(inspect.getattr_static(serial.B200ModelRunner, "vocab_size"), property)
    # verify_proposal takes the reference's four arguments (the fifth, the kernel's argmax ids, is optional)
    params = list(inspect.signature(serial.verify_proposal).parameters)
    assert params[:4] == list(inspect.signature(ref_mod.verifier.verify_proposal).parameters)


def test_torch_generators_map_to_philox_streams_by_seed() -> None:
    serial = submodule("serial")
    a, b = torch.Generator().manual_seed(42), torch.Generator().manual_seed(42)
    sa, sb = serial.philox_stream(a), serial.philox_stream(b)
    assert sa is not sb and sa.seed == sb.seed == 42 and sa.draws == 0
    assert serial.philox_stream(a) is sa  # one stream per generator object, kept while it lives
    mine = serial.create_sampling_generator(7)
    assert serial.philox_stream(mine) is mine
    serial.release_stream(a)
    serial.release_stream(b)
    with pytest.raises(ValueError):
        serial.philox_stream(None)


def test_stop_fixture_cuts_inside_an_accepted_run() -> None:
    """The draft fixture's stopping step is cut: the reference dropped guesses it had kept after
    the stop token, so a device path that only checked a step's last token would fail the GPU tests."""
    golden = load_golden("spec_small_stop_draft.pt")
    record = golden["records"][golden["stop_record"]]
    stop = golden["stop_ids"][0]
    last = record["steps"][-1]["new_tokens"]
    j = last.index(stop)
    assert j < len(last) - 1
    before = 1 + sum(len(s["new_tokens"]) for s in record["steps"][:-1])
    assert len(record["tokens"]) == before + j + 1
    assert record["tokens"][-1] == stop and record["finish_reason"] == "stop"
