"""Step-level parity of the B200 speculative path with the reference (golden fixtures) and the oracle.

* the serial drop-in (B200ModelRunner + SpeculativeGenerator + GPU NgramProposer) reproduces the
  reference's drafts, block tables, emitted tokens and (within 2e-2, bf16) logits step by step;
* the batched device-resident engine reproduces the same per-request outputs, serially (block
  tables bit-exact) and with continuous batching, with and without CUDA graphs.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import speculative as ospec
from tests import reference_seam as seam
from tests.conftest import load_golden, package, submodule

pytestmark = pytest.mark.gpu

LOGITS_ATOL_BF16 = 2e-2
LOGITS_ATOL_INT8 = 5e-2


@pytest.fixture(scope="module")
def small():
    submodule("build").build()
    pkg = package()
    cfg = pkg.SMALL_TEST
    weights = pkg.make_weights(cfg, seed=0)
    model = submodule("model").B200Model(cfg, weights, num_slots=64 * 16, device="cuda:0", max_positions=512,
                                         max_rows=512, max_seqs=8)
    return cfg, weights, model


@pytest.fixture(scope="module")
def small_int8():
    submodule("build").build()
    pkg = package()
    cfg = pkg.SMALL_TEST
    weights = pkg.make_weights(cfg, seed=0)
    model = submodule("model").B200Model(cfg, weights, num_slots=64 * 16, device="cuda:0", max_positions=512,
                                         max_rows=512, max_seqs=8, kv_int8=True, weight_int8=True)
    return cfg, weights, model


def _reset_pool(model) -> None:
    model.kv.zero_()


@pytest.mark.parametrize("variant", ["bf16", "int8"])
def test_serial_drop_in_matches_the_reference_step_by_step(small, small_int8, variant) -> None:
    """int8: int8 weights (bf16(q * scale) operands) and the int8 KV pool, logits within 5e-2."""
    cfg, _, model = small if variant == "bf16" else small_int8
    atol = LOGITS_ATOL_BF16 if variant == "bf16" else LOGITS_ATOL_INT8
    serial = submodule("serial")
    golden = load_golden(f"spec_small_{variant}.pt")
    assert golden["int8"] == (variant == "int8")
    ids = golden["digest_ids"]
    allocator = seam.PagedSlotAllocator(golden["num_blocks"], 16)
    runner = serial.B200ModelRunner(model, allocator)
    proposer = serial.NgramProposer(golden["max_ngram"], max_model_len=256, device="cuda:0")
    for index, record in enumerate(golden["records"]):
        counters = seam.StepRecords()
        gen = seam.SpeculativeGenerator(runner, proposer, golden["k"], frozenset(), metrics=counters)
        params = seam.SamplingParams(max_new_tokens=golden["max_new"], ignore_eos=True)
        events = list(gen.generate(seam.GenerationRequest(f"r{index}", record["prompt"], params)))
        assert [e.token_id for e in events] == record["tokens"]
        assert len(counters.steps) == len(record["steps"])
        for (draft, table, logits, new_tokens), ref in zip(counters.steps, record["steps"]):
            assert draft == ref["draft"]
            assert table == ref["block_table"]
            assert new_tokens == ref["new_tokens"]
            got = logits.float().cpu()
            torch.testing.assert_close(got[:, ids], ref["logits"]["at_ids"], atol=atol, rtol=0)
            top2 = torch.topk(got, 2, dim=-1).values
            torch.testing.assert_close(top2, ref["logits"]["top2"], atol=atol, rtol=0)
        assert allocator.num_free_blocks == record["free_blocks_after"]


def _engine(model, max_seqs, graphs, k=4):
    return submodule("engine").B200SpeculativeEngine(model, k=k, max_ngram=3, max_seqs=max_seqs, max_model_len=256,
                                                     num_blocks=64, cuda_graphs=graphs)


@pytest.mark.parametrize("graphs", [False, True])
def test_batched_engine_serial_block_tables_match_the_reference(small, graphs) -> None:
    _, _, model = small
    golden = load_golden("spec_small_bf16.pt")
    eng = _engine(model, 1, graphs)
    for record in golden["records"]:
        slot = eng.add_request(record["prompt"], golden["max_new"], ignore_eos=True)
        res = eng.prefill([slot], [len(record["prompt"])])
        assert eng.state.block_table(slot) == record["prefill_block_table"]
        tokens = list(res.tokens[slot])
        for ref in record["steps"]:
            res = eng.step([slot])
            assert res.proposed == len(ref["draft"])
            assert res.tokens[slot] == ref["new_tokens"]
            assert eng.state.block_table(slot) == ref["block_table"]
            tokens += res.tokens[slot]
        assert res.finish[slot] == "length"
        assert tokens == record["tokens"]
        eng.release([slot])
        assert eng.state.num_free_blocks() == record["free_blocks_after"]
    model.raise_on_device_error()


@pytest.mark.parametrize("graphs", [False, True])
def test_continuous_batching_gives_each_request_its_serial_output(small, graphs) -> None:
    _, _, model = small
    golden = load_golden("spec_small_bf16.pt")
    prompts = [r["prompt"] for r in golden["records"]]
    eng = _engine(model, 2, graphs)  # 3 requests through 2 slots: admission after a release
    outs = eng.generate(prompts, golden["max_new"])
    assert outs == [r["tokens"] for r in golden["records"]]
    assert eng.accepted_total == golden["accepted"] and eng.proposed_total == golden["proposed"]
    model.raise_on_device_error()


def test_int8_engine_serves_the_int8_reference_outputs(small_int8) -> None:
    """Config 3's arithmetic (int8 weights + int8 KV) through the batched engine with CUDA graphs."""
    _, _, model = small_int8
    golden = load_golden("spec_small_int8.pt")
    prompts = [r["prompt"] for r in golden["records"]]
    eng = _engine(model, 2, True)
    outs = eng.generate(prompts, golden["max_new"])
    assert outs == [r["tokens"] for r in golden["records"]]
    model.raise_on_device_error()


@pytest.mark.parametrize("chunk", [None, 16, 40])
def test_shared_prefix_blocks_and_chunked_prefill_serve_the_same_outputs(small, chunk) -> None:
    """Config 3's shared-prefix blocks and config 4's chunked prefill change no request's output;
    every block returns to the FIFO afterwards."""
    cfg, _, model = small
    pkg = package()
    g = torch.Generator().manual_seed(17)
    prefix = torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist()  # 2 full blocks + 8 tokens
    prompts = [prefix + t for t in pkg.make_prompts(4, cfg.vocab_size, length=30, seed=3)]
    plain = _engine(model, 2, True).generate(prompts, 24)
    eng = _engine(model, 2, True)
    free_before = eng.state.num_free_blocks()
    shared = eng.generate(prompts, 24, shared_prefix=len(prefix), prefill_chunk=chunk)
    assert shared == plain
    assert eng.state.num_free_blocks() == free_before
    model.raise_on_device_error()


def test_verify_with_full_length_drafts_matches_the_oracle(small) -> None:
    """Random-init greedy output collapses to 1-token drafts; force k-token drafts through the
    serial runner to check the k+1-row verify forward and greedy acceptance against the oracle."""
    cfg, weights, model = small
    serial = submodule("serial")
    bf16 = {k: v.to(torch.bfloat16) for k, v in weights.items()}
    oracle_runner = ospec.OracleRunner(bf16, cfg, 64, 16, torch.bfloat16)
    allocator = seam.PagedSlotAllocator(64, 16)
    runner = serial.B200ModelRunner(model, allocator)
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, cfg.vocab_size, (37,), generator=g).tolist()
    mine = seam.Sequence.from_request(seam.GenerationRequest("a", prompt, seam.SamplingParams(64)))
    ref = ospec.Seq("a", list(prompt), len(prompt), 64)
    allocator.reserve(mine, mine.num_tokens)
    oracle_runner.tables.reserve("a", ref.num_tokens)
    first = runner.run_step([mine])[0]
    ref_first, _ = oracle_runner.run_step([ref])
    assert first == ref_first[0]
    mine.token_ids.append(first)
    ref.token_ids.append(first)
    for step in range(6):
        k = [4, 8, 1, 3, 8, 2][step]
        draft = torch.randint(0, cfg.vocab_size, (k,), generator=g).tolist()
        for seq in (mine, ref):
            seq.token_ids.extend(draft)
        allocator.reserve(mine, mine.num_tokens)
        oracle_runner.tables.reserve("a", ref.num_tokens)
        logits = runner.score_tokens(mine, 1 + k).float().cpu()
        want = oracle_runner.score_tokens(ref, 1 + k).float()
        torch.testing.assert_close(logits, want, atol=LOGITS_ATOL_BF16, rtol=0)
        # accept a prefix of the target's own argmax so that some guesses survive
        target = runner.last_argmax
        keep = step % (k + 1)
        new_tokens = draft[:keep] + [target[keep]]
        for seq in (mine, ref):
            del seq.token_ids[len(seq.token_ids) - k:]
            seq.num_cached_tokens = seq.num_tokens + keep
            seq.token_ids.extend(new_tokens)
        assert mine.token_ids == ref.token_ids


def _rerun_in_a_fresh_process(env_overrides: dict, selection: str) -> None:
    import os
    import subprocess
    import sys

    from tests.conftest import REPO

    env = dict(os.environ, **env_overrides)
    proc = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", "tests/test_gpu_engine.py",
         "-k", selection], cwd=REPO, env=env, capture_output=True, text=True, timeout=900)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-2000:]


def test_fused_rmsnorm_path_serves_the_reference_outputs() -> None:
    """NE_FUSED_NORM=1 (RMSNorm folded into the QKV and gate/up GEMMs' X operand) in a fresh
    process: the serial drop-in and continuous batching still reproduce the reference fixtures."""
    _rerun_in_a_fresh_process({"NE_FUSED_NORM": "1"},
                              "serial_drop_in or continuous_batching or int8_engine")


def test_persistent_step_kernel_serves_the_reference_outputs() -> None:
    """NE_STEP_KERNEL=1 (every eligible greedy verify step as the persistent kernel): the same
    batched-engine tests, in a fresh process."""
    _rerun_in_a_fresh_process({"NE_STEP_KERNEL": "1"},
                              "batched_engine_serial or continuous_batching or shared_prefix or full_length_drafts "
                              "or preempts")


def test_profile_times_every_launch_eagerly_and_inside_a_captured_step(small) -> None:
    """ne_model_profile_*: one interval per kernel launch of the step, whether the step runs eagerly
    or was captured into a CUDA graph (event-record nodes) and replayed."""
    _, _, model = small
    lib_mod = submodule("_lib")
    pkg = package()
    eng = _engine(model, 4, graphs=False)
    prompts = pkg.make_prompts(4, model.cfg.vocab_size, length=40, seed=3)
    slots = [eng.add_request(p, 64, ignore_eos=True) for p in prompts]
    eng.prefill(slots)
    nk = len(lib_mod.KERNEL_KINDS)
    lib = model.lib
    results = []
    for captured in (False, True):
        ms_by = (ctypes.c_float * nk)()
        n_by = (ctypes.c_int * nk)()
        lib_mod.check(lib.ne_model_profile_begin(model.handle, lib_mod.stream_handle()), "profile_begin")
        lib_mod.check(lib.ne_model_profile_end(model.handle, ms_by, n_by, nk), "profile_end")  # creates events
        eng._set_slots(slots, len(slots))
        before = lib.ne_model_launch_count(model.handle)
        if captured:
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                lib_mod.check(lib.ne_model_profile_begin(model.handle, lib_mod.stream_handle()), "profile_begin")
                eng._launch_step(len(slots))
            graph.replay()
        else:
            lib_mod.check(lib.ne_model_profile_begin(model.handle, lib_mod.stream_handle()), "profile_begin")
            eng._launch_step(len(slots))
        lib_mod.check(lib.ne_model_profile_end(model.handle, ms_by, n_by, nk), "profile_end")
        launches = lib.ne_model_launch_count(model.handle) - before
        eng._collect(slots)
        model.raise_on_device_error()
        assert sum(n_by) == launches > 0
        assert all(ms_by[i] > 0 for i in range(nk) if n_by[i])
        results.append([n_by[i] for i in range(nk)])
    assert results[0] == results[1]
    eng.release(slots)


@pytest.mark.parametrize("k", [4, 8])
def test_int8_shared_prefix_reads_dequantised_block_copies(k) -> None:
    """int8 KV: the shared prefix's blocks are dequantised once (bf16(q * scale), the attention's
    own conversion) and the attention reads the copies; outputs equal the unshared run, the copies
    equal the pool blocks they stand for, and dropping the prefix unmaps them. k = 8 gives two
    query tiles per KV head (the warps of a pair share each int8 block's conversion)."""
    submodule("build").build()
    pkg = package()
    cfg = pkg.SMALL_TEST
    model = submodule("model").B200Model(cfg, pkg.make_weights(cfg, seed=0), num_slots=64 * 16, device="cuda:0",
                                         max_positions=512, max_rows=512, max_seqs=8, kv_int8=True,
                                         weight_int8=True, kv_copy_blocks=4)
    g = torch.Generator().manual_seed(17)
    prefix = torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist()  # 2 full blocks + 8 tokens
    prompts = [prefix + t for t in pkg.make_prompts(4, cfg.vocab_size, length=30, seed=3)]
    plain = _engine(model, 2, True, k=k).generate(prompts, 24)
    assert int((model.kv_copy_map >= 0).sum()) == 0
    eng = _engine(model, 2, True, k=k)
    shared = eng.generate(prompts, 24, shared_prefix=len(prefix))
    assert shared == plain
    assert int((model.kv_copy_map >= 0).sum()) == 0  # generate dropped its prefix
    holder = eng.add_prefix(prefix)
    mapped = (model.kv_copy_map >= 0).nonzero().flatten().tolist()
    assert sorted(mapped) == sorted(eng.state.block_table(holder)[:2])
    for blk in mapped:
        c = int(model.kv_copy_map[blk])
        for layer in range(cfg.num_hidden_layers):
            for kv in range(2):
                q = model.kv[layer, kv, blk * 16:(blk + 1) * 16].float()
                s = model.kv_scales[layer, kv, blk * 16:(blk + 1) * 16].float()
                want = (q * s[..., None]).to(torch.bfloat16)
                assert torch.equal(model.kv_copies[layer, kv, c * 16:(c + 1) * 16], want)
    eng.drop_prefix(holder)
    torch.cuda.synchronize()
    assert int((model.kv_copy_map >= 0).sum()) == 0
    model.raise_on_device_error()
    model.close()


def test_generate_preempts_when_the_kv_pool_runs_short(small) -> None:
    """A pool too small for every request's full length: generate() preempts the newest
    sequences (ContinuousBatchScheduler.reserve_next_tokens, batch_scheduler.py:67-85), which
    resume later by recompute; greedy outputs equal the roomy run and every block returns."""
    cfg, _, model = small
    pkg = package()
    prompts = pkg.make_prompts(4, cfg.vocab_size, length=48, seed=21)
    roomy = _engine(model, 4, False)
    expected = roomy.generate(prompts, 64)
    assert roomy.preemptions == 0
    tight = submodule("engine").B200SpeculativeEngine(model, k=4, max_ngram=3, max_seqs=4, max_model_len=256,
                                                      num_blocks=20, cuda_graphs=False)
    got = tight.generate(prompts, 64)
    assert tight.preemptions > 0
    assert got == expected
    assert tight.state.num_free_blocks() == 20
    model.raise_on_device_error()


def test_capture_all_buckets_before_serving(small) -> None:
    """Every bucket's step graph captured up front (DecodeGraphRunner.capture_all_buckets,
    cuda_graph_runner.py:93-104): both result buffers per bucket, no capture while serving, and
    the served tokens equal the eager engine's."""
    cfg, _, model = small
    pkg = package()
    prompts = pkg.make_prompts(6, cfg.vocab_size, length=40, seed=9)
    eager = _engine(model, 4, False).generate(prompts, 24)
    eng = _engine(model, 4, True)
    held = eng.capture_all_buckets()
    assert held == 2 * len(eng.buckets)
    assert eng.generate(prompts, 24) == eager
    assert len(eng._graphs) == held


def test_add_requests_validates_before_taking_slots(small) -> None:
    """add_requests refuses a batch with a prompt that does not fit, mismatched per-request lists
    or more requests than free slots, and takes no slot when it does; an accepted batch lands in
    order and prefills to the same first tokens as one request at a time."""
    cfg, _, model = small
    pkg = package()
    eng = _engine(model, 4, False)
    free = list(eng.state.free_slots)
    prompts = pkg.make_prompts(3, cfg.vocab_size, length=20, seed=4)
    with pytest.raises(ValueError):
        eng.add_requests(prompts[:2] + [list(range(1, 300))], [8, 8, 8])
    with pytest.raises(ValueError):
        eng.add_requests(prompts, [8, 8])
    with pytest.raises(RuntimeError):
        eng.add_requests(pkg.make_prompts(5, cfg.vocab_size, length=20, seed=5), [8] * 5)
    assert eng.state.free_slots == free
    slots = eng.add_requests(prompts, [8, 8, 8], ignore_eos=True)
    assert slots == free[:3]
    batched = eng.prefill(slots)
    eng.release(slots)
    one = _engine(model, 4, False)
    singles = [one.add_request(p, 8, ignore_eos=True) for p in prompts]
    single = one.prefill(singles)
    assert [batched.tokens[s] for s in slots] == [single.tokens[s] for s in singles]
    one.release(singles)
