#!/usr/bin/env python
"""Accepted tokens/s of the B200 speculative step on BASELINE config 2 (Qwen3-0.6B, bf16, n-gram k=4,
64 users, short_chat: 64-token prompts, 128 outputs).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

* ``value``: steady-state speculative steps (draft -> (k+1)-token verify -> accept -> commit for all
  64 users, one CUDA graph per step) timed with CUDA events over exactly K steps, inputs and state
  resident in HBM; emitted tokens / device time. Every step streams 1.19 GB of weights plus the KV
  cache, far more than the 126 MB L2, so no L2 flush is needed between steps.
* ``e2e``: the whole short_chat job (64 prompts from pinned host memory, prefill, every step until
  each user has 128 tokens, one device->host read of the results per step) through the public API
  ``B200SpeculativeEngine.generate``; emitted tokens / time.
* ``roofline``: the dominant kernel of one profiled step (a CUDA graph of the step with an event
  after every launch, replayed once: device time per kernel without host launch gaps), its
  algorithmic bytes per launch over its average duration, against MEASURED_PEAKS.json.
* ``cpu_baseline``: the CPU oracle (the reference's serial speculative path restated, fp32, config 1's
  prompt) on this host's cores for a bounded sample.
* ``repeats``: the steady-state measurement repeated ``--repeats`` times on fresh copies of the
  workload (per-step times, median, spread); ``value`` is the first.
* ``per_users`` (config 2 at 1, 4 and 16 users) and ``workloads`` (configs 3 and 4) on one GPU.

Other BASELINE workloads (alone, with ``--workload``): ``--workload c3`` (int8 weights + int8 KV, 64 users,
k=8, 1024-token prompts whose first 512 tokens are one shared prefix served from shared KV blocks,
256 outputs) and ``--workload c4`` (256 users, sampled T=0.8 / top-p 0.95 on per-request Philox
streams, prompt lengths uniform in [32, 2048], chunked prefill of 512 tokens, 256 outputs, k=4),
``--workload c5b`` (Qwen3-8B shape, bf16, tensor-parallel over the N torchrun ranks:
o_proj / down_proj push their fp32 partials into every rank's exchange region over NVLink for
steps of up to ``--tp-exchange-rows`` rows, NCCL all-reduce above that; 32 users, 512-token
prompts, 256 outputs, k=4).

Multi-GPU: one process per GPU (torchrun); each rank serves its own 64 users on an independent
replica (no collectives on the data path); NCCL only carries the barrier and the max-over-ranks
timing. ``--impl reference`` times the reference's CPU path (the oracle port) on rank 0.
"""

from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
PACKAGE = "inference-engine-from-scratch_b200"
METRIC = "accepted tok/s, Qwen3-0.6B spec-decode at 64 users (n-gram k=4, greedy)"
UNIT = "tok/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--no-kv-copies", action="store_true",
                   help="c3: convert the shared prefix's int8 blocks in every attention launch (no bf16 copies)")
    p.add_argument("--tp-two-phase", choices=("auto", "0", "1"), default="auto",
                   help="c5b: two-phase peer exchange (auto: from 8 ranks up)")
    p.add_argument("--tp-exchange-rows", type=int, default=512,
                   help="c5b: steps of up to this many rows use the NVLink peer exchange (0: NCCL only)")
    p.add_argument("--workload", choices=("c2", "c3", "c4", "c5b"), default="c2",
                   help="BASELINE config: c2 (default, the headline), c3 (int8, shared prefix), c4 (sampled), "
                        "c5b (Qwen3-8B shape, tensor parallel over the torchrun ranks)")
    p.add_argument("--users", type=int, default=64)
    p.add_argument("--k", type=int, default=4)
    p.add_argument("--prompt-len", type=int, default=64)
    p.add_argument("--max-new", type=int, default=128)
    p.add_argument("--cpu-seconds", type=float, default=15.0)
    p.add_argument("--repeats", type=int, default=4,
                   help="times the steady-state measurement is repeated on a fresh copy of the workload (reported "
                        "under 'repeats'; value is the first)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extra", action="store_true",
                   help="skip the 1/4/16-user lines and the config 3 / 4 block of the default run")
    p.add_argument("--profile-step", action="store_true",
                   help="prefill, then --profile-steps eager speculative steps and exit (a short target for ncu)")
    p.add_argument("--profile-steps", type=int, default=2,
                   help="with --profile-step: how many eager steps (later steps verify more rows)")
    p.add_argument("--profile-users", type=int, default=0,
                   help="with --profile-step: serve this many users instead of the workload's (small ncu captures)")
    return p.parse_args()


# ---------------------------------------------------------------------------- distributed plumbing
class _RankZero:
    rank = 0
    world = 1


class Dist:
    def __init__(self, gpus: int) -> None:
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.enabled = self.world > 1
        if self.enabled:
            import torch.distributed as dist

            torch.cuda.set_device(self.local_rank)
            dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local_rank))
            self.dist = dist

    def barrier(self) -> None:
        if self.enabled:
            self.dist.barrier()

    def max(self, value: float) -> float:
        if not self.enabled:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=f"cuda:{self.local_rank}")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, value: float) -> float:
        if not self.enabled:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=f"cuda:{self.local_rank}")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def broadcast_bytes(self, data: bytes | None) -> bytes:
        if not self.enabled:
            return data
        box = [data]
        self.dist.broadcast_object_list(box, src=0)
        return box[0]

    def close(self) -> None:
        if self.enabled:
            self.dist.destroy_process_group()


# ---------------------------------------------------------------------------- clocks (NVML, read-only)
class ClockSampler:
    """Samples SM clock and clock-event reasons every ``interval`` s while the timed region runs."""

    REASONS = {
        0x0000000000000008: "hw_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000004: "sw_power_cap",
        0x0000000000000080: "hw_power_brake_slowdown",
    }

    def __init__(self, device_index: int, interval: float = 0.005) -> None:
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML: report no clocks rather than guess
            self.nvml = None
        self.interval = interval

    def _run(self) -> None:
        get_reasons = getattr(self.nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            self.nvml.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                mhz = self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM)
                reasons = get_reasons(self.handle)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            time.sleep(self.interval)

    def __enter__(self):
        # (re-entered for every timed region: the samples of all of them add up)
        if self.nvml is not None:
            self._stop.clear()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict | None:
        if self.nvml is None:
            return None
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [m for m, _ in self.samples]
        active = 0
        for _, r in self.samples:
            active |= r
        reasons = [name for bit, name in self.REASONS.items() if active & bit]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(mhz)}


def measured_peak() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic() -> dict:
    path = REPO / "profiles" / "ncu_traffic.json"
    try:
        return json.loads(path.read_text())
    except Exception:
        return {}


# ---------------------------------------------------------------------------- CPU side (oracle)
def cpu_oracle_run(pkg, seconds: float, warmup_steps: int = 0, timed_steps: int | None = None):
    """The reference's serial speculative path restated (oracle), fp32 on this host's cores.

    Returns (emitted tokens, seconds, steps) over a bounded sample: config 1's request (prefill
    of the 64-token prompt, then speculative steps to 128 tokens) served again and again, one at a
    time as the reference serves requests, until ``timed_steps`` steps or ``seconds`` elapse.
    """
    from oracle import ngram, speculative as ospec, verify

    cfg = pkg.QWEN3_0_6B
    weights = pkg.make_weights(cfg, seed=0)
    runner = ospec.OracleRunner(weights, cfg, 64, 16, torch.float32)
    prompt = pkg.make_prompt(cfg.vocab_size, 64, 0, True)
    state = {"seq": None, "n": 0}

    def new_request() -> int:
        if state["seq"] is not None:
            runner.tables.free(state["seq"].request_id)
        state["n"] += 1
        seq = ospec.Seq(f"cpu{state['n']}", list(prompt), len(prompt), 128, ignore_eos=True)
        runner.tables.reserve(seq.request_id, seq.num_tokens)
        first, _ = runner.run_step([seq])
        seq.token_ids.append(first[0])
        state["seq"] = seq
        return 1

    def one_step() -> int:
        seq = state["seq"]
        if seq is None or seq.num_generated_tokens >= seq.max_new_tokens:
            return new_request()
        remaining = seq.max_new_tokens - seq.num_generated_tokens
        g = max(0, min(4, remaining - 1))
        draft = ngram.propose(seq.token_ids, g, 3) if g else []
        before = seq.num_tokens
        seq.token_ids.extend(draft)
        runner.tables.reserve(seq.request_id, seq.num_tokens)
        logits = runner.score_tokens(seq, 1 + len(draft))
        new = verify.verify_proposal(draft, None, logits, 0.0, 1.0, iter(()))
        del seq.token_ids[before:]
        seq.num_cached_tokens = before + len(new) - 1
        seq.token_ids.extend(new)
        return len(new)

    for _ in range(warmup_steps):
        one_step()
    emitted, steps = 0, 0
    start = time.perf_counter()
    while True:
        emitted += one_step()
        steps += 1
        elapsed = time.perf_counter() - start
        if timed_steps is not None and steps >= timed_steps:
            break
        if timed_steps is None and elapsed >= seconds:
            break
    return emitted, time.perf_counter() - start, steps


def run_reference(args, dist: Dist) -> None:
    """The reference arm: the reference's CPU speculative path (oracle port) on the host cores."""
    if dist.rank != 0:
        return
    pkg = importlib.import_module(PACKAGE)
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    emitted, seconds, steps = cpu_oracle_run(pkg, args.cpu_seconds, warmup_steps=args.warmup,
                                             timed_steps=args.steps)
    value = emitted / seconds
    sample = (f"1 user (requests are served one at a time by the reference, so its 64-user rate equals "
              f"this), config 1 prompt, {steps} speculative steps after {args.warmup} warm-up, fp32")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
        "warmup": args.warmup, "ms_per_step": 1000 * seconds / max(steps, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": "BASELINE config 1 (the reference's CPU configuration): Qwen3-0.6B random-init "
                               "(seed 0) fp32, 1 user, 64-token motif prompt, 128 greedy outputs, n-gram n=3 k=4, "
                               "16-token paged KV; the reference serves requests one at a time, so this is also "
                               "its rate at 64 users",
                   "users_per_gpu": 1, "k": 4, "parallelism": "cpu (host cores)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(args) -> dict:
    return {
        "workload": f"BASELINE config 2: Qwen3-0.6B random-init (seed 0), short_chat ({args.prompt_len}-token "
                    f"prompts, 50% motif-repeated / 50% uniform, {args.max_new} outputs), {args.users} users "
                    f"per GPU, n-gram n=3 k={args.k}, greedy, 16-token paged KV",
        "users_per_gpu": args.users,
        "k": args.k,
        "parallelism": f"dp{args.gpus} (independent replicas)",
        "l2": "no flush: every step streams 1.19 GB of weights + KV (> 126 MB L2)",
    }


class Workload:
    """One BASELINE configuration on one GPU: model arithmetic, users, prompts and decoding."""

    def __init__(self, args, pkg, vocab: int, rank: int) -> None:
        self.name = args.workload
        self.cfg = pkg.QWEN3_0_6B
        self.tp = False
        self.weight_int8 = self.kv_int8 = False
        self.temperature, self.top_p = 0.0, 1.0
        self.shared_prefix, self.prefill_chunk = 0, None
        if self.name == "c2":
            self.users, self.k, self.max_new = args.users, args.k, args.max_new
            self.prompts = pkg.make_prompts(self.users, vocab, args.prompt_len, seed=rank * self.users)
            self.metric = METRIC
            self.config = workload_config(args)
        elif self.name == "c3":
            self.users, self.k, self.max_new = 64, 8, 256
            self.weight_int8 = self.kv_int8 = True
            g = torch.Generator().manual_seed(1000 + rank)
            prefix = torch.randint(0, vocab, (512,), generator=g).tolist()
            self.prompts = [prefix + torch.randint(0, vocab, (512,), generator=g).tolist() for _ in range(self.users)]
            self.shared_prefix = 512
            self.metric = "accepted tok/s, Qwen3-0.6B int8 spec-decode at 64 users (n-gram k=8, greedy)"
            self.config = {
                "workload": "BASELINE config 3: Qwen3-0.6B random-init (seed 0), int8 per-output-channel weights "
                            "(scales from the bf16 init) + int8 KV (bf16 scales per token and head), 64 users, "
                            "1024-token prompts = one seeded 512-token prefix served from shared KV blocks + 512 "
                            "seeded uniform IDs, 256 outputs, n-gram n=3 k=8, greedy",
                "users_per_gpu": 64, "k": 8, "parallelism": f"dp{args.gpus} (independent replicas)",
                "l2": "no flush: every step streams 0.75 GB of weights + 2.4 GB of KV (> 126 MB L2)"}
        elif self.name == "c5b":
            self.cfg = pkg.QWEN3_8B_SHAPE
            self.tp = True
            self.users, self.k, self.max_new = 32, 4, 256
            self.prompts = pkg.make_prompts(self.users, vocab, 512, seed=7000)  # the same on every rank
            self.metric = "accepted tok/s, Qwen3-8B-shape spec-decode at 32 users (n-gram k=4, greedy), tensor parallel"
            self.config = {
                "workload": "BASELINE config 5b: Qwen3-8B shape (36 layers, hidden 4096, 32/8 heads, MLP 12288, "
                            "vocab 151936, untied head) random-init bf16, tensor-parallel over the GPUs (fp32 "
                            "partials of o_proj and down_proj pushed to every rank over NVLink peer memory and "
                            "summed in the next RMSNorm launch for steps of up to tp_exchange_rows rows, NCCL "
                            "all-reduce above; vocabulary-split LM head, argmax keys exchanged the same way), "
                            "32 users, 512-token prompts (50% motif-repeated), 256 outputs, n-gram n=3 k=4, greedy",
                "users": 32, "k": 4, "parallelism": f"tp{args.gpus}", "tp_exchange_rows": args.tp_exchange_rows,
                "tp_two_phase": args.tp_two_phase,
                "l2": "no flush: every step streams 15.1 GB / N of weights + KV (> 126 MB L2)"}
        else:
            self.users, self.k, self.max_new = 256, 4, 256
            self.temperature, self.top_p = 0.8, 0.95
            self.prefill_chunk = 512
            g = torch.Generator().manual_seed(2000 + rank)
            lengths = torch.randint(32, 2049, (self.users,), generator=g).tolist()
            self.prompts = [pkg.make_prompt(vocab, n, 5000 + rank * self.users + i, motif=(i % 2 == 0))
                            for i, n in enumerate(lengths)]
            self.metric = "accepted tok/s, Qwen3-0.6B spec-decode at 256 users (sampled T=0.8 top-p 0.95, k=4)"
            self.config = {
                "workload": "BASELINE config 4: Qwen3-0.6B random-init (seed 0) bf16, 256 users, sampled decoding "
                            "T=0.8 top-p 0.95 with rejection sampling on per-request Philox4x32-10 streams "
                            "(seed = request index), prompt lengths uniform in [32, 2048] (seeded; 50% "
                            "motif-repeated), chunked prefill 512, 256 outputs, n-gram n=3 k=4",
                "users_per_gpu": 256, "k": 4, "parallelism": f"dp{args.gpus} (independent replicas)",
                "l2": "no flush: every step streams 1.19 GB of weights + ~35 GB of KV (> 126 MB L2)"}
        self.sampled = self.temperature > 0.0
        if args.profile_step and args.profile_users:
            self.users = min(self.users, args.profile_users)
            self.prompts = self.prompts[: self.users]


# ---------------------------------------------------------------------------- B200 arm
def time_steady_steps(engine, engine_mod, slots: list[int], steps: int, warmup: int, dist=None, sampler=None):
    """Warm-up steps, then exactly ``steps`` replays of the bucket's CUDA graph between CUDA events
    (barrier + synchronize on both sides). Returns (ms, emitted tokens, clock summary or None)."""
    for _ in range(warmup):
        engine.step(slots)
    engine.model.raise_on_device_error()
    bucket = engine_mod.round_up_to_bucket(len(slots), engine.buckets)
    engine._set_slots(slots, bucket)
    lens_before = engine.state.seq_len.sum().item()
    graph = engine._graphs[(bucket, 0)]
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = sampler or _NoClocks()
    with sampler:
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    emitted = engine.state.seq_len.sum().item() - lens_before
    engine.model.raise_on_device_error()
    return start.elapsed_time(end), emitted, graph


class _NoClocks:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return None


def step_bytes_of(model, engine, slots: list[int], ms_per_step: float, steps: int, emitted: int,
                  shared_prefix: int = 0) -> float:
    """Algorithmic bytes of an average timed step: weights + the KV each row reads (shared prefix
    blocks once) + the KV rows written, from the contexts after the timed steps."""
    lens = engine.state.seq_len[torch.tensor(slots, device=model.device).long()]
    rows = emitted / steps  # ~ verify rows that were kept per step; the written rows are >= this
    ctx = float(lens.sum().item()) - emitted / 2.0  # mean context over the timed steps
    if shared_prefix:
        ctx -= (len(slots) - 1) * (shared_prefix // 16 * 16)
    per_token = model.kv_bytes_per_token()
    return model.weight_bytes + ctx * per_token + rows * per_token


def per_user_counts(args, pkg, engine, engine_mod, model, peak: float) -> dict:
    """BASELINE config 2 at 1, 4 and 16 users (the metric's "at 1 & 64 users"): the same engine, model
    and captured bucket graphs, a fresh set of requests per count."""
    out = {}
    for users in (1, 4, 16):
        prompts = pkg.make_prompts(users, pkg.QWEN3_0_6B.vocab_size, args.prompt_len, seed=100 + users)
        new = max(args.max_new, (args.warmup + args.steps + 3) * (args.k + 1))
        slots = engine.add_requests(prompts, [new] * users, ignore_eos=True, seeds=list(range(users)))
        engine.prefill(slots)
        ms, emitted, _ = time_steady_steps(engine, engine_mod, slots, args.steps, max(3, args.warmup))
        ms_step = ms / args.steps
        nbytes = step_bytes_of(model, engine, slots, ms_step, args.steps, emitted)
        out[str(users)] = {"value": round(emitted / (ms / 1000.0), 1), "unit": UNIT, "ms_per_step": round(ms_step, 4),
                           "step_bytes": int(nbytes), "step_frac": round(nbytes / (ms_step / 1000.0) / 1e9 / peak, 4),
                           "tokens_per_step_per_user": round(emitted / args.steps / users, 3)}
        engine.release(slots)
    return out


def other_workloads(args, pkg, model_mod, engine_mod, device, peak: float) -> dict:
    """Compact steady-state lines (no e2e) of BASELINE configs 3 and 4 on this GPU, so the default
    run carries them: a model and engine per workload, built, timed and freed in turn."""
    out = {}
    for name in ("c3", "c4"):
        try:
            sub = argparse.Namespace(**{**vars(args), "workload": name, "profile_step": False, "profile_users": 0})
            wl = Workload(sub, pkg, pkg.QWEN3_0_6B.vocab_size, 0)
            steps = max(5, args.steps // 2)
            warm = 3
            longest = max(len(p) for p in wl.prompts)
            new = max(wl.max_new, (warm + steps + 3) * (wl.k + 1))
            max_len = longest + new + 8
            blocks = (wl.users + 1) * -(-(max_len + wl.k + 1) // 16) + 16
            weights = pkg.make_weights(wl.cfg, seed=0)
            copies = wl.shared_prefix // 16 if (wl.kv_int8 and wl.shared_prefix) else 0
            model = model_mod.B200Model(wl.cfg, weights, num_slots=blocks * 16, device=device,
                                        max_positions=max_len + wl.k + 16,
                                        max_rows=max(wl.users * (wl.k + 1), 16384), max_seqs=wl.users + 1,
                                        kv_int8=wl.kv_int8, weight_int8=wl.weight_int8, kv_copy_blocks=copies)
            del weights
            engine = engine_mod.B200SpeculativeEngine(model, k=wl.k, max_ngram=3,
                                                      max_seqs=wl.users + (1 if wl.shared_prefix else 0),
                                                      max_model_len=max_len, num_blocks=blocks, cuda_graphs=True,
                                                      sampling=wl.sampled)
            prefix = engine.add_prefix(wl.prompts[0][: wl.shared_prefix]) if wl.shared_prefix else None
            slots = engine.add_requests(wl.prompts, [new] * wl.users, ignore_eos=True, temperature=wl.temperature,
                                        top_p=wl.top_p, seeds=list(range(wl.users)), prefix=prefix)
            engine.prefill(slots, chunk=wl.prefill_chunk)
            bucket = engine_mod.round_up_to_bucket(len(slots), engine.buckets)
            for buf in (0, 1):
                engine._capture(bucket, buf)
            ms, emitted, graph = time_steady_steps(engine, engine_mod, slots, steps, warm)
            ms_step = ms / steps
            nbytes = step_bytes_of(model, engine, slots, ms_step, steps, emitted, wl.shared_prefix)
            out[name] = {"metric": wl.metric, "value": round(emitted / (ms / 1000.0), 1), "unit": UNIT,
                         "ms_per_step": round(ms_step, 4), "steps": steps, "warmup": warm,
                         "step_bytes": int(nbytes),
                         "step_frac": round(nbytes / (ms_step / 1000.0) / 1e9 / peak, 4),
                         "workload": wl.config["workload"]}
            del graph
            engine._graphs.clear()
            del engine
            torch.cuda.synchronize()
            model.close()
            del model
            torch.cuda.empty_cache()
        except Exception as exc:  # the headline line must still print
            out[name] = {"error": f"{type(exc).__name__}: {exc}"}
    return out


def algorithmic_bytes(kind: str, cfg, M: int, ctx_sum: int, kv_bytes_per_token_layer: int, wb: float = 2.0,
                      slices: int = 8) -> float:
    """Unique bytes one launch of ``kind`` must move (weights at ``wb`` bytes per element plus one
    bf16 scale per row when int8, activations in/out, KV). ``slices``: fp32 partial rows an RMSNorm
    adds first (the unsplit model's split-K slices of o_proj / down_proj, or one per rank of a split
    model)."""
    H, I, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    q, kv = cfg.num_attention_heads * 128, cfg.num_key_value_heads * 128
    sc = 2 if wb == 1 else 0
    if kind == "gemm_qkv":
        return (q + 2 * kv) * (H * wb + sc) + M * H * 2 + M * q * 2 + 2 * M * kv * 2
    if kind == "gemm_o":
        return H * (q * wb + sc) + M * q * 2 + 2 * M * H * 2
    if kind == "gemm_gateup":
        return 2 * I * (H * wb + sc) + M * H * 2 + M * I * 2
    if kind == "gemm_down":
        return H * (I * wb + sc) + M * I * 2 + 2 * M * H * 2
    if kind == "lm_head":
        return V * H * 2 + M * H * 2 + M * 8
    if kind == "attention":
        return ctx_sum * kv_bytes_per_token_layer + 2 * M * q * 2
    if kind == "rmsnorm":  # partials + residual row in, residual row and normed row out, the weights
        return slices * M * H * 4 + 3 * M * H * 2 + H * 2
    if kind == "step":  # the persistent kernel: every layer's projections, attention and the LM head
        layer = sum(algorithmic_bytes(k, cfg, M, ctx_sum, kv_bytes_per_token_layer, wb)
                    for k in ("gemm_qkv", "attention", "gemm_o", "gemm_gateup", "gemm_down"))
        return cfg.num_hidden_layers * layer + algorithmic_bytes("lm_head", cfg, M, ctx_sum, kv_bytes_per_token_layer)
    return 0.0


def run_b200(args, dist: Dist) -> None:
    pkg = importlib.import_module(PACKAGE)
    model_mod = importlib.import_module(f"{PACKAGE}.model")
    engine_mod = importlib.import_module(f"{PACKAGE}.engine")
    lib_mod = importlib.import_module(f"{PACKAGE}._lib")
    importlib.import_module(f"{PACKAGE}.build").build()
    device = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(device)
    wl = Workload(args, pkg, pkg.QWEN3_0_6B.vocab_size, dist.rank)
    cfg = wl.cfg
    users, k, prompts = wl.users, wl.k, wl.prompts
    longest = max(len(p) for p in prompts)
    steady_new = max(wl.max_new, (args.warmup + args.steps + 3) * (k + 1))
    max_model_len = longest + steady_new + 8
    blocks_per_user = -(-(max_model_len + k + 1) // 16)
    num_blocks = (users + 1) * blocks_per_user + 16  # (+1: the holder of a shared prefix)
    max_rows = max(users * (k + 1), min(sum(len(p) for p in prompts), 16384))
    if wl.tp:
        tp_mod = importlib.import_module(f"{PACKAGE}.tp")
        plan = tp_mod.shard_plan(cfg, dist.rank, dist.world)
        lib_path = tp_mod.nccl_library_path()
        uid = dist.broadcast_bytes(tp_mod.unique_id(lib_path) if dist.rank == 0 else None)
        if args.tp_two_phase != "auto":
            os.environ["NE_TP_TWO_PHASE"] = args.tp_two_phase
        weights = tp_mod.make_sharded_weights(cfg, plan, seed=0, device=device)
        model = model_mod.B200Model(tp_mod.rank_config(cfg, plan), weights, num_slots=num_blocks * 16, device=device,
                                    max_positions=max_model_len + k + 16, max_rows=max_rows, max_seqs=users + 1,
                                    tp=tp_mod.TensorParallel(dist.rank, dist.world, uid, lib_path,
                                                             exchange_rows=args.tp_exchange_rows),
                                    lm_offset=plan.vocab[0])
        cfg = tp_mod.rank_config(cfg, plan)  # per-rank shapes for the byte counts below
    else:
        weights = pkg.make_weights(cfg, seed=0)
        # int8 KV with a shared prefix: the prefix blocks are dequantised once (engine.add_prefix)
        copies = wl.shared_prefix // 16 if (wl.kv_int8 and wl.shared_prefix and not args.no_kv_copies) else 0
        model = model_mod.B200Model(cfg, weights, num_slots=num_blocks * 16, device=device,
                                    max_positions=max_model_len + k + 16, max_rows=max_rows, max_seqs=users + 1,
                                    kv_int8=wl.kv_int8, weight_int8=wl.weight_int8, kv_copy_blocks=copies)
    del weights
    engine = engine_mod.B200SpeculativeEngine(model, k=k, max_ngram=3, max_seqs=users + (1 if wl.shared_prefix else 0),
                                              max_model_len=max_model_len, num_blocks=num_blocks, cuda_graphs=True,
                                              sampling=wl.sampled)
    if not args.profile_step and not wl.tp:
        # every bucket's step graph before any timing, as the reference's runtime does at start-up
        engine.capture_all_buckets()

    # ------------------------------------------------------------ steady state (value)
    prefix = engine.add_prefix(prompts[0][: wl.shared_prefix]) if wl.shared_prefix else None
    slots = engine.add_requests(prompts, [steady_new] * len(prompts), ignore_eos=True, temperature=wl.temperature,
                                top_p=wl.top_p, seeds=list(range(len(prompts))), prefix=prefix)
    engine.prefill(slots, chunk=wl.prefill_chunk)
    if args.profile_step:
        # eager steps; print what each processed so that ncu byte counts can be scaled per unit
        for i in range(args.profile_steps):
            idx = torch.tensor(slots, device=device).long()
            ctx_before = int(engine.state.seq_len[idx].sum().item())
            engine._set_slots(slots, len(slots))
            engine._launch_step(len(slots))
            res = engine._collect(slots)
            rows = len(slots) + res.proposed
            print(json.dumps({"profile_step": i, "rows": rows, "attention_ctx_sum": ctx_before + res.proposed,
                              "users": len(slots)}), flush=True)
        model.raise_on_device_error()
        model.close()
        return
    clocks = ClockSampler(dist.local_rank)
    ms, emitted, graph = time_steady_steps(engine, engine_mod, slots, args.steps, args.warmup, dist, clocks)
    stream = torch.cuda.current_stream()
    max_ms = dist.max(ms)
    total_emitted = emitted if wl.tp else dist.sum(emitted)  # a split model's ranks emit the same tokens
    value = total_emitted / (max_ms / 1000.0)

    # ------------------------------------------------------------ one profiled (eager) step: roofline
    lens = engine.state.seq_len[torch.tensor(slots, device=device).long()]
    ctx_before = int(lens.sum().item())
    launches_before = model.lib.ne_model_launch_count(model.handle)
    nk = len(lib_mod.KERNEL_KINDS)
    ms_by = (ctypes.c_float * nk)()
    n_by = (ctypes.c_int * nk)()
    engine._set_slots(slots, len(slots))
    # the step is captured with an event-record node after every launch and replayed once, so the
    # intervals are device time per kernel (serialised by the events) without host launch gaps
    lib_mod.check(model.lib.ne_model_profile_begin(model.handle, stream.cuda_stream), "profile_begin")  # events
    lib_mod.check(model.lib.ne_model_profile_end(model.handle, ms_by, n_by, nk), "profile_end")
    torch.cuda.synchronize()
    prof_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(prof_graph):
        cap = torch.cuda.current_stream().cuda_stream
        lib_mod.check(model.lib.ne_model_profile_begin(model.handle, cap), "profile_begin")
        engine._launch_step(len(slots))
    prof_graph.replay()
    lib_mod.check(model.lib.ne_model_profile_end(model.handle, ms_by, n_by, nk), "profile_end")
    res = engine._collect(slots)
    del prof_graph
    launches_per_step = model.lib.ne_model_launch_count(model.handle) - launches_before
    M = len(slots) + res.proposed
    ctx_sum = ctx_before + res.proposed  # keys visible to the last row of every sequence
    per_layer_kv = model.kv_bytes_per_token() // cfg.num_hidden_layers
    kinds = lib_mod.KERNEL_KINDS
    profile = {kinds[i]: {"ms": round(ms_by[i], 4), "launches": n_by[i]} for i in range(nk) if n_by[i]}
    step_ms_profiled = sum(ms_by[i] for i in range(nk))
    # the dominant kernel of ours (NCCL's all-reduce is timed in the profile but is not one of ours)
    dominant = max((kinds[i] for i in range(nk) if n_by[i] and kinds[i] != "collective"),
                   key=lambda kk: ms_by[kinds.index(kk)])
    di = kinds.index(dominant)
    avg_ms = ms_by[di] / n_by[di]
    wb = 1.0 if wl.weight_int8 else 2.0
    bytes_launch = algorithmic_bytes(dominant, cfg, M, ctx_sum, per_layer_kv, wb,
                                     slices=dist.world if wl.tp else 8)
    peak, peak_src = measured_peak()
    achieved = bytes_launch / (avg_ms / 1000.0) / 1e9
    # DRAM bytes per launch from the committed ncu capture of the same kernel variant (attention
    # scaled to this step's context); int8 KV / int8 weights have captures of their own
    variant = dominant
    if dominant == "attention" and model.kv_int8:
        variant = "attention_int8"
    elif dominant != "attention" and wl.weight_int8:
        variant = dominant + "_w8"
    t_rec = ncu_traffic().get(variant)
    traffic = None
    if isinstance(t_rec, dict) and "dram_bytes" in t_rec:
        traffic = float(t_rec["dram_bytes"])
        if dominant == "attention" and t_rec.get("ctx_sum"):
            traffic *= ctx_sum / float(t_rec["ctx_sum"])
        traffic = int(traffic)
    roofline = {"bound": "hbm", "kernel": dominant, "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": peak_src,
                "bytes_per_launch": int(bytes_launch), "avg_launch_ms": round(avg_ms, 5)}
    # shared prefix blocks are read once per step (unique bytes), not once per user
    unique_ctx = ctx_sum - (len(slots) - 1) * (wl.shared_prefix // 16 * 16) if wl.shared_prefix else ctx_sum
    step_bytes = model.weight_bytes + unique_ctx * model.kv_bytes_per_token() + M * model.kv_bytes_per_token()
    step_time_s = max_ms / 1000.0 / args.steps
    # the profiled step serialises its launches with an event after each one; inside the timed
    # graph the launches overlap (programmatic dependent launch), so the same kernel takes a
    # smaller share of a shorter step: its in-graph time, scaled so that all kernels sum to the
    # timed step, and the fraction of the peak that time gives
    scale = (1000.0 * step_time_s) / step_ms_profiled if step_ms_profiled > 0 else 1.0
    roofline["avg_launch_ms_in_graph"] = round(avg_ms * scale, 5)
    roofline["frac_in_graph"] = round(bytes_launch / (avg_ms * scale / 1000.0) / 1e9 / peak, 4)
    step_roofline = {"bytes_per_step": int(step_bytes), "ms_per_step": round(1000 * step_time_s, 4),
                     "achieved_gbs": round(step_bytes / step_time_s / 1e9, 1),
                     "frac": round(step_bytes / step_time_s / 1e9 / peak, 4),
                     "profiled_rows": M, "profiled_ms_sum": round(step_ms_profiled, 4)}
    engine.release(slots)
    if prefix is not None:
        engine.drop_prefix(prefix)

    # ------------------------------------------------------------ repeats of the steady-state timing
    # the same measurement again on a fresh copy of the workload (requests loaded and prefilled
    # anew, the same warm-up, exactly ``steps`` timed replays), so that the line shows how steady
    # the headline is; ``value`` stays the first timing
    repeat_ms = [max_ms / args.steps]
    for _ in range(args.repeats):
        rep_prefix = engine.add_prefix(prompts[0][: wl.shared_prefix]) if wl.shared_prefix else None
        rep_slots = engine.add_requests(prompts, [steady_new] * len(prompts), ignore_eos=True,
                                        temperature=wl.temperature, top_p=wl.top_p, seeds=list(range(len(prompts))),
                                        prefix=rep_prefix)
        engine.prefill(rep_slots, chunk=wl.prefill_chunk)
        rep, _, _ = time_steady_steps(engine, engine_mod, rep_slots, args.steps, args.warmup, dist, clocks)
        repeat_ms.append(dist.max(rep) / args.steps)
        engine.release(rep_slots)
        if rep_prefix is not None:
            engine.drop_prefix(rep_prefix)
    ordered = sorted(repeat_ms)
    repeats = {"ms_per_step": [round(x, 4) for x in repeat_ms],
               "median_ms_per_step": round(ordered[len(ordered) // 2], 4),
               "spread": round(ordered[-1] / ordered[0] - 1.0, 4)}

    # ------------------------------------------------------------ e2e: the whole job through the public API
    e2e = None
    if not args.no_e2e:
        engine.h2d_bytes = engine.d2h_bytes = 0
        dist.barrier()
        torch.cuda.synchronize()
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        steps_before = engine.steps_run
        outs = engine.generate(prompts, wl.max_new, ignore_eos=True, temperature=wl.temperature, top_p=wl.top_p,
                               shared_prefix=wl.shared_prefix, prefill_chunk=wl.prefill_chunk)
        e_end.record(stream)
        torch.cuda.synchronize()
        e_ms = dist.max(e_start.elapsed_time(e_end))
        tokens = sum(len(o) for o in outs) if wl.tp else dist.sum(sum(len(o) for o in outs))
        n_steps = max(1, engine.steps_run - steps_before)
        e2e = {"value": tokens / (e_ms / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": int(engine.h2d_bytes / n_steps),
               "d2h_bytes_per_step": int(engine.d2h_bytes / n_steps),
               "steps": n_steps, "tokens": int(tokens), "ms": round(e_ms, 3)}
        model.raise_on_device_error()

    # ------------------------------------------------------------ config 2 at 1 / 4 / 16 users (N = 1)
    per_users = None
    if wl.name == "c2" and dist.world == 1 and not args.no_extra:
        per_users = per_user_counts(args, pkg, engine, engine_mod, model, peak)

    # ------------------------------------------------------------ CPU baseline (rank 0, N = 1)
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline and wl.name == "c2":
        threads = len(os.sched_getaffinity(0))
        torch.set_num_threads(threads)
        c_emitted, c_seconds, c_steps = cpu_oracle_run(pkg, args.cpu_seconds)
        cpu = {"value": c_emitted / c_seconds, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"CPU oracle (reference serial speculative path restated), fp32, config 1's request "
                         f"served repeatedly one at a time (prefill + steps to 128 tokens), {c_steps} steps "
                         f"(prefills included) in {c_seconds:.1f} s"}

    workloads = None
    if wl.name == "c2" and dist.world == 1 and not args.no_extra:
        # free the headline's model first: config 4's KV pool alone takes ~70 GB
        del graph
        engine._graphs.clear()
        del engine
        torch.cuda.synchronize()
        model.close()
        torch.cuda.empty_cache()
        engine = graph = None
        model = None
        workloads = other_workloads(args, pkg, model_mod, engine_mod, device, peak)

    if dist.rank == 0:
        line = {
            "metric": wl.metric, "value": value, "unit": UNIT, "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": max_ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if wl.tp else "weak",
            "vs_baseline": None, "dtype": "bf16 (int8 weights / KV dequantised to bf16)" if wl.weight_int8 else "bf16",
            "data": "synthetic (seeded token-ID prompts, random-init weights)",
            "config": wl.config | {"steady_state_max_new_tokens": steady_new},
            "e2e": e2e, "roofline": roofline, "step_roofline": step_roofline, "cpu_baseline": cpu,
            "clocks": clocks.summary(), "gpu_launches": int(launches_per_step * args.steps),
            "launches_per_step": int(launches_per_step), "emitted_tokens": int(total_emitted),
            "tokens_per_step_per_user": round(total_emitted / (1 if wl.tp else dist.world) / args.steps / users, 3),
            "kernel_profile": profile, "repeats": repeats,
        }
        if per_users is not None:
            line["per_users"] = per_users
        if workloads is not None:
            line["workloads"] = workloads
        print(json.dumps(line), flush=True)
    # CUDA graphs hold the model's NCCL calls (tensor parallel): release them before the communicator
    if model is not None:
        del graph
        engine._graphs.clear()
        del engine
        torch.cuda.synchronize()
        model.close()


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        # CPU work only: no process group; under torchrun the ranks other than 0 exit at once
        if int(os.environ.get("RANK", "0")) == 0:
            run_reference(args, _RankZero())
        return
    dist = Dist(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, dist)
        else:
            run_b200(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
