"""Tensor parallelism on 2 GPUs: a split model serves exactly what the unsplit model serves, over
the peer exchange and over NCCL, and a rank left alone reports a timeout instead of hanging.

Skipped on a host with fewer than two GPUs. The ranks run as child processes under torchrun
(tests/tp_worker.py) with NVLS off, bounded by a timeout.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest
import torch

from tests.conftest import REPO

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_split_serves_the_unsplit_outputs(tmp_path) -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    out = tmp_path / "rank"
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(REPO / "tests" / "tp_worker.py"), "--out", str(out)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    proc = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    r0 = json.loads((tmp_path / "rank.0.json").read_text())
    r1 = json.loads((tmp_path / "rank.1.json").read_text())
    assert r0["peer_exchange"] and r1["peer_exchange"]
    # both ranks take the same decisions (max-reduced argmax keys), eagerly and through graphs,
    # over the peer exchange (one and two phases), the exchange for steps only, and NCCL only
    for name in ("eager", "graphs", "mixed", "nccl", "two_phase"):
        assert r0[name] == r1[name] == r0["graphs"], name
    # and they equal the unsplit model's tokens (fp32 partial sums: only the summation order differs)
    assert r0["graphs"] == r0["unsplit"]
    assert all(len(o) == 32 for o in r0["unsplit"])
    # a rank whose peer launches nothing: its exchange waits end (bounded) with the timeout status
    assert "bounded device wait ran out" in r0["lone_rank"], r0["lone_rank"]
