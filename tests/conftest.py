"""Shared fixtures. GPU tests are marked ``gpu``; everything else runs on a CPU-only host."""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

PACKAGE = "inference-engine-from-scratch_b200"
# pytest loads this file as ``conftest``; the test modules import it as ``tests.conftest``: one
# module object for both names, so that state the hooks below read is the state the tests write
sys.modules.setdefault("tests.conftest", sys.modules[__name__])


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


# near-tie excuses of the sampled and full-model parity tests: (test, cases, exact, excused margins)
NEAR_TIES: list[tuple[str, int, int, list[float]]] = []


def report_near_ties(test: str, cases: int, exact: int, margins: list[float]) -> None:
    """Record how many of a test's cases matched bit for bit and the margins of the excused ones."""
    NEAR_TIES.append((test, cases, exact, sorted(margins)))


def pytest_terminal_summary(terminalreporter) -> None:
    if not NEAR_TIES:
        return
    terminalreporter.section("near-tie excuses (cases matched exactly / excused, largest excused margin)")
    for test, cases, exact, margins in NEAR_TIES:
        worst = f"{max(margins):.3g}" if margins else "-"
        terminalreporter.write_line(f"{test}: {exact}/{cases} exact, {len(margins)} excused, largest margin {worst}")


def package():
    return importlib.import_module(PACKAGE)


def submodule(name: str):
    return importlib.import_module(f"{PACKAGE}.{name}")


def reference_src() -> Path | None:
    """The reference's Python sources, where this host has them (``NANOENGINE_REFERENCE_SRC``, or a
    ``reference`` checkout beside this repository); GPU hosts have none."""
    for candidate in (os.environ.get("NANOENGINE_REFERENCE_SRC"), REPO.parent / "reference" / "nanoengine" / "src"):
        if candidate and (Path(candidate) / "nanoengine" / "engine" / "speculative").is_dir():
            return Path(candidate)
    return None


def load_golden(name: str):
    return torch.load(GOLDEN / name, weights_only=False)


@pytest.fixture(scope="session")
def pkg():
    return package()


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device; run it with -m gpu on a B200")
    return torch.device("cuda", 0)
