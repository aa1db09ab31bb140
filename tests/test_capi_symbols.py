"""The C-ABI library builds for sm_100a, loads without a GPU and exports every symbol of include/nespec.h."""

from __future__ import annotations

import ctypes
import re

from tests.conftest import REPO, submodule


def header_symbols() -> list[str]:
    text = (REPO / "include" / "nespec.h").read_text()
    return re.findall(r"^NE_API [^(]*?\b(ne_\w+)\(", text, flags=re.M)


def test_library_exports_every_header_symbol() -> None:
    submodule("build").build()
    lib = ctypes.CDLL(str(REPO / "inference-engine-from-scratch_b200" / "libnespec.so"))
    names = header_symbols()
    assert len(names) >= 19
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_declares_exactly_the_header_symbols() -> None:
    lib_mod = submodule("_lib")
    assert sorted(lib_mod.EXPORTS) == sorted(header_symbols())
    lib = lib_mod.load()
    assert lib.ne_abi_version() == 2
    assert lib.ne_status_string(0) == b"ok"


def test_invalid_arguments_are_rejected_without_a_gpu() -> None:
    lib = submodule("_lib").load()
    assert lib.ne_model_create(None, None) == 1
    assert lib.ne_gemm_bf16(None, None, None, 1, 128, 64, None, None) == 1
    cfg = submodule("_lib").ModelConfig(vocab_size=4096, hidden_size=256, intermediate_size=512, num_layers=1,
                                        num_heads=4, num_kv_heads=2, head_dim=64, rms_norm_eps=1e-6, block_size=16,
                                        kv_int8=0, weight_int8=0, num_cache_slots=17, max_positions=64)
    handle = ctypes.c_void_p()
    assert lib.ne_model_create(ctypes.byref(cfg), ctypes.byref(handle)) == 1  # head_dim must be 128
