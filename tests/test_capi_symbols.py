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
    assert lib.ne_abi_version() == lib_mod.ABI_VERSION
    header = (REPO / "include" / "nespec.h").read_text()
    assert f"#define NE_ABI_VERSION {lib_mod.ABI_VERSION}" in header
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


def test_new_entry_points_refuse_bad_arguments_without_a_gpu() -> None:
    """Argument checks of the sampling, tensor-parallel, sharing and int8 entries (no device work)."""
    _lib = submodule("_lib")
    lib = _lib.load()
    assert lib.ne_sampling_buffer_bytes(None, 16) == 0
    assert lib.ne_model_set_sampling_buffer(None, None, 0, 0) == 1
    assert lib.ne_verify_logits(None, None, 1, 4, None, None, None, 4096, 5, None, 0, None, None, None) == 1
    assert lib.ne_state_share_blocks(None, 0, None, 0, 1, None, None) == 1
    assert lib.ne_gemm_w8(None, None, None, None, 1, 128, 64, None, None) == 1
    assert lib.ne_tp_unique_id(None, None) == 1
    assert lib.ne_model_set_tp(None, b"libnccl.so.2", 0, 2, None) == 1
    # an unknown NCCL library path is reported, not crashed on
    buf = (ctypes.c_char * 128)()
    assert lib.ne_tp_unique_id(b"/nonexistent/libnccl.so.2", buf) == _lib_status(lib, "unsupported")
    cfg = _lib.ModelConfig(vocab_size=4096, hidden_size=256, intermediate_size=512, num_layers=1, num_heads=4,
                           num_kv_heads=2, head_dim=128, rms_norm_eps=1e-6, block_size=16, kv_int8=0, weight_int8=0,
                           num_cache_slots=17, max_positions=64, lm_rows=100, lm_offset=0)
    handle = ctypes.c_void_p()
    assert lib.ne_model_create(ctypes.byref(cfg), ctypes.byref(handle)) == 1  # LM-head rows: whole 128-row tiles
    cfg.lm_rows, cfg.hidden_size = 0, 768
    assert lib.ne_model_create(ctypes.byref(cfg), ctypes.byref(handle)) == 4  # hidden 768: no RMSNorm variant


def _lib_status(lib, name: str) -> int:
    return {"invalid": 1, "cuda": 2, "device": 3, "unsupported": 4, "workspace": 5}[name]


def test_quality_report_renders_the_reference_table() -> None:
    quality = submodule("quality")
    report = quality.QualityReport(12.5, 13.0, 0.9375, 6, 8, "weights=int8, kv_cache=int8")
    text = quality.render_quality_markdown(report)
    assert "| Perplexity on the fixed token sequence | 12.500 | 13.000 |" in text
    assert "| Greedy token agreement | 100% | 93.8% |" in text
    assert "| Identical completions | 8 | 6 |" in text
