"""ctypes binding of ``libnespec.so`` (the C ABI in include/nespec.h).

The library is the product: there is no Python or torch fallback for any kernel. If the library
is missing or a CUDA device is absent, the calls below raise instead of computing anything.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_int32, c_longlong, c_size_t, c_void_p
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "libnespec.so"
ABI_VERSION = 3  # NE_ABI_VERSION of include/nespec.h

NE_OK = 0
NE_LM_NONE, NE_LM_ARGMAX, NE_LM_LOGITS = 0, 1, 2
NE_SEQ_IGNORE_EOS, NE_SEQ_FINISHED = 1, 2
NE_FINISH_NONE, NE_FINISH_STOP, NE_FINISH_LENGTH = 0, 1, 2
DEVICE_STATUS_BITS = {
    1: "a bounded device wait ran out",
    2: "a slot or block index outside the KV pool",
    4: "the free-block FIFO could not cover a reservation (out of KV blocks)",
    8: "a token id outside the vocabulary",
    16: "a sequence outgrew its history or block-table row",
    32: "a sequence with temperature > 0 on a model without a sampling buffer",
}

# (name, restype, argtypes) for every entry point of include/nespec.h
TP_HANDLE_BYTES = 64  # NE_TP_HANDLE_BYTES (CUDA IPC handle)

EXPORTS = {
    "ne_abi_version": (c_int, []),
    "ne_model_step_wait_record": (c_int, [c_void_p, c_void_p, c_int]),
    "ne_model_step_trace_bytes": (c_size_t, [c_void_p]),
    "ne_model_set_step_trace": (c_int, [c_void_p, c_void_p, c_size_t]),
    "ne_status_string": (ctypes.c_char_p, [c_int]),
    "ne_read_status": (c_int, [c_void_p, c_int, POINTER(c_int32), c_void_p]),
    "ne_model_create": (c_int, [c_void_p, POINTER(c_void_p)]),
    "ne_model_destroy": (c_int, [c_void_p]),
    "ne_model_set_layer": (c_int, [c_void_p, c_int, c_void_p]),
    "ne_model_set_head": (c_int, [c_void_p, c_void_p]),
    "ne_model_workspace_bytes": (c_int, [c_void_p, c_int, c_int, POINTER(c_size_t)]),
    "ne_model_set_workspace": (c_int, [c_void_p, c_void_p, c_size_t, c_int, c_int]),
    "ne_model_status_word": (c_void_p, [c_void_p]),
    "ne_forward": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "ne_state_reset_blocks": (c_int, [c_void_p, c_void_p]),
    "ne_state_free_slots": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "ne_ngram_propose": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "ne_prefill": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "ne_state_share_blocks": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "ne_spec_step": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "ne_draft_sync": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "ne_spec_step_drafted": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p,
                                     c_void_p]),
    "ne_model_lm_start": (c_void_p, [c_void_p]),
    "ne_gemm_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "ne_gemm_w8": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "ne_paged_attention": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int,
         c_longlong, c_void_p, c_size_t, c_void_p, c_void_p],
    ),
    "ne_paged_attention_static_scratch": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int,
         c_longlong, c_int, c_void_p, c_void_p],
    ),
    "ne_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]),
    "ne_sampling_buffer_bytes": (c_size_t, [c_void_p, c_int]),
    "ne_model_set_sampling_buffer": (c_int, [c_void_p, c_void_p, c_size_t, c_int]),
    "ne_verify_logits": (
        c_int,
        [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_size_t, c_void_p,
         c_void_p, c_void_p],
    ),
    "ne_verify_logits_drafted": (
        c_int,
        [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int,
         c_void_p, c_size_t, c_void_p, c_void_p, c_void_p],
    ),
    "ne_tp_unique_id": (c_int, [ctypes.c_char_p, c_void_p]),
    "ne_model_set_tp": (c_int, [c_void_p, ctypes.c_char_p, c_int, c_int, c_void_p]),
    "ne_model_tp_exchange_create": (c_int, [c_void_p, c_int, c_void_p]),
    "ne_model_set_kv_shadow": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int]),
    "ne_kv_shadow_fill": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    "ne_kv_shadow_clear": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "ne_model_tp_exchange_open": (c_int, [c_void_p, c_void_p]),
    "ne_model_launch_count": (c_longlong, [c_void_p]),
    "ne_model_profile_begin": (c_int, [c_void_p, c_void_p]),
    "ne_model_profile_end": (c_int, [c_void_p, POINTER(c_float), POINTER(c_int), c_int]),
}

KERNEL_KINDS = ("embed", "rmsnorm", "gemm_qkv", "attention", "gemm_o", "gemm_gateup", "gemm_down", "lm_head",
                "ngram", "plan", "accept", "other", "sample", "collective", "step")


class ModelConfig(ctypes.Structure):
    _fields_ = [
        ("vocab_size", c_int),
        ("hidden_size", c_int),
        ("intermediate_size", c_int),
        ("num_layers", c_int),
        ("num_heads", c_int),
        ("num_kv_heads", c_int),
        ("head_dim", c_int),
        ("rms_norm_eps", c_float),
        ("block_size", c_int),
        ("kv_int8", c_int),
        ("weight_int8", c_int),
        ("num_cache_slots", c_longlong),
        ("max_positions", c_int),
        ("lm_rows", c_int),
        ("lm_offset", c_int),
    ]


class LayerWeights(ctypes.Structure):
    _fields_ = [(name, c_void_p) for name in (
        "w_qkv", "w_o", "w_gateup", "w_down", "ln_in", "ln_post", "q_norm", "k_norm",
        "k_cache", "v_cache", "k_scale", "v_scale",
        "w_qkv_scale", "w_o_scale", "w_gateup_scale", "w_down_scale")]


class HeadWeights(ctypes.Structure):
    _fields_ = [(name, c_void_p) for name in ("embed", "lm_head", "final_norm", "rope_cos", "rope_sin")]


class Rows(ctypes.Structure):
    _fields_ = [
        ("max_rows", c_int),
        ("num_seqs", c_int),
        ("num_rows", c_void_p),
        ("token_ids", c_void_p),
        ("positions", c_void_p),
        ("slot_mapping", c_void_p),
        ("q_start", c_void_p),
        ("q_len", c_void_p),
        ("block_tables", c_void_p),
        ("table_index", c_void_p),
        ("block_table_stride", c_int),
        ("max_context", c_int),
        ("max_q_len", c_int),
        ("lm_rows", c_void_p),
        ("lm_count", c_void_p),
        ("lm_max", c_int),
    ]


class BatchState(ctypes.Structure):
    _fields_ = [
        ("max_seqs", c_int),
        ("history_stride", c_int),
        ("block_table_stride", c_int),
        ("num_blocks", c_int),
        ("history", c_void_p),
        ("seq_len", c_void_p),
        ("num_cached", c_void_p),
        ("num_prompt", c_void_p),
        ("max_new_tokens", c_void_p),
        ("flags", c_void_p),
        ("temperature", c_void_p),
        ("top_p", c_void_p),
        ("rng_seed", c_void_p),
        ("rng_draws", c_void_p),
        ("block_tables", c_void_p),
        ("num_blocks_used", c_void_p),
        ("num_shared_blocks", c_void_p),
        ("free_ring", c_void_p),
        ("ring_head_tail", c_void_p),
        ("stop_ids", c_void_p),
        ("num_stop_ids", c_int),
    ]


class DraftRows(ctypes.Structure):
    _fields_ = [("logits", c_void_p), ("start", c_void_p), ("stride", c_int), ("rows", c_int), ("stats", c_void_p)]


class StepOutputs(ctypes.Structure):
    _fields_ = [(name, c_void_p) for name in ("tokens", "count", "finish", "proposed", "accepted")]


_LIB = None


def load(required: bool = True):
    """Load the library once. Raises if it is missing (build it with ``__graft_entry__.build()``)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIBRARY_PATH.exists():
        if not required:
            return None
        raise RuntimeError(
            f"{LIBRARY_PATH.name} is not built; the B200 speculative step has no fallback. "
            "Run __graft_entry__.build() (nvcc, sm_100a) first."
        )
    lib = ctypes.CDLL(str(LIBRARY_PATH))
    for name, (restype, argtypes) in EXPORTS.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


class NativeError(RuntimeError):
    pass


def check(status: int, what: str) -> None:
    if status != NE_OK:
        message = load().ne_status_string(status).decode()
        raise NativeError(f"{what} failed: {message} (status {status})")


def describe_device_status(word: int) -> str:
    return "; ".join(text for bit, text in DEVICE_STATUS_BITS.items() if word & bit) or "ok"


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class _DeviceArray:
    """A device array the library owns, seen by torch through ``__cuda_array_interface__``."""

    def __init__(self, address: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (address, False), "version": 3}


def device_int32(address: int, n: int, device) -> torch.Tensor:
    """A copy of ``n`` int32 values at a device address returned by the library."""
    return torch.as_tensor(_DeviceArray(address, n, "<i4"), device=device).clone()


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the B200 path has no CPU fallback)")
