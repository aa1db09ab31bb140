"""B200-native speculative-decoding step for nanoengine (Qwen3), a drop-in for the runner's
speculative path: n-gram drafting, (k+1)-token verify forward over the paged KV cache,
greedy / rejection-sampling acceptance and KV commit, all as hand-written sm_100a CUDA kernels
behind the C ABI declared in ``include/nespec.h``.

The package directory name contains hyphens, so import it with
``importlib.import_module("inference-engine-from-scratch_b200")``.
"""

from .config import QWEN3_0_6B, QWEN3_8B_SHAPE, SMALL_TEST, Qwen3Config, SpeculativeSettings
from .weights import cast_weights, make_prompt, make_prompts, make_weights

__all__ = [
    "QWEN3_0_6B",
    "QWEN3_8B_SHAPE",
    "SMALL_TEST",
    "Qwen3Config",
    "SpeculativeSettings",
    "cast_weights",
    "make_prompt",
    "make_prompts",
    "make_weights",
]
