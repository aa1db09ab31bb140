"""Device-resident Qwen3 weights, KV pool and workspace bound to one ``ne_model`` handle.

HBM layout (all bf16 unless noted; one CUDA device):

* per layer: ``w_qkv`` = cat(q_proj, k_proj, v_proj) ``[(nh + 2 nkv) * 128, H]``; ``w_o`` ``[H, nh*128]``;
  ``w_gateup`` = gate/up interleaved in 64-row groups ``[2 I, H]`` (so one 128-row GEMM tile holds 64
  gate rows and the 64 matching up rows and the SwiGLU fuses into its epilogue); ``w_down`` ``[H, I]``;
  the four RMSNorm weights;
* ``embed`` ``[V, H]`` (also the LM head when tied), ``final_norm`` ``[H]``, RoPE cos/sin tables
  ``[max_positions, 128]`` computed exactly as models/qwen3.py:47-57 (fp32 angles, cast to bf16);
* the KV pool: one tensor ``[L, 2, num_slots + 1, nkv, 128]`` whose ``[l, 0]`` / ``[l, 1]`` views are the
  reference's per-layer key / value caches (engine/memory/kv_cache_pool.py:34-69, last row = scratch
  slot); an int8 pool adds ``[L, 2, num_slots + 1, nkv]`` bf16 scales;
* int8 weights (``weight_int8``): the four projections become int8 ``[out, in]`` in the same row order
  plus one bf16 scale per output row (models/int8_quantization.py:30-73, the LM head stays bf16);
* the workspace (activations, row metadata, argmax keys), sized for ``max_rows`` token rows.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .config import Qwen3Config


def rope_tables(max_positions: int, head_dim: int, theta: float, dtype=torch.bfloat16):
    """cos / sin ``[max_positions, head_dim]`` with the arithmetic of models/qwen3.py:47-57."""
    exponents = torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim
    inverse = 1.0 / (theta**exponents)
    angles = torch.arange(max_positions).float()[:, None] * inverse
    angles = torch.cat((angles, angles), dim=-1)
    return angles.cos().to(dtype), angles.sin().to(dtype)


INT8_MAX = 127
MIN_SCALE = 1e-8


def quantize_rows(values: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """One symmetric int8 scale per row (quantize_vectors, models/int8_quantization.py:30-34): the
    scale max|w| / 127 in fp32 (at least 1e-8), stored in the weight dtype; q = round(w / scale)."""
    scales = values.abs().amax(dim=-1, keepdim=True).float().clamp(min=MIN_SCALE) / INT8_MAX
    quantized = torch.round(values.float() / scales).clamp(-INT8_MAX, INT8_MAX).to(torch.int8)
    return quantized, scales.to(values.dtype)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, group: int = 64) -> torch.Tensor:
    rows, hidden = gate.shape
    return torch.stack((gate.view(rows // group, group, hidden), up.view(rows // group, group, hidden)), dim=1).reshape(
        2 * rows, hidden
    )


class B200Model:
    """Packs a HF-named state dict onto one GPU and binds it to the native ``ne_model``."""

    def __init__(
        self,
        cfg: Qwen3Config,
        weights: dict[str, torch.Tensor],
        num_slots: int,
        device: torch.device | str = "cuda",
        max_positions: int = 4096,
        kv_int8: bool = False,
        max_rows: int = 4096,
        max_seqs: int = 256,
        weight_int8: bool = False,
        tp=None,
        lm_offset: int = 0,
        kv_copy_blocks: int = 0,
    ) -> None:
        """``tp`` (tp.TensorParallel): this process is one rank of a split model; ``cfg`` is then the
        rank's shape (tp.rank_config), ``weights`` its shard (tp.shard_weights / make_sharded_weights)
        and ``lm_offset`` the first vocabulary id of its LM-head rows. ``kv_copy_blocks`` (int8 KV):
        room for that many dequantised copies of shared prefix blocks (ne_model_set_kv_shadow)."""
        self.lib = _lib.load()
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("B200Model lives on a CUDA device; the oracle is the CPU path")
        self.num_slots = num_slots
        self.max_positions = max_positions
        self.kv_int8 = kv_int8
        self.weight_int8 = weight_int8
        self.max_rows = max_rows
        self.max_seqs = max_seqs
        bf16 = torch.bfloat16
        dev = self.device

        def put(t: torch.Tensor) -> torch.Tensor:
            return t.to(device=dev, dtype=bf16).contiguous()

        L, nkv, d = cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim

        def proj(name: str) -> tuple[torch.Tensor, torch.Tensor | None]:
            """A projection in the model dtype, or its int8 rows and bf16 row scales. Quantised on
            the host CPU like the reference's CPU run: the same torch ops on the GPU were seen to
            give a different int8 value for rare elements (a quotient near .5)."""
            if not weight_int8:
                return put(weights[name]), None
            q, s = quantize_rows(weights[name].to("cpu", bf16))
            return q.to(dev).contiguous(), s.to(dev).contiguous()

        self.layers: list[dict[str, torch.Tensor]] = []
        for layer in range(L):
            p = f"model.layers.{layer}."
            parts = [proj(p + f"self_attn.{n}_proj.weight") for n in ("q", "k", "v")]
            o, o_s = proj(p + "self_attn.o_proj.weight")
            gate, gate_s = proj(p + "mlp.gate_proj.weight")
            up, up_s = proj(p + "mlp.up_proj.weight")
            down, down_s = proj(p + "mlp.down_proj.weight")
            entry = {
                "w_qkv": torch.cat([t for t, _ in parts], dim=0).contiguous(),
                "w_o": o,
                "w_gateup": interleave_gate_up(gate, up).contiguous(),
                "w_down": down,
                "ln_in": put(weights[p + "input_layernorm.weight"]),
                "ln_post": put(weights[p + "post_attention_layernorm.weight"]),
                "q_norm": put(weights[p + "self_attn.q_norm.weight"]),
                "k_norm": put(weights[p + "self_attn.k_norm.weight"]),
            }
            if weight_int8:
                entry["w_qkv_scale"] = torch.cat([t for _, t in parts], dim=0).reshape(-1).contiguous()
                entry["w_o_scale"] = o_s.reshape(-1).contiguous()
                entry["w_gateup_scale"] = interleave_gate_up(gate_s, up_s).reshape(-1).contiguous()
                entry["w_down_scale"] = down_s.reshape(-1).contiguous()
            self.layers.append(entry)
        self.embed = put(weights["model.embed_tokens.weight"])
        head = weights.get("lm_head.weight")
        if tp is not None and head is None:
            raise ValueError("a tensor-parallel rank needs its LM-head shard (lm_head.weight)")
        tied = head is None or (cfg.tie_word_embeddings and tp is None)
        self.lm_head = self.embed if tied else put(head)
        self.tp = tp
        self.lm_offset = lm_offset
        self.final_norm = put(weights["model.norm.weight"])
        cos, sin = rope_tables(max_positions, d, cfg.rope_theta)
        self.rope_cos, self.rope_sin = cos.to(dev), sin.to(dev)

        cache_dtype = torch.int8 if kv_int8 else bf16
        self.kv = torch.zeros((L, 2, num_slots + 1, nkv, d), dtype=cache_dtype, device=dev)
        self.kv_scales = torch.zeros((L, 2, num_slots + 1, nkv), dtype=bf16, device=dev) if kv_int8 else None

        config = _lib.ModelConfig(
            vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
            num_layers=L, num_heads=cfg.num_attention_heads, num_kv_heads=nkv, head_dim=d,
            rms_norm_eps=cfg.rms_norm_eps, block_size=16, kv_int8=int(kv_int8), weight_int8=int(weight_int8),
            num_cache_slots=num_slots + 1, max_positions=max_positions,
            lm_rows=0 if tp is None else self.lm_head.shape[0], lm_offset=0 if tp is None else lm_offset,
        )
        handle = ctypes.c_void_p()
        _lib.check(self.lib.ne_model_create(ctypes.byref(config), ctypes.byref(handle)), "ne_model_create")
        self.handle = handle
        if tp is not None and tp.world > 1:
            uid = ctypes.create_string_buffer(tp.unique_id, 128)
            _lib.check(self.lib.ne_model_set_tp(handle, tp.nccl_library.encode(), tp.rank, tp.world, uid),
                       "ne_model_set_tp")
        from .tp import open_exchange

        self.peer_exchange = tp is not None and open_exchange(self.lib, handle, tp, max_rows)
        self._layer_structs = []
        for layer, w in enumerate(self.layers):
            lw = _lib.LayerWeights(
                w_qkv=w["w_qkv"].data_ptr(), w_o=w["w_o"].data_ptr(), w_gateup=w["w_gateup"].data_ptr(),
                w_down=w["w_down"].data_ptr(), ln_in=w["ln_in"].data_ptr(), ln_post=w["ln_post"].data_ptr(),
                q_norm=w["q_norm"].data_ptr(), k_norm=w["k_norm"].data_ptr(),
                k_cache=self.k_cache(layer).data_ptr(), v_cache=self.v_cache(layer).data_ptr(),
                k_scale=self.kv_scales[layer, 0].data_ptr() if kv_int8 else None,
                v_scale=self.kv_scales[layer, 1].data_ptr() if kv_int8 else None,
                **{k: w[k].data_ptr() for k in ("w_qkv_scale", "w_o_scale", "w_gateup_scale", "w_down_scale")
                   if weight_int8},
            )
            _lib.check(self.lib.ne_model_set_layer(handle, layer, ctypes.byref(lw)), "ne_model_set_layer")
            self._layer_structs.append(lw)
        hw = _lib.HeadWeights(
            embed=self.embed.data_ptr(), lm_head=self.lm_head.data_ptr(), final_norm=self.final_norm.data_ptr(),
            rope_cos=self.rope_cos.data_ptr(), rope_sin=self.rope_sin.data_ptr(),
        )
        _lib.check(self.lib.ne_model_set_head(handle, ctypes.byref(hw)), "ne_model_set_head")
        self._head_struct = hw
        nbytes = ctypes.c_size_t()
        _lib.check(self.lib.ne_model_workspace_bytes(handle, max_rows, max_seqs, ctypes.byref(nbytes)),
                   "ne_model_workspace_bytes")
        self.workspace = torch.empty(nbytes.value + 256, dtype=torch.uint8, device=dev)
        base = (self.workspace.data_ptr() + 255) // 256 * 256
        _lib.check(self.lib.ne_model_set_workspace(handle, base, nbytes.value, max_rows, max_seqs),
                   "ne_model_set_workspace")
        self.status_ptr = self.lib.ne_model_status_word(handle)
        self.kv_copies = None
        self._copy_free: list[tuple[int, int]] = []
        if kv_copy_blocks > 0 and kv_int8:
            if num_slots % 16:
                raise ValueError("dequantised block copies need a pool of whole 16-slot blocks")
            self.kv_copies = torch.empty((L, 2, kv_copy_blocks * 16, nkv, d), dtype=bf16, device=dev)
            self.kv_copy_map = torch.full((num_slots // 16,), -1, dtype=torch.int32, device=dev)
            _lib.check(self.lib.ne_model_set_kv_shadow(handle, self.kv_copies.data_ptr(), kv_copy_blocks,
                                                       self.kv_copy_map.data_ptr(), num_slots // 16),
                       "ne_model_set_kv_shadow")
            self._copy_free = [(0, kv_copy_blocks)]

    # ------------------------------------------------------------------ dequantised block copies
    def take_kv_copies(self, blocks: int) -> int | None:
        """First index of ``blocks`` contiguous free copies, or None (no copies / no room: the
        attention then converts those blocks itself)."""
        for i, (start, n) in enumerate(self._copy_free):
            if n >= blocks:
                self._copy_free[i] = (start + blocks, n - blocks)
                return start
        return None

    def return_kv_copies(self, first: int, blocks: int) -> None:
        free = sorted(self._copy_free + [(first, blocks)])
        merged: list[tuple[int, int]] = []
        for start, n in free:
            if merged and merged[-1][0] + merged[-1][1] == start:
                merged[-1] = (merged[-1][0], merged[-1][1] + n)
            elif n:
                merged.append((start, n))
        self._copy_free = merged

    # ------------------------------------------------------------------ views
    def k_cache(self, layer: int) -> torch.Tensor:
        return self.kv[layer, 0]

    def v_cache(self, layer: int) -> torch.Tensor:
        return self.kv[layer, 1]

    @property
    def scratch_slot(self) -> int:
        return self.num_slots

    @property
    def weight_bytes(self) -> int:
        """Unique weight bytes one verify step streams (linear weights + LM head + norms)."""
        seen, total = set(), 0
        tensors = [t for w in self.layers for t in w.values()] + [self.lm_head, self.final_norm]
        for t in tensors:
            if t.data_ptr() not in seen:
                seen.add(t.data_ptr())
                total += t.numel() * t.element_size()
        return total

    def kv_bytes_per_token(self) -> int:
        """engine/memory/kv_cache_pool.py:11-24."""
        per_head = self.cfg.head_dim * (1 if self.kv_int8 else 2) + (2 if self.kv_int8 else 0)
        return 2 * self.cfg.num_hidden_layers * self.cfg.num_key_value_heads * per_head

    # ------------------------------------------------------------------ status
    def read_status(self, clear: bool = True) -> int:
        word = ctypes.c_int32()
        _lib.check(self.lib.ne_read_status(self.status_ptr, int(clear), ctypes.byref(word), _lib.stream_handle()),
                   "ne_read_status")
        return word.value

    def raise_on_device_error(self) -> None:
        word = self.read_status(clear=True)
        if word:
            raise _lib.NativeError(f"device reported: {_lib.describe_device_status(word)} (0x{word:x})")

    def close(self) -> None:
        """Destroy the native model. A split model with a peer exchange is collective here: every
        rank's kernels must be done before any rank frees its exchange region."""
        if getattr(self, "handle", None) is not None and self.handle.value:
            if getattr(self, "peer_exchange", False):
                from .tp import quiesce

                quiesce(self.device)
            self.lib.ne_model_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self) -> None:
        try:
            if getattr(self, "peer_exchange", False):
                return  # never free an exchange region without the collective close()
            self.close()
        except Exception:
            pass
