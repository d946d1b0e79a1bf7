"""Backbone decoder with the API of the reference's ``qwentts_turbo/megakernel_backbone.py``.

``MegakernelTTSDecoder`` mirrors the reference's pybind class (megakernel_backbone.py:109-316):
it borrows the weight tensors, owns the bf16 KV cache [L, 8, max_seq, 128] and the output
buffers, keeps the host-side ``position_`` counter, and calls the drop-in launchers
``launch_tts_decode_with_embedding`` / ``launch_tts_decode`` of libqtt.so (the sm_100a
persistent kernel) on the current CUDA stream. ``TTSMegakernelGenerator`` mirrors the Python
wrapper (megakernel_backbone.py:412-488).

Unlike the reference, every launch is checked: a failed launch raises ``QTTError``.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .checkpoint import load_qwen_tts, weights_from_model
from .config import DEFAULT_DIMS, LAYER_TENSORS
from .weights import rope_tables

HIDDEN_SIZE = DEFAULT_DIMS.hidden
INTERMEDIATE_SIZE = DEFAULT_DIMS.intermediate
NUM_Q_HEADS = DEFAULT_DIMS.n_q_heads
NUM_KV_HEADS = DEFAULT_DIMS.n_kv_heads
HEAD_DIM = DEFAULT_DIMS.head_dim
Q_SIZE = NUM_Q_HEADS * HEAD_DIM
KV_SIZE = NUM_KV_HEADS * HEAD_DIM


def device_layer_table(layer_tensors: list, num_layers: int) -> torch.Tensor:
    """Device array of TTSLayerWeights structs (the reference copies it with cudaMemcpy,
    megakernel_backbone.py:147-151)."""
    arr = (_lib.TTSLayerWeights * num_layers)(
        *[_lib.TTSLayerWeights(*[t.data_ptr() for t in layer_tensors[11 * i:11 * i + 11]]) for i in range(num_layers)])
    host = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
    return host.to("cuda")


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class MegakernelTTSDecoder:
    """Mirror of the reference's C++ MegakernelTTSDecoder (megakernel_backbone.py:109-316)."""

    def __init__(self, embed_weight, layer_weights_flat, final_norm_weight, codec_head_weight, cos_table,
                 sin_table, num_layers, max_seq_len):
        self.lib = _lib.load()
        self.num_layers = num_layers
        self.max_seq_len = max_seq_len
        self.embed_weight = embed_weight
        self.final_norm_weight = final_norm_weight
        self.codec_head_weight = codec_head_weight
        self.cos_table = cos_table
        self.sin_table = sin_table
        self.layer_weights_tensors = list(layer_weights_flat)
        self.d_layer_weights = device_layer_table(self.layer_weights_tensors, num_layers)
        dev = embed_weight.device
        self.k_cache = torch.zeros(num_layers, NUM_KV_HEADS, max_seq_len, HEAD_DIM, dtype=torch.bfloat16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.hidden_buffer = torch.empty(HIDDEN_SIZE, dtype=torch.bfloat16, device=dev)
        self.g_normalized = torch.empty(HIDDEN_SIZE, dtype=torch.float32, device=dev)
        self.position_ = 0
        self.attn_scale = 1.0 / math.sqrt(HEAD_DIM)

    def _launch(self, emb: torch.Tensor | None, token: int | None):
        cache_len = self.position_ + 1
        args = [self.d_layer_weights.data_ptr(), self.final_norm_weight.data_ptr(), self.cos_table.data_ptr(),
                self.sin_table.data_ptr(), self.k_cache.data_ptr(), self.v_cache.data_ptr(),
                self.hidden_buffer.data_ptr(), None, None, None, None, None, None, None,
                self.g_normalized.data_ptr(), self.num_layers, self.position_, cache_len, self.max_seq_len,
                ctypes.c_float(self.attn_scale), _stream()]
        args[0] = ctypes.cast(args[0], ctypes.POINTER(_lib.TTSLayerWeights))
        if token is None:
            self.lib.launch_tts_decode_with_embedding(emb.data_ptr(), *args)
        else:
            self.lib.launch_tts_decode(int(token), self.embed_weight.data_ptr(), *args)
        _lib.check(self.lib.qtt_last_launch_status(), "launch_tts_decode")
        self.position_ += 1
        return self.g_normalized.clone()

    def decode_step(self, input_token_id: int) -> torch.Tensor:
        return self._launch(None, input_token_id)

    def decode_step_with_argmax(self, input_token_id: int) -> int:
        hidden = self.decode_step(input_token_id)
        logits = torch.matmul(hidden.to(torch.bfloat16), self.codec_head_weight.t())
        return int(logits.argmax().item())

    def decode_step_with_embedding(self, input_embedding: torch.Tensor) -> torch.Tensor:
        if input_embedding.dim() == 2:
            input_embedding = input_embedding.squeeze(0)
        input_embedding = input_embedding.to(torch.bfloat16).contiguous()
        return self._launch(input_embedding, None)

    def reset(self):
        self.position_ = 0
        self.k_cache.zero_()
        self.v_cache.zero_()

    def position(self) -> int:
        return self.position_

    def set_position(self, pos: int):
        self.position_ = int(pos)

    def get_hidden_states(self) -> torch.Tensor:
        return self.g_normalized.clone()

    def get_k_cache(self) -> torch.Tensor:
        return self.k_cache

    def get_v_cache(self) -> torch.Tensor:
        return self.v_cache

    def set_kv_cache(self, k_cache: torch.Tensor, v_cache: torch.Tensor):
        n = k_cache.size(2)
        self.k_cache[:, :, :n] = k_cache.to(torch.bfloat16)
        self.v_cache[:, :, :n] = v_cache.to(torch.bfloat16)


def extract_backbone_weights(weights: dict, max_seq_len: int = 4096, rope_theta: float | None = None,
                             device="cuda") -> dict:
    """Counterpart of _extract_tts_backbone_weights (megakernel_backbone.py:358-409) working
    on a weight dict (qwentts_turbo_b200.weights naming)."""
    n = sum(1 for k in weights if k.startswith("talker.layers.") and k.endswith(".q_proj"))
    t = {k: v.to(device, dtype=torch.bfloat16).contiguous() for k, v in weights.items() if k.startswith("talker.")}
    layer_weights = [t[f"talker.layers.{i}.{name}"] for i in range(n) for name in LAYER_TENSORS]
    cos, sin = rope_tables(max_seq_len, HEAD_DIM, rope_theta or DEFAULT_DIMS.rope_theta)
    return {
        "embed_weight": t["talker.codec_embedding"],
        "layer_weights": layer_weights,
        "final_norm_weight": t["talker.norm"],
        "codec_head_weight": t["talker.codec_head"],
        "cos_table": cos.to(device),
        "sin_table": sin.to(device),
        "num_layers": n,
        "vocab_size": t["talker.codec_embedding"].shape[0],
    }


class TTSMegakernelGenerator:
    """Mirror of the reference's TTSMegakernelGenerator (megakernel_backbone.py:412-488).

    ``weights`` (a weight dict) replaces loading a checkpoint when given; otherwise ``model``
    (a loaded Qwen3-TTS model object) or ``model_path`` (needs the qwen_tts package)."""

    def __init__(self, model_path: str = "Qwen/Qwen3-TTS-12Hz-0.6B-Base", model=None, max_seq_len: int = 4096,
                 weights: dict | None = None):
        if weights is None:
            if model is None:
                model = load_qwen_tts(model_path)
            weights = weights_from_model(model)
        w = extract_backbone_weights(weights, max_seq_len)
        self._w = w
        self.decoder = MegakernelTTSDecoder(w["embed_weight"], w["layer_weights"], w["final_norm_weight"],
                                            w["codec_head_weight"], w["cos_table"], w["sin_table"],
                                            w["num_layers"], max_seq_len)
        self.max_seq_len = max_seq_len
        self.vocab_size = w["vocab_size"]

    def decode_step(self, input_token_id: int) -> torch.Tensor:
        return self.decoder.decode_step(input_token_id)

    def decode_step_with_argmax(self, input_token_id: int) -> int:
        return self.decoder.decode_step_with_argmax(input_token_id)

    def decode_step_with_embedding(self, input_embedding: torch.Tensor) -> torch.Tensor:
        return self.decoder.decode_step_with_embedding(input_embedding)

    def reset(self):
        self.decoder.reset()

    def set_position(self, pos: int):
        self.decoder.set_position(pos)

    def set_kv_cache(self, k_cache: torch.Tensor, v_cache: torch.Tensor):
        self.decoder.set_kv_cache(k_cache, v_cache)

    def get_k_cache(self) -> torch.Tensor:
        return self.decoder.get_k_cache()

    def get_v_cache(self) -> torch.Tensor:
        return self.decoder.get_v_cache()

    @property
    def position(self) -> int:
        return self.decoder.position()
