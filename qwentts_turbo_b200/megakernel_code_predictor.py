"""Code-predictor decoder with the API of the reference's
``qwentts_turbo/megakernel_code_predictor.py``.

``MegakernelCodePredictorDecoder`` mirrors the reference's pybind class
(megakernel_code_predictor.py:86-231): fp32 KV cache [5, 8, max_seq, 128], host-side position,
``decode_step_with_embedding`` returning the fp32 final-normed hidden. It calls the drop-in
launcher ``launch_cp_decode_with_embedding`` of libqtt.so.
``CodePredictorMegakernelGenerator`` mirrors megakernel_code_predictor.py:319-350.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .checkpoint import load_qwen_tts, weights_from_model
from .config import DEFAULT_DIMS, LAYER_TENSORS
from .megakernel_backbone import device_layer_table
from .weights import rope_tables

CP_HIDDEN_SIZE = DEFAULT_DIMS.hidden
CP_INTERMEDIATE_SIZE = DEFAULT_DIMS.intermediate
CP_NUM_Q_HEADS = DEFAULT_DIMS.n_q_heads
CP_NUM_KV_HEADS = DEFAULT_DIMS.n_kv_heads
CP_HEAD_DIM = DEFAULT_DIMS.head_dim
CP_Q_SIZE = CP_NUM_Q_HEADS * CP_HEAD_DIM
CP_KV_SIZE = CP_NUM_KV_HEADS * CP_HEAD_DIM
CP_NUM_LAYERS = DEFAULT_DIMS.cp_layers


class MegakernelCodePredictorDecoder:
    def __init__(self, layer_weights_flat, final_norm_weight, cos_table, sin_table, num_layers, max_seq_len):
        self.lib = _lib.load()
        self.num_layers = num_layers
        self.max_seq_len = max_seq_len
        self.final_norm_weight = final_norm_weight
        self.cos_table = cos_table
        self.sin_table = sin_table
        self.layer_weights_tensors = list(layer_weights_flat)
        self.d_layer_weights = device_layer_table(self.layer_weights_tensors, num_layers)
        dev = final_norm_weight.device
        self.k_cache = torch.zeros(num_layers, CP_NUM_KV_HEADS, max_seq_len, CP_HEAD_DIM, dtype=torch.float32,
                                   device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.g_normalized = torch.empty(CP_HIDDEN_SIZE, dtype=torch.float32, device=dev)
        self.position_ = 0
        self.attn_scale = 1.0 / math.sqrt(CP_HEAD_DIM)

    def decode_step_with_embedding(self, input_embedding: torch.Tensor) -> torch.Tensor:
        if input_embedding.dim() == 2:
            input_embedding = input_embedding.squeeze(0)
        input_embedding = input_embedding.to(torch.bfloat16).contiguous()
        cache_len = self.position_ + 1
        self.lib.launch_cp_decode_with_embedding(
            input_embedding.data_ptr(), ctypes.cast(self.d_layer_weights.data_ptr(), ctypes.POINTER(_lib.TTSLayerWeights)),
            self.final_norm_weight.data_ptr(), self.cos_table.data_ptr(), self.sin_table.data_ptr(),
            self.k_cache.data_ptr(), self.v_cache.data_ptr(), None, None, None, None, None, None, None, None,
            self.g_normalized.data_ptr(), self.num_layers, self.position_, cache_len, self.max_seq_len,
            ctypes.c_float(self.attn_scale), torch.cuda.current_stream().cuda_stream)
        _lib.check(self.lib.qtt_last_launch_status(), "launch_cp_decode_with_embedding")
        self.position_ += 1
        return self.g_normalized.clone()

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

    def set_kv_cache(self, k_cache: torch.Tensor, v_cache: torch.Tensor):
        n = k_cache.size(2)
        self.k_cache[:, :, :n] = k_cache.to(torch.float32)
        self.v_cache[:, :, :n] = v_cache.to(torch.float32)


def extract_code_predictor_weights(weights: dict, max_seq_len: int = 4096, device="cuda") -> dict:
    """Counterpart of extract_code_predictor_weights (megakernel_code_predictor.py:265-316)."""
    n = sum(1 for k in weights if k.startswith("cp.layers.") and k.endswith(".q_proj"))
    t = {k: v.to(device, dtype=torch.bfloat16).contiguous() for k, v in weights.items() if k.startswith("cp.")}
    cos, sin = rope_tables(max_seq_len, CP_HEAD_DIM, DEFAULT_DIMS.rope_theta)
    return {
        "layer_weights": [t[f"cp.layers.{i}.{name}"] for i in range(n) for name in LAYER_TENSORS],
        "final_norm_weight": t["cp.norm"],
        "cos_table": cos.to(device),
        "sin_table": sin.to(device),
        "num_layers": n,
    }


class CodePredictorMegakernelGenerator:
    def __init__(self, model_path: str | None = None, max_seq_len: int = 256, weights: dict | None = None,
                 model=None):
        if weights is None:
            if model is None:
                model = load_qwen_tts(model_path)
            weights = weights_from_model(model)
        self.weights = extract_code_predictor_weights(weights)
        self.decoder = MegakernelCodePredictorDecoder(self.weights["layer_weights"], self.weights["final_norm_weight"],
                                                      self.weights["cos_table"], self.weights["sin_table"],
                                                      self.weights["num_layers"], max_seq_len)
        self.max_seq_len = max_seq_len

    def decode_step_with_embedding(self, input_embedding: torch.Tensor) -> torch.Tensor:
        return self.decoder.decode_step_with_embedding(input_embedding)

    def reset(self):
        self.decoder.reset()

    @property
    def position(self) -> int:
        return self.decoder.position()
