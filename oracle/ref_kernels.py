"""ctypes access to the reference's own CUDA decode kernels, compiled from
hamza1brh/qwenTTS-turbo's qwentts_turbo/csrc/ sources by oracle/Makefile into oracle/_ref/.

TEST INFRASTRUCTURE ONLY (GPU parity oracle and same-GPU baseline). It reproduces what the
reference's pybind classes do around the launchers (megakernel_backbone.py:109-316,
megakernel_code_predictor.py:86-231): device layer-pointer table, KV caches, scratch buffers,
cache_len = position + 1, output = g_normalized.
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
TTS_SO = os.path.join(REF_DIR, "libref_tts.so")
CP_SO = os.path.join(REF_DIR, "libref_cp.so")

_P = ctypes.c_void_p
_ARGS = [_P] * 16 + [ctypes.c_int] * 4 + [ctypes.c_float, _P]


def available() -> bool:
    return os.path.exists(TTS_SO) and os.path.exists(CP_SO)


def _layer_table(layer_tensors, n):
    ptrs = []
    for t in layer_tensors[: 11 * n]:
        ptrs.append(t.data_ptr())
    host = torch.tensor(ptrs, dtype=torch.int64)
    return host.to("cuda")


class RefDecoder:
    """One reference megakernel (backbone: bf16 KV, CP: fp32 KV) with its own state."""

    def __init__(self, kind: str, layer_tensors, final_norm, cos, sin, num_layers: int, max_seq_len: int):
        assert kind in ("tts", "cp")
        self.kind = kind
        self.lib = ctypes.CDLL(TTS_SO if kind == "tts" else CP_SO)
        self.fn = self.lib.launch_tts_decode_with_embedding if kind == "tts" else self.lib.launch_cp_decode_with_embedding
        self.fn.restype = None
        self.fn.argtypes = _ARGS
        self.keep = list(layer_tensors)
        self.table = _layer_table(layer_tensors, num_layers)
        self.final_norm, self.cos, self.sin = final_norm, cos, sin
        self.num_layers, self.max_seq_len = num_layers, max_seq_len
        kv_dtype = torch.bfloat16 if kind == "tts" else torch.float32
        self.k = torch.zeros(num_layers, 8, max_seq_len, 128, dtype=kv_dtype, device="cuda")
        self.v = torch.zeros_like(self.k)
        hb_dtype = torch.bfloat16 if kind == "tts" else torch.float32
        f = dict(dtype=torch.float32, device="cuda")
        self.hidden_buffer = torch.empty(1024, dtype=hb_dtype, device="cuda")
        self.g_act = torch.empty(1024, **f)
        self.g_res = torch.empty(1024, **f)
        self.g_q = torch.empty(2048, **f)
        self.g_k = torch.empty(1024, **f)
        self.g_v = torch.empty(1024, **f)
        self.g_attn = torch.empty(2048, **f)
        self.g_mlp = torch.empty(3072, **f)
        self.g_norm = torch.empty(1024, **f)
        self.position = 0
        self.scale = 1.0 / math.sqrt(128.0)

    def step(self, emb_bf16: torch.Tensor) -> torch.Tensor:
        emb = emb_bf16.reshape(-1).to(torch.bfloat16).contiguous()
        assert self.position < self.max_seq_len
        self.fn(emb.data_ptr(), self.table.data_ptr(), self.final_norm.data_ptr(), self.cos.data_ptr(),
                self.sin.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), self.hidden_buffer.data_ptr(),
                self.g_act.data_ptr(), self.g_res.data_ptr(), self.g_q.data_ptr(), self.g_k.data_ptr(),
                self.g_v.data_ptr(), self.g_attn.data_ptr(), self.g_mlp.data_ptr(), self.g_norm.data_ptr(),
                self.num_layers, self.position, self.position + 1, self.max_seq_len, self.scale,
                torch.cuda.current_stream().cuda_stream)
        self.position += 1
        return self.g_norm.clone()
