"""Python handle on the libqtt engine API (include/qtt.h section 2).

``DeviceModel`` puts a weight dict (names as in :mod:`qwentts_turbo_b200.weights`) on the GPU
and builds the ``qtt_weights`` view; ``Engine`` owns a ``qtt_engine`` (per-utterance KV caches
and device-side decode state) and exposes prefill / frame-loop / step calls on the current
torch CUDA stream.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .config import DEFAULT_DIMS, LAYER_TENSORS, ModelDims, frame_weight_bytes
from .weights import rope_tables


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _stream_handle(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class _DevArray:
    """Zero-copy torch view of a raw device pointer (CUDA array interface)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 2, "strides": None}


def layer_struct(tensors) -> _lib.TTSLayerWeights:
    """TTSLayerWeights from 11 device tensors in LAYER_TENSORS order."""
    return _lib.TTSLayerWeights(*[_ptr(t) for t in tensors])


class DeviceModel:
    """Device-resident bf16 weights + RoPE tables and the C structs that point at them."""

    def __init__(self, weights: dict, dims: ModelDims = DEFAULT_DIMS, device: int = 0, rope_rows: int = 4096,
                 backbone_layers: int | None = None, cp_layers: int | None = None):
        self.dims = dims
        self.device = device
        dev = torch.device("cuda", device)
        self.nb = dims.backbone_layers if backbone_layers is None else backbone_layers
        self.nc = dims.cp_layers if cp_layers is None else cp_layers
        self.t = {k: v.to(dev, dtype=torch.bfloat16).contiguous() for k, v in weights.items()}
        cos, sin = rope_tables(rope_rows, dims.head_dim, dims.rope_theta)
        self.cos, self.sin = cos.to(dev), sin.to(dev)
        self.rope_rows = rope_rows
        self.bb_layers = (_lib.TTSLayerWeights * self.nb)(
            *[layer_struct([self.t[f"talker.layers.{i}.{n}"] for n in LAYER_TENSORS]) for i in range(self.nb)])
        self.cp_layers = (_lib.TTSLayerWeights * self.nc)(
            *[layer_struct([self.t[f"cp.layers.{i}.{n}"] for n in LAYER_TENSORS]) for i in range(self.nc)])
        qw = _lib.QttWeights()
        qw.backbone_layers = ctypes.cast(self.bb_layers, ctypes.POINTER(_lib.TTSLayerWeights))
        qw.backbone_norm = _ptr(self.t["talker.norm"])
        qw.codec_embedding = _ptr(self.t["talker.codec_embedding"])
        qw.codec_head = _ptr(self.t["talker.codec_head"])
        qw.cp_layers = ctypes.cast(self.cp_layers, ctypes.POINTER(_lib.TTSLayerWeights))
        qw.cp_norm = _ptr(self.t["cp.norm"])
        for g in range(dims.n_groups - 1):
            qw.cp_codec_embedding[g] = _ptr(self.t[f"cp.codec_embedding.{g}"])
            qw.cp_lm_head[g] = _ptr(self.t[f"cp.lm_head.{g}"])
        qw.rope_cos = _ptr(self.cos)
        qw.rope_sin = _ptr(self.sin)
        qw.rope_rows = rope_rows
        self.qw = qw
        d = _lib.QttDims()
        d.hidden, d.intermediate = dims.hidden, dims.intermediate
        d.n_q_heads, d.n_kv_heads, d.head_dim = dims.n_q_heads, dims.n_kv_heads, dims.head_dim
        d.vocab, d.cp_vocab, d.n_groups = dims.vocab, dims.cp_vocab, dims.n_groups
        d.backbone_layers, d.cp_layers = self.nb, self.nc
        d.rms_eps = dims.rms_eps
        d.attn_scale = 1.0 / math.sqrt(dims.head_dim)
        self.qdims = d

    def weight_bytes_per_frame(self) -> int:
        return frame_weight_bytes(self.dims, self.nb, self.nc)


def sampling_struct(do_sample=False, temperature=0.9, top_k=50, top_p=1.0, cp_do_sample=False, cp_temperature=0.9,
                    cp_top_k=50, min_new_tokens=2, repetition_penalty=1.0, eos_token_id=None, seed=0,
                    philox_stream=0, dims: ModelDims = DEFAULT_DIMS) -> _lib.QttSampling:
    s = _lib.QttSampling()
    s.do_sample = int(bool(do_sample))
    s.temperature = float(temperature)
    s.top_k = int(top_k)
    s.top_p = float(top_p)
    s.cp_do_sample = int(bool(cp_do_sample))
    s.cp_temperature = float(cp_temperature)
    s.cp_top_k = int(cp_top_k)
    s.min_new_tokens = int(min_new_tokens)
    s.repetition_penalty = float(repetition_penalty)
    s.eos_token_id = int(dims.eos_token_id if eos_token_id is None else eos_token_id)
    s.philox_stream = int(philox_stream)
    s.seed = int(seed) & 0xFFFFFFFFFFFFFFFF
    return s


class Engine:
    """A qtt_engine: KV caches + device decode state for ``max_streams`` utterances."""

    def __init__(self, model: DeviceModel, max_streams: int = 1, max_seq: int = 4096, max_frames: int = 4096):
        self.lib = _lib.load()
        self.model = model
        self.max_streams, self.max_seq, self.max_frames = max_streams, max_seq, max_frames
        h = ctypes.c_void_p()
        torch.cuda.set_device(model.device)
        _lib.check(self.lib.qtt_engine_create(ctypes.byref(model.qw), ctypes.byref(model.qdims), model.device,
                                              max_streams, max_seq, max_frames, ctypes.byref(h)),
                   "qtt_engine_create")
        self.h = h

    # ---- lifetime --------------------------------------------------------------------------
    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            self.lib.qtt_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def device(self) -> torch.device:
        return torch.device("cuda", self.model.device)

    @property
    def num_ctas(self) -> int:
        return self.lib.qtt_engine_num_ctas(self.h)

    # ---- state -----------------------------------------------------------------------------
    def reset(self, s: int = 0, stream=None):
        _lib.check(self.lib.qtt_reset(self.h, s, _stream_handle(stream)), "qtt_reset")

    def set_kv(self, s: int, k: torch.Tensor, v: torch.Tensor, stream=None):
        assert k.is_cuda and k.shape == v.shape and k.dim() == 4
        dtype = {torch.bfloat16: 0, torch.float32: 1}[k.dtype]
        k, v = k.contiguous(), v.contiguous()
        _lib.check(self.lib.qtt_set_kv(self.h, s, _ptr(k), _ptr(v), k.shape[2], dtype, _stream_handle(stream)),
                   "qtt_set_kv")

    def kv(self, s: int = 0):
        """(k, v) zero-copy views [L, 8, max_seq, 128] bf16 of the stream's caches."""
        kp, vp, ms = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_int()
        _lib.check(self.lib.qtt_get_kv(self.h, s, ctypes.byref(kp), ctypes.byref(vp), ctypes.byref(ms)),
                   "qtt_get_kv")
        shape = (self.model.nb, self.model.dims.n_kv_heads, ms.value, self.model.dims.head_dim)
        k = torch.as_tensor(_DevArray(kp.value, shape, "<f2"), device=f"cuda:{self.model.device}").view(torch.bfloat16)
        v = torch.as_tensor(_DevArray(vp.value, shape, "<f2"), device=f"cuda:{self.model.device}").view(torch.bfloat16)
        return k, v

    def set_position(self, s: int, pos: int, stream=None):
        _lib.check(self.lib.qtt_set_position(self.h, s, pos, _stream_handle(stream)), "qtt_set_position")

    def state(self, s: int = 0, stream=None) -> dict:
        a, b, c, d = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        _lib.check(self.lib.qtt_get_state(self.h, s, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c),
                                          ctypes.byref(d), _stream_handle(stream)), "qtt_get_state")
        return {"position": a.value, "frames": b.value, "g0": c.value, "done": d.value}

    def codes(self, s: int = 0) -> torch.Tensor:
        """Zero-copy int32 view [max_frames, 16] of the stream's code buffer."""
        p = ctypes.POINTER(ctypes.c_int32)()
        _lib.check(self.lib.qtt_codes_ptr(self.h, s, ctypes.byref(p)), "qtt_codes_ptr")
        addr = ctypes.cast(p, ctypes.c_void_p).value
        return torch.as_tensor(_DevArray(addr, (self.max_frames, self.model.dims.n_groups), "<i4"),
                               device=f"cuda:{self.model.device}")

    # ---- compute ---------------------------------------------------------------------------
    def backbone_step(self, s: int, emb: torch.Tensor, position: int, out: torch.Tensor | None = None,
                      stream=None) -> torch.Tensor | None:
        assert emb.is_cuda and emb.dtype == torch.bfloat16 and emb.numel() == self.model.dims.hidden
        emb = emb.contiguous()
        if out is not None:
            assert out.is_cuda and out.dtype == torch.float32 and out.numel() == self.model.dims.hidden
        _lib.check(self.lib.qtt_backbone_step(self.h, s, _ptr(emb), position, _ptr(out) if out is not None else None,
                                              _stream_handle(stream)), "qtt_backbone_step")
        return out

    def cp_step(self, emb: torch.Tensor, position: int, out: torch.Tensor, stream=None) -> torch.Tensor:
        emb = emb.contiguous()
        _lib.check(self.lib.qtt_cp_step(self.h, _ptr(emb), position, _ptr(out), _stream_handle(stream)),
                   "qtt_cp_step")
        return out

    def prefill(self, s: int, embeds: torch.Tensor, sampling: _lib.QttSampling, stream=None):
        assert embeds.is_cuda and embeds.dtype == torch.bfloat16 and embeds.dim() == 2
        embeds = embeds.contiguous()
        self._keep = embeds
        _lib.check(self.lib.qtt_prefill(self.h, s, _ptr(embeds), embeds.shape[0], ctypes.byref(sampling),
                                        _stream_handle(stream)), "qtt_prefill")

    def frames(self, s: int, n: int, trailing: torch.Tensor | None, pad: torch.Tensor,
               sampling: _lib.QttSampling, stream=None):
        nt = 0 if trailing is None else trailing.shape[0]
        tp = _ptr(trailing) if trailing is not None and nt > 0 else None
        _lib.check(self.lib.qtt_frames(self.h, s, n, tp, nt, _ptr(pad), ctypes.byref(sampling),
                                       _stream_handle(stream)), "qtt_frames")

    # ---- batched decode (streams 0..B-1 advance together, tcgen05 GEMMs) ----------------------
    def prefill_tc(self, s: int, embeds: torch.Tensor, sampling: _lib.QttSampling, stream=None):
        """Prefill stream s with the tensor-core path (chunks of up to 128 context positions per
        launch); same results as ``prefill``."""
        embeds = embeds.contiguous()
        assert embeds.is_cuda and embeds.dtype == torch.bfloat16 and embeds.dim() == 2
        self._keep_tc = embeds
        _lib.check(self.lib.qtt_prefill_tc(self.h, s, _ptr(embeds), embeds.shape[0], ctypes.byref(sampling),
                                           _stream_handle(stream)), "qtt_prefill_tc")

    def batch_prefill(self, embeds: list, sampling: _lib.QttSampling, stream=None):
        """Prefill utterances 0..B-1 (``embeds[s]``: bf16 [len_s, 1024] on the engine's GPU) and
        sample each one's first group-0 token."""
        embeds = [e.contiguous() for e in embeds]
        for e in embeds:
            assert e.is_cuda and e.dtype == torch.bfloat16 and e.dim() == 2
        B = len(embeds)
        self._keep_b = embeds
        ptrs = (ctypes.c_void_p * B)(*[_ptr(e) for e in embeds])
        lens = (ctypes.c_int * B)(*[e.shape[0] for e in embeds])
        _lib.check(self.lib.qtt_batch_prefill(self.h, B, ptrs, lens, ctypes.byref(sampling), _stream_handle(stream)),
                   "qtt_batch_prefill")

    def batch_frames(self, n: int, trailing: list, pads: list, sampling: _lib.QttSampling, stream=None):
        """n frames of utterances 0..B-1 (``trailing[s]``: bf16 [T_s, 1024] or None, ``pads[s]``:
        bf16 [1024])."""
        B = len(pads)
        trailing = [None if t is None else t.contiguous() for t in trailing]
        pads = [x.contiguous() for x in pads]
        self._keep_f = (trailing, pads)
        tp = (ctypes.c_void_p * B)(*[None if t is None or t.shape[0] == 0 else _ptr(t) for t in trailing])
        nt = (ctypes.c_int * B)(*[0 if t is None else t.shape[0] for t in trailing])
        pp = (ctypes.c_void_p * B)(*[_ptr(x) for x in pads])
        _lib.check(self.lib.qtt_batch_frames(self.h, B, n, tp, nt, pp, ctypes.byref(sampling), _stream_handle(stream)),
                   "qtt_batch_frames")

    def set_stream_params(self, s: int, philox_stream: int = -1, frame_limit: int = 0):
        """Stream s's own Philox stream (-1: the launch's default) and frame limit (> 0: stop after
        that many frames, 0: max_frames, < 0: parked) for the batched launches that follow."""
        _lib.check(self.lib.qtt_set_stream_params(self.h, s, philox_stream, frame_limit), "qtt_set_stream_params")

    def batch_states(self, B: int, stream=None) -> list:
        """[position, frames, g0, done] of streams 0..B-1 (one device-to-host copy; synchronizes)."""
        out = (ctypes.c_int * (4 * B))()
        _lib.check(self.lib.qtt_batch_states(self.h, B, out, _stream_handle(stream)), "qtt_batch_states")
        return [list(out[4 * s:4 * s + 4]) for s in range(B)]

    def batch_last_codes(self, B: int, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """int32 [B, 16] on the engine's GPU: the codes of each stream's latest frame (-1s if it has
        none), gathered by one kernel on ``stream`` (asynchronous)."""
        if out is None:
            out = torch.empty(B, self.model.dims.n_groups, dtype=torch.int32, device=self.device)
        assert out.is_cuda and out.dtype == torch.int32 and out.is_contiguous() and out.numel() >= 16 * B
        _lib.check(self.lib.qtt_batch_last_codes(self.h, B, _ptr(out), _stream_handle(stream)), "qtt_batch_last_codes")
        return out

    def batch_set_debug_outputs(self, cp_logits: torch.Tensor | None, g0_logits: torch.Tensor | None):
        """Parity tests: batched frames also write each head's logits into cp_logits fp32
        [B, 15, cp_vocab] and g0_logits fp32 [B, vocab]."""
        self._bdbg = (cp_logits, g0_logits)
        _lib.check(self.lib.qtt_batch_set_debug_outputs(
            self.h, None if cp_logits is None else _ptr(cp_logits), None if g0_logits is None else _ptr(g0_logits)),
            "qtt_batch_set_debug_outputs")

    def batch_buffers(self) -> dict:
        """Diagnostic views of the batched path's scratch (GEMM operand planes, sampled logits,
        frame tokens, activations of the last stage that wrote them)."""
        ptrs = (ctypes.c_void_p * 9)()
        _lib.check(self.lib.qtt_batch_debug_buffers(self.h, ptrs, 9), "qtt_batch_debug_buffers")
        dev = f"cuda:{self.model.device}"
        view = lambda i, shape, ts: torch.as_tensor(_DevArray(ptrs[i], shape, ts), device=dev)
        return {"abuf0": view(0, (2, 128, 3072), "<u2").view(torch.bfloat16),
                "abuf1": view(1, (2, 128, 3072), "<u2").view(torch.bfloat16),
                "logits": view(2, (64, 3072), "<f4"), "tok": view(3, (64, 16), "<i4"),
                "x": view(4, (128, 1024), "<f4"), "hb0": view(5, (128, 1024), "<f4"),
                "hb1": view(6, (128, 1024), "<f4"), "hmid": view(7, (128, 1024), "<f4"),
                "qkv": view(8, (128, 4096), "<f4")}

    def set_decode_state(self, s: int, h: torch.Tensor, g0: int, position: int, stream=None):
        """KV handoff: decode from ``position`` with hidden ``h`` (fp32 [1024]) and token g0."""
        h = h.to(torch.float32).contiguous()
        _lib.check(self.lib.qtt_set_decode_state(self.h, s, _ptr(h), int(g0), int(position),
                                                 _stream_handle(stream)), "qtt_set_decode_state")
        torch.cuda.current_stream().synchronize()

    def hidden(self, s: int = 0, stream=None) -> torch.Tensor:
        out = torch.empty(self.model.dims.hidden, dtype=torch.float32, device=f"cuda:{self.model.device}")
        _lib.check(self.lib.qtt_get_hidden(self.h, s, _ptr(out), _stream_handle(stream)), "qtt_get_hidden")
        return out

    def set_debug_outputs(self, cp_logits: torch.Tensor | None, g0_logits: torch.Tensor | None):
        self._dbg = (cp_logits, g0_logits)
        _lib.check(self.lib.qtt_set_debug_outputs(self.h, _ptr(cp_logits) if cp_logits is not None else None,
                                                  _ptr(g0_logits) if g0_logits is not None else None),
                   "qtt_set_debug_outputs")

    def set_debug_timeline(self, stamps: torch.Tensor | None):
        """stamps: int64 cuda tensor; each launch writes %globaltimer at start and after each
        grid barrier into it (profiling). None turns it off."""
        self._timeline = stamps
        n = 0 if stamps is None else stamps.numel()
        _lib.check(self.lib.qtt_set_debug_timeline(self.h, _ptr(stamps) if stamps is not None else None, n),
                   "qtt_set_debug_timeline")

    def check(self, stream=None):
        _lib.check(self.lib.qtt_check(self.h, _stream_handle(stream)), "qtt_check")
