"""ctypes binding of libqtt.so (include/qtt.h).

The shared library is built in-tree by ``qwentts_turbo_b200.build.build_library()`` (or
``__graft_entry__.build()``). There is no fallback: if the library is missing or fails to
load, every GPU entry point raises :class:`QTTError`.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqtt.so")

# qtt_status (include/qtt.h)
STATUS = {
    0: "ok",
    1: "invalid argument",
    2: "CUDA error",
    3: "out of device memory",
    4: "device wait timed out",
    5: "unsupported shape or option",
    6: "token id out of range",
    7: "position beyond the KV cache",
    8: "device error",
}
QTT_OK = 0
QTT_ERR_INVALID_ARG = 1
QTT_ERR_TIMEOUT = 4
QTT_ERR_UNSUPPORTED = 5


class QTTError(RuntimeError):
    def __init__(self, status: int, where: str):
        super().__init__(f"{where}: {STATUS.get(status, 'unknown status')} (qtt_status={status})")
        self.status = status


class TTSLayerWeights(ctypes.Structure):
    """Same layout as the reference's TTSLayerWeights (fused_decode_tts.cu:22-34)."""
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "input_layernorm_weight", "q_proj_weight", "k_proj_weight", "v_proj_weight",
        "q_norm_weight", "k_norm_weight", "o_proj_weight", "post_attn_layernorm_weight",
        "gate_proj_weight", "up_proj_weight", "down_proj_weight")]


class QttDims(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("intermediate", ctypes.c_int), ("n_q_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("vocab", ctypes.c_int),
                ("cp_vocab", ctypes.c_int), ("n_groups", ctypes.c_int), ("backbone_layers", ctypes.c_int),
                ("cp_layers", ctypes.c_int), ("rms_eps", ctypes.c_float), ("attn_scale", ctypes.c_float)]


class QttWeights(ctypes.Structure):
    _fields_ = [("backbone_layers", ctypes.POINTER(TTSLayerWeights)), ("backbone_norm", ctypes.c_void_p),
                ("codec_embedding", ctypes.c_void_p), ("codec_head", ctypes.c_void_p),
                ("cp_layers", ctypes.POINTER(TTSLayerWeights)), ("cp_norm", ctypes.c_void_p),
                ("cp_codec_embedding", ctypes.c_void_p * 15), ("cp_lm_head", ctypes.c_void_p * 15),
                ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p), ("rope_rows", ctypes.c_int)]


class QttSampling(ctypes.Structure):
    _fields_ = [("do_sample", ctypes.c_int), ("temperature", ctypes.c_float), ("top_k", ctypes.c_int),
                ("top_p", ctypes.c_float), ("cp_do_sample", ctypes.c_int), ("cp_temperature", ctypes.c_float),
                ("cp_top_k", ctypes.c_int), ("min_new_tokens", ctypes.c_int),
                ("repetition_penalty", ctypes.c_float), ("eos_token_id", ctypes.c_int),
                ("philox_stream", ctypes.c_int), ("seed", ctypes.c_uint64)]


# name -> (restype, argtypes)
_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_LAUNCH_ARGS = [_P, ctypes.POINTER(TTSLayerWeights), _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                _I, _I, _I, _I, _F, _P]
SIGNATURES = {
    "launch_tts_decode_with_embedding": (None, _LAUNCH_ARGS),
    "launch_tts_decode": (None, [_I] + _LAUNCH_ARGS),
    "launch_cp_decode_with_embedding": (None, _LAUNCH_ARGS),
    "qtt_last_launch_status": (_I, []),
    "qtt_build_id": (ctypes.c_char_p, []),
    "qtt_stream_check": (_I, [_P]),
    "qtt_status_string": (ctypes.c_char_p, [_I]),
    "qtt_engine_create": (_I, [ctypes.POINTER(QttWeights), ctypes.POINTER(QttDims), _I, _I, _I, _I,
                               ctypes.POINTER(_P)]),
    "qtt_engine_destroy": (_I, [_P]),
    "qtt_engine_num_ctas": (_I, [_P]),
    "qtt_reset": (_I, [_P, _I, _P]),
    "qtt_set_kv": (_I, [_P, _I, _P, _P, _I, _I, _P]),
    "qtt_get_kv": (_I, [_P, _I, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_I)]),
    "qtt_set_position": (_I, [_P, _I, _I, _P]),
    "qtt_get_state": (_I, [_P, _I, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I),
                           ctypes.POINTER(_I), _P]),
    "qtt_backbone_step": (_I, [_P, _I, _P, _I, _P, _P]),
    "qtt_prefill": (_I, [_P, _I, _P, _I, ctypes.POINTER(QttSampling), _P]),
    "qtt_frames": (_I, [_P, _I, _I, _P, _I, _P, ctypes.POINTER(QttSampling), _P]),
    "qtt_codes_ptr": (_I, [_P, _I, ctypes.POINTER(ctypes.POINTER(ctypes.c_int32))]),
    "qtt_cp_step": (_I, [_P, _P, _I, _P, _P]),
    "qtt_set_debug_outputs": (_I, [_P, _P, _P]),
    "qtt_set_decode_state": (_I, [_P, _I, _P, _I, _I, _P]),
    "qtt_set_debug_timeline": (_I, [_P, _P, _I]),
    "qtt_set_debug_profile": (_I, [_P, _P, _I, _P, _I, _I]),
    "qtt_get_hidden": (_I, [_P, _I, _P, _P]),
    "qtt_check": (_I, [_P, _P]),
    "qtt_set_refill_policy": (_I, [_P, _I]),
    "qtt_set_debug_barrier_fault": (_I, [_P, _I, ctypes.c_uint64]),
    "qtt_set_debug_kv_in_attention": (_I, [_P, _I]),
    "qtt_batch_prefill": (_I, [_P, _I, ctypes.POINTER(_P), ctypes.POINTER(_I), ctypes.POINTER(QttSampling), _P]),
    "qtt_prefill_tc": (_I, [_P, _I, _P, _I, ctypes.POINTER(QttSampling), _P]),
    "qtt_set_stream_params": (_I, [_P, _I, _I, _I]),
    "qtt_batch_states": (_I, [_P, _I, ctypes.POINTER(_I), _P]),
    "qtt_batch_frames": (_I, [_P, _I, _I, ctypes.POINTER(_P), ctypes.POINTER(_I), ctypes.POINTER(_P),
                              ctypes.POINTER(QttSampling), _P]),
    "qtt_batch_last_codes": (_I, [_P, _I, _P, _P]),
    "qtt_batch_debug_buffers": (_I, [_P, ctypes.POINTER(_P), _I]),
    "qtt_batch_set_debug_outputs": (_I, [_P, _P, _P]),
    "qtt_backbone_step_noalloc": (_I, [_P, ctypes.POINTER(TTSLayerWeights), _P, _P, _P, _P, _P, _P, _P,
                                       _I, _I, _I, _F, _P]),
}

_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libqtt.so once and declare every entry point. Raises QTTError when absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise QTTError(2, f"libqtt.so not found at {path}; build it with "
                          "`python -c 'import qwentts_turbo_b200.build as b; b.build_library()'`")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, where: str):
    if status != QTT_OK:
        raise QTTError(status, where)
