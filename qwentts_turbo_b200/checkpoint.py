"""Weight extraction from a loaded Qwen3-TTS model object.

Follows the attribute paths the reference reads (generator.py:55-68,
megakernel_backbone.py:358-387, megakernel_code_predictor.py:271-292):
``model.talker.model.layers[i].{input_layernorm, self_attn.{q,k,v,o}_proj, self_attn.{q,k}_norm,
post_attention_layernorm, mlp.{gate,up,down}_proj}``, ``model.talker.model.norm``,
``model.talker.model.codec_embedding``, ``model.talker.codec_head``,
``model.talker.code_predictor.model.{layers, norm, codec_embedding[g]}``,
``model.talker.code_predictor.lm_head[g]``.
"""
from __future__ import annotations

from .config import LAYER_TENSORS

_LAYER_ATTR = {
    "input_layernorm": ("input_layernorm",),
    "q_proj": ("self_attn", "q_proj"),
    "k_proj": ("self_attn", "k_proj"),
    "v_proj": ("self_attn", "v_proj"),
    "q_norm": ("self_attn", "q_norm"),
    "k_norm": ("self_attn", "k_norm"),
    "o_proj": ("self_attn", "o_proj"),
    "post_attention_layernorm": ("post_attention_layernorm",),
    "gate_proj": ("mlp", "gate_proj"),
    "up_proj": ("mlp", "up_proj"),
    "down_proj": ("mlp", "down_proj"),
}


def _get(obj, path):
    for p in path:
        obj = getattr(obj, p)
    return obj.weight.data


def load_qwen_tts(model_path):
    """Load the checkpoint through qwen_tts (the reference's loader, generator.py:50-53)."""
    try:
        from qwen_tts.inference.qwen3_tts_model import Qwen3TTSModel
    except ImportError as e:  # pragma: no cover - depends on the environment
        raise ImportError("loading a checkpoint needs the qwen_tts package; pass `weights=` "
                          "(e.g. qwentts_turbo_b200.weights.synthetic_weights()) instead") from e
    tts = Qwen3TTSModel.from_pretrained(model_path, dtype="bfloat16", device_map="cuda")
    return tts.model


def weights_from_model(model) -> dict:
    talker = model.talker
    bb = talker.model
    cp = talker.code_predictor
    out = {}
    for i, layer in enumerate(bb.layers):
        for t in LAYER_TENSORS:
            out[f"talker.layers.{i}.{t}"] = _get(layer, _LAYER_ATTR[t])
    out["talker.norm"] = bb.norm.weight.data
    out["talker.codec_embedding"] = bb.codec_embedding.weight.data
    out["talker.codec_head"] = talker.codec_head.weight.data
    for i, layer in enumerate(cp.model.layers):
        for t in LAYER_TENSORS:
            out[f"cp.layers.{i}.{t}"] = _get(layer, _LAYER_ATTR[t])
    out["cp.norm"] = cp.model.norm.weight.data
    for g, emb in enumerate(cp.model.codec_embedding):
        out[f"cp.codec_embedding.{g}"] = emb.weight.data
    for g, head in enumerate(cp.lm_head):
        out[f"cp.lm_head.{g}"] = head.weight.data
    return out


def eos_from_model(model, default: int) -> int:
    try:
        return int(model.config.talker_config.codec_eos_token_id)
    except AttributeError:
        return default
