"""Seeded random-init weights with the Qwen3-TTS-12Hz-0.6B shapes.

There is no checkpoint in this environment, so benchmarks and parity tests run on
random-init weights: every linear / embedding / head matrix is bf16 N(0, std) with
std = 0.02, RMSNorm weights are 1.0 (the HF initialisation) unless ``norm_std`` > 0,
in which case they are 1 + N(0, norm_std) (tests use that to catch mixed-up norms).

Each tensor draws from its own ``torch.Generator`` seeded with
``base_seed * 1_000_003 + index`` (index = position in :func:`tensor_specs`), so the
tensors can be generated in parallel threads and any subset reproduces exactly.
Backbone tensors (layers, final norm, codec_embedding, codec_head) use ``seed_backbone``
(0); code-predictor tensors use ``seed_cp`` (1).

Names follow the module paths of the reference's model object
(``talker.model.layers[i].self_attn.q_proj`` etc., generator.py:55-65):

* ``talker.layers.{i}.{tensor}`` for tensor in :data:`LAYER_TENSORS`
* ``talker.norm``, ``talker.codec_embedding`` [vocab, hidden], ``talker.codec_head`` [vocab, hidden]
* ``cp.layers.{i}.{tensor}``, ``cp.norm``
* ``cp.codec_embedding.{g}`` / ``cp.lm_head.{g}`` for g in 0..14, each [cp_vocab, hidden]
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import torch

from .config import DEFAULT_DIMS, LAYER_TENSORS, ModelDims


def _layer_shapes(d: ModelDims) -> dict:
    h, i = d.hidden, d.intermediate
    return {
        "input_layernorm": (h,),
        "q_proj": (d.q_size, h),
        "k_proj": (d.kv_size, h),
        "v_proj": (d.kv_size, h),
        "q_norm": (d.head_dim,),
        "k_norm": (d.head_dim,),
        "o_proj": (h, d.q_size),
        "post_attention_layernorm": (h,),
        "gate_proj": (i, h),
        "up_proj": (i, h),
        "down_proj": (h, i),
    }


def tensor_specs(d: ModelDims = DEFAULT_DIMS, backbone_layers: int | None = None,
                 cp_layers: int | None = None) -> list:
    """Ordered list of (name, shape, is_norm, part) with part in {"backbone", "cp"}."""
    nb = d.backbone_layers if backbone_layers is None else backbone_layers
    nc = d.cp_layers if cp_layers is None else cp_layers
    shapes = _layer_shapes(d)
    specs = []
    for li in range(nb):
        for t in LAYER_TENSORS:
            specs.append((f"talker.layers.{li}.{t}", shapes[t], len(shapes[t]) == 1, "backbone"))
    specs.append(("talker.norm", (d.hidden,), True, "backbone"))
    specs.append(("talker.codec_embedding", (d.vocab, d.hidden), False, "backbone"))
    specs.append(("talker.codec_head", (d.vocab, d.hidden), False, "backbone"))
    for li in range(nc):
        for t in LAYER_TENSORS:
            specs.append((f"cp.layers.{li}.{t}", shapes[t], len(shapes[t]) == 1, "cp"))
    specs.append(("cp.norm", (d.hidden,), True, "cp"))
    for g in range(d.n_groups - 1):
        specs.append((f"cp.codec_embedding.{g}", (d.cp_vocab, d.hidden), False, "cp"))
    for g in range(d.n_groups - 1):
        specs.append((f"cp.lm_head.{g}", (d.cp_vocab, d.hidden), False, "cp"))
    return specs


def _one(index: int, shape, is_norm: bool, seed: int, std: float, norm_std: float):
    g = torch.Generator().manual_seed(seed * 1_000_003 + index)
    if is_norm:
        if norm_std <= 0.0:
            return torch.ones(shape, dtype=torch.bfloat16)
        return (1.0 + norm_std * torch.randn(shape, generator=g)).to(torch.bfloat16)
    return (std * torch.randn(shape, generator=g)).to(torch.bfloat16)


def synthetic_weights(dims: ModelDims = DEFAULT_DIMS, backbone_layers: int | None = None,
                      cp_layers: int | None = None, seed_backbone: int = 0, seed_cp: int = 1,
                      std: float = 0.02, norm_std: float = 0.0, threads: int | None = None) -> dict:
    """Return {name: CPU bf16 tensor} for the whole model (see module docstring)."""
    specs = tensor_specs(dims, backbone_layers, cp_layers)
    threads = threads or min(32, os.cpu_count() or 1)

    def job(arg):
        idx, (name, shape, is_norm, part) = arg
        seed = seed_backbone if part == "backbone" else seed_cp
        return name, _one(idx, shape, is_norm, seed, std, norm_std)

    with ThreadPoolExecutor(max_workers=threads) as ex:
        out = dict(ex.map(job, enumerate(specs)))
    return out


def layer_list(weights: dict, prefix: str, n_layers: int) -> list:
    """Flat list of 11 tensors per layer in the reference struct order
    (megakernel_backbone.py:371-387)."""
    flat = []
    for li in range(n_layers):
        for t in LAYER_TENSORS:
            flat.append(weights[f"{prefix}.layers.{li}.{t}"])
    return flat


def rope_tables(max_seq_len: int, head_dim: int = 128, theta: float = 1e6):
    """bf16 cos/sin tables [max_seq_len, head_dim] with the frequencies repeated over both
    halves, built exactly as the reference does (megakernel_backbone.py:389-398,
    megakernel_code_predictor.py:294-308): fp32 inv_freq, fp32 outer product, fp32 cos/sin,
    then a bf16 cast. With all three mRoPE position ids equal (decode, generator.py:213,230)
    the multimodal rotation reduces to these 1D tables."""
    half = head_dim // 2
    inv_freq = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float32) / half))
    pos = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return torch.cos(emb).to(torch.bfloat16).contiguous(), torch.sin(emb).to(torch.bfloat16).contiguous()
