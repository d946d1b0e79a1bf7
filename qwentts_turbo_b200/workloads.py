"""Seeded synthetic inputs for the benchmark configurations (no datasets or checkpoints exist
in this environment). All tensors are generated on the CPU with torch.Generator so that the
GPU engine and the CPU oracle see identical values.

* C1: backbone step, 256-position KV cache N(0,1) bf16 + one N(0,1) embedding (seed 2).
* C2: code-predictor chain from an N(0,1) backbone hidden and a group-0 token (seed 3).
* C3: frame loop, 200-token N(0,1) prefill context, 64 trailing-text rows, pad row (seed 4).
* C4/C5: per-utterance contexts drawn uniformly from [100, 400] / [100, 600] (seed 4 / 5);
  ``c4_inputs`` generates a whole C4 batch (the bench's and the full-size parity test's inputs).
"""
from __future__ import annotations

import torch

from .config import DEFAULT_DIMS


def c1_inputs(n_layers: int = DEFAULT_DIMS.backbone_layers, ctx: int = 256, seed: int = 2):
    g = torch.Generator().manual_seed(seed)
    d = DEFAULT_DIMS
    k = torch.randn(n_layers, d.n_kv_heads, ctx, d.head_dim, generator=g).to(torch.bfloat16)
    v = torch.randn(n_layers, d.n_kv_heads, ctx, d.head_dim, generator=g).to(torch.bfloat16)
    emb = torch.randn(d.hidden, generator=g).to(torch.bfloat16)
    return k, v, emb


def c2_inputs(seed: int = 3):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(DEFAULT_DIMS.hidden, generator=g).to(torch.bfloat16)
    g0 = int(torch.randint(0, DEFAULT_DIMS.vocab - 1024, (1,), generator=g))
    return h, g0


def c3_inputs(ctx: int = 200, n_trailing: int = 64, seed: int = 4):
    g = torch.Generator().manual_seed(seed)
    d = DEFAULT_DIMS.hidden
    embeds = torch.randn(ctx, d, generator=g).to(torch.bfloat16)
    trailing = torch.randn(n_trailing, d, generator=g).to(torch.bfloat16)
    pad = torch.randn(d, generator=g).to(torch.bfloat16)
    return embeds, trailing, pad


def batch_contexts(n: int, lo: int, hi: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (n,), generator=g)]


def c4_inputs(B: int = 64, lo: int = 100, hi: int = 400, n_trailing: int = 64, seed: int = 4):
    """C4: B utterances with contexts ~ U[lo, hi] of N(0,1) embeddings, n_trailing trailing-text
    rows and a pad row each (bf16, CPU). Returns (contexts, embeds, trailing, pads)."""
    g = torch.Generator().manual_seed(seed)
    d = DEFAULT_DIMS.hidden
    ctx = torch.randint(lo, hi + 1, (B,), generator=g).tolist()
    embeds = [torch.randn(L, d, generator=g).to(torch.bfloat16) for L in ctx]
    trailing = [torch.randn(n_trailing, d, generator=g).to(torch.bfloat16) for _ in range(B)]
    pads = [torch.randn(d, generator=g).to(torch.bfloat16) for _ in range(B)]
    return ctx, embeds, trailing, pads
