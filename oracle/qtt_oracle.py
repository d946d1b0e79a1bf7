"""CPU oracle for the Qwen3-TTS per-frame decode path.

TEST INFRASTRUCTURE ONLY. This module is imported by ``tests/``, by
``__graft_entry__.smoke()`` (as the checker) and by ``bench.py`` (its ``cpu_baseline`` leg
and the ``--impl reference`` arm). The product path (``qwentts_turbo_b200``) never imports
it and has no CPU fallback.

It restates, in fp32 PyTorch on the CPU, the math of the reference's decode path with
the reference's rounding points (paths relative to the hamza1brh/qwenTTS-turbo tree):

* decoder layer: ``qwentts_turbo/csrc/fused_decode_tts.cu:56-547`` (backbone) and
  ``qwentts_turbo/csrc/fused_decode_code_predictor.cu:64-559`` (code predictor)
* frame loop, sampler, CP chain, combine: ``qwentts_turbo/generator.py:77-207,309-362``
* RoPE tables: ``qwentts_turbo/megakernel_backbone.py:389-398``; mRoPE interleave rule:
  ``qwentts_turbo/csrc/rope_multimodal.cuh:26-54``

Rounding points kept from the reference:
* backbone hidden state is bf16 between layers (fused_decode_tts.cu:541); inside a layer the
  residual stream is fp32 (fused_decode_tts.cu:84-85,434,449);
* backbone K/V are stored to the cache as bf16 (fused_decode_tts.cu:271-272) and the
  attention reads the rounded values, including the row written in the same step;
* code-predictor hidden state and K/V cache are fp32 (fused_decode_code_predictor.cu:553,287-289);
* head logits are bf16: ``torch.mv`` of a bf16 matrix with the bf16-cast hidden
  (generator.py:158,351);
* the 16-embedding combine is a chain of bf16 adds (generator.py:356-362), then one more
  bf16 add of the trailing-text row or the pad embedding (generator.py:146-149).

Deliberate definitions where the reference has none on device:
* sampling draws come from Philox4x32-10 (Salmon et al., SC'11) keyed by the stream seed,
  counter (frame, group, stream, 0); the categorical draw is an inverse CDF over the
  bf16 probabilities in vocabulary order, accumulated in exact 2^-60 fixed point, so the
  pick does not depend on summation order;
* the 2-token code-predictor prefill (generator.py:319-325) is computed with the same
  fp32 layer math as the following decode steps;
* the backbone prefill is the same layer math run causally over the context.

Parity is pinned by ``tests/test_oracle_pins.py``: against transformers' ``Qwen3Model``
(the PyTorch forward the reference's talker/code-predictor are built from) and, when
present, against golden outputs of the reference's own CUDA kernels
(``tests/golden/ref_megakernel_golden.npz``, generated on a B200 by
``tests/golden/make_ref_golden.py``).
"""
from __future__ import annotations

import math

import numpy as np
import torch

HEAD_DIM = 128


def bf16r(x: torch.Tensor) -> torch.Tensor:
    """Round to bf16 (round-to-nearest-even) and back to the input's dtype (fp32 or fp64)."""
    return x.to(torch.bfloat16).to(x.dtype)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * w over the last dim (fused_decode_tts.cu:74-109)."""
    rstd = torch.rsqrt((x * x).mean(-1, keepdim=True) + eps)
    return x * rstd * w


def rope_rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """out[i<64] = x_i c_i - x_{i+64} s_i ; out[i>=64] = x_i c_i + x_{i-64} s_i
    (fused_decode_tts.cu:205-216; the rotate_half form in fused_decode_code_predictor.cu:218-239
    is the same rotation)."""
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos + rot * sin


def mrope_angles(t: int, h: int, w: int, inv_freq: torch.Tensor, sections=(24, 20, 20)) -> torch.Tensor:
    """Rotation angles [head_dim] of interleaved multimodal RoPE for position ids (t, h, w).

    Frequency j in [0, 64) takes the height position when j % 3 == 1 and j < 3*sections[1],
    the width position when j % 3 == 2 and j < 3*sections[2], else the temporal position
    (rope_multimodal.cuh:41-54: T/H/W interleaved, sections [24, 20, 20] = 24 T, 20 H, 20 W
    frequencies). The angles repeat over both halves of the head."""
    half = inv_freq.shape[0]
    pos = torch.full((half,), float(t))
    j = torch.arange(half)
    pos[(j % 3 == 1) & (j < 3 * sections[1])] = float(h)
    pos[(j % 3 == 2) & (j < 3 * sections[2])] = float(w)
    ang = pos * inv_freq
    return torch.cat((ang, ang))


def mrope_cos_sin(t: int, h: int, w: int, theta: float = 1e6, head_dim: int = HEAD_DIM,
                  sections=(24, 20, 20)):
    """bf16-rounded cos/sin rows for one (t, h, w) position; equals the 1D table row when
    t == h == w (the decode case, generator.py:213,230)."""
    half = head_dim // 2
    inv_freq = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float32) / half))
    ang = mrope_angles(t, h, w, inv_freq, sections)
    return bf16r(torch.cos(ang)), bf16r(torch.sin(ang))


# ----------------------------------------------------------------------------------------
# Philox4x32-10 and the inverse-CDF draw
# ----------------------------------------------------------------------------------------
_PHILOX_M0, _PHILOX_M1 = 0xD2511F53, 0xCD9E8D57
_PHILOX_W0, _PHILOX_W1 = 0x9E3779B9, 0xBB67AE85
_M32 = 0xFFFFFFFF


def philox4x32_10(counter, key):
    """Philox4x32 with 10 rounds (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as
    easy as 1, 2, 3", SC'11). counter: 4 uint32, key: 2 uint32. Returns 4 uint32."""
    c0, c1, c2, c3 = (int(v) & _M32 for v in counter)
    k0, k1 = (int(v) & _M32 for v in key)
    for r in range(10):
        p0 = _PHILOX_M0 * c0
        p1 = _PHILOX_M1 * c2
        hi0, lo0 = p0 >> 32, p0 & _M32
        hi1, lo1 = p1 >> 32, p1 & _M32
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & _M32, lo1, (hi0 ^ c3 ^ k1) & _M32, lo0
        if r != 9:
            k0 = (k0 + _PHILOX_W0) & _M32
            k1 = (k1 + _PHILOX_W1) & _M32
    return c0, c1, c2, c3


def draw_u24(seed: int, frame: int, group: int, stream: int) -> int:
    """24-bit uniform integer for token (frame, group) of a stream: the top 24 bits of the
    first Philox output word. frame 0 / group 0 is the token sampled from the prefill."""
    x0 = philox4x32_10((frame, group, stream, 0), (seed & _M32, (seed >> 32) & _M32))[0]
    return x0 >> 8


FIX_SHIFT = 60


def inverse_cdf_pick(probs_bf16: torch.Tensor, u24: int) -> int:
    """First index i with cum[i] > floor(u24 * total / 2^24), where cum is the prefix sum of
    floor(p * 2^60) in index order (exact integer arithmetic, order independent)."""
    p = probs_bf16.to(torch.float64).numpy()
    fixed = np.floor(np.ldexp(p, FIX_SHIFT)).astype(np.uint64)
    cum = np.cumsum(fixed, dtype=np.uint64)
    total = int(cum[-1])
    target = (u24 * total) >> 24
    idx = int(np.searchsorted(cum, np.uint64(target), side="right"))
    return min(idx, probs_bf16.shape[0] - 1)


def argmax_first(x: torch.Tensor) -> int:
    """Index of the first maximum (torch.argmax semantics, generator.py:187)."""
    m = x.max()
    return int(torch.nonzero(x == m)[0, 0])


def filter_logits(logits: torch.Tensor, temperature: float, top_k: int, top_p: float = 1.0) -> torch.Tensor:
    """generator.py:188-203: scaled = bf16(l / T), top-k keeps values >= the k-th (ties kept), and
    top-p (nucleus) on the bf16 tensors the reference uses: the values sorted descending (ties in
    index order), probs = bf16(softmax), cum = bf16(fp32 running sum), and entry i of the sorted
    order removed when cum[i - 1] > bf16(top_p) (torch compares a bf16 tensor with a Python float in
    bf16). Returns the filtered scaled logits (-inf = removed), fp32."""
    scaled = bf16r(logits.to(torch.float32) / temperature)
    if top_k > 0:
        k = min(top_k, scaled.shape[-1])
        thr = torch.topk(scaled, k)[0][-1]
        scaled[scaled < thr] = float("-inf")
    if top_p < 1.0:
        sorted_logits, sorted_idx = torch.sort(scaled, descending=True, stable=True)
        e = torch.exp(sorted_logits - sorted_logits[0])
        probs = bf16r(e / e.sum())
        cum = bf16r(torch.cumsum(probs, dim=-1))
        remove = cum > bf16r(torch.tensor(float(top_p)))
        remove[1:] = remove[:-1].clone()
        remove[0] = False
        sorted_logits[remove] = float("-inf")
        scaled = scaled.scatter(0, sorted_idx, sorted_logits)
    return scaled


def sample_token(logits: torch.Tensor, do_sample: bool, temperature: float, top_k: int,
                 top_p: float = 1.0, suppress_eos_id=None, u24: int | None = None) -> int:
    """generator.py:178-207 with the multinomial draw replaced by :func:`inverse_cdf_pick`.
    ``logits`` holds bf16 values (fp32 dtype). Intermediate tensors are bf16 as in the
    reference: scaled = bf16(l / T), probs = bf16(softmax), all with fp32 arithmetic (torch's
    opmath for bf16 tensors) whatever the oracle's compute dtype."""
    logits = logits.to(torch.float32).clone()
    if suppress_eos_id is not None:
        logits[suppress_eos_id] = float("-inf")
    if not do_sample:
        return argmax_first(logits)
    scaled = filter_logits(logits, temperature, top_k, top_p)
    mx = scaled.max()
    e = torch.exp(scaled - mx)
    probs = bf16r(e / e.sum())
    assert u24 is not None, "sampling needs a uniform draw"
    return inverse_cdf_pick(probs, u24)


def apply_repetition_penalty(logits: torch.Tensor, history, penalty: float) -> torch.Tensor:
    """generator.py:161-167: s > 0 ? s / p : s * p on the history's tokens, bf16 result."""
    if penalty == 1.0 or not history:
        return logits
    out = logits.to(torch.float32).clone()
    idx = torch.tensor(sorted(set(int(t) for t in history)), dtype=torch.long)
    s = out[idx]
    out[idx] = bf16r(torch.where(s > 0, s / penalty, s * penalty))
    return out


# ----------------------------------------------------------------------------------------
# Model
# ----------------------------------------------------------------------------------------
class _Stack:
    """fp32 (or fp64) copies of one decoder stack (backbone or code predictor)."""

    def __init__(self, weights: dict, prefix: str, n_layers: int, dtype=torch.float32):
        from qwentts_turbo_b200.config import LAYER_TENSORS
        self.layers = []
        for li in range(n_layers):
            self.layers.append({t: weights[f"{prefix}.layers.{li}.{t}"].to(dtype).contiguous()
                                for t in LAYER_TENSORS})
        self.norm = weights[f"{prefix}.norm"].to(dtype)


class Qwen3TTSOracle:
    """fp32 CPU restatement of the backbone + code-predictor decode (see module docstring)."""

    def __init__(self, weights: dict, dims=None, backbone_layers: int | None = None,
                 cp_layers: int | None = None, max_seq: int = 4096, cp_max_seq: int = 32,
                 exact_rope: bool = False, dtype=torch.float32):
        from qwentts_turbo_b200.config import DEFAULT_DIMS
        from qwentts_turbo_b200.weights import rope_tables
        d = dims or DEFAULT_DIMS
        self.d = d
        self.nb = d.backbone_layers if backbone_layers is None else backbone_layers
        self.nc = d.cp_layers if cp_layers is None else cp_layers
        self.max_seq = max_seq
        self.cp_max_seq = cp_max_seq
        self.dt = dtype
        self.bb = _Stack(weights, "talker", self.nb, dtype)
        self.cp = _Stack(weights, "cp", self.nc, dtype)
        self.codec_embedding = weights["talker.codec_embedding"].to(dtype)
        self.codec_head = weights["talker.codec_head"].to(dtype)
        self.cp_embed = [weights[f"cp.codec_embedding.{g}"].to(dtype) for g in range(d.n_groups - 1)]
        self.cp_head = [weights[f"cp.lm_head.{g}"].to(dtype) for g in range(d.n_groups - 1)]
        rows = max(max_seq, cp_max_seq)
        if exact_rope:
            # fp32 tables without the bf16 cast (HF Qwen3RotaryEmbedding), for pinning the layer
            # math against transformers.
            half = d.head_dim // 2
            inv = 1.0 / (d.rope_theta ** (torch.arange(0, half, dtype=torch.float32) / half))
            emb = torch.outer(torch.arange(rows, dtype=torch.float32), inv)
            emb = torch.cat((emb, emb), dim=-1)
            self.cos, self.sin = torch.cos(emb).to(dtype), torch.sin(emb).to(dtype)
        else:
            cos, sin = rope_tables(rows, d.head_dim, d.rope_theta)
            self.cos, self.sin = cos.to(dtype), sin.to(dtype)
        self.scale = 1.0 / math.sqrt(d.head_dim)
        self.reset_backbone()
        self.reset_cp()

    # ---- state -------------------------------------------------------------------------
    def reset_backbone(self):
        d = self.d
        self.bk = torch.zeros(self.nb, d.n_kv_heads, self.max_seq, d.head_dim, dtype=self.dt)
        self.bv = torch.zeros_like(self.bk)
        self.position = 0

    def reset_cp(self):
        d = self.d
        self.ck = torch.zeros(self.nc, d.n_kv_heads, self.cp_max_seq, d.head_dim, dtype=self.dt)
        self.cv = torch.zeros_like(self.ck)
        self.cp_position = 0

    def set_kv_cache(self, k: torch.Tensor, v: torch.Tensor):
        """megakernel_backbone.py:285-294: copy [L, n_kv, len, hd] into the cache (bf16)."""
        n = k.shape[2]
        self.bk[:, :, :n] = bf16r(k.to(self.dt))
        self.bv[:, :, :n] = bf16r(v.to(self.dt))

    # ---- layer -------------------------------------------------------------------------
    def _layer(self, x, W, kc, vc, positions, kv_bf16: bool, out_bf16: bool):
        d = self.d
        T = x.shape[0]
        res = x
        n = rms_norm(x, W["input_layernorm"], d.rms_eps)
        q = (n @ W["q_proj"].T).view(T, d.n_q_heads, d.head_dim)
        k = (n @ W["k_proj"].T).view(T, d.n_kv_heads, d.head_dim)
        v = (n @ W["v_proj"].T).view(T, d.n_kv_heads, d.head_dim)
        q = rms_norm(q, W["q_norm"], d.rms_eps)
        k = rms_norm(k, W["k_norm"], d.rms_eps)
        pos = torch.tensor(positions, dtype=torch.long)
        c = self.cos[pos][:, None, :]
        s = self.sin[pos][:, None, :]
        q = rope_rotate(q, c, s)
        k = rope_rotate(k, c, s)
        if kv_bf16:
            k, v = bf16r(k), bf16r(v)
        kc[:, pos] = k.transpose(0, 1)
        vc[:, pos] = v.transpose(0, 1)
        S = int(pos.max()) + 1
        group = d.n_q_heads // d.n_kv_heads
        K = kc[:, :S].repeat_interleave(group, dim=0)      # [nq, S, hd]
        V = vc[:, :S].repeat_interleave(group, dim=0)
        scores = torch.einsum("thd,hsd->hts", q, K) * self.scale      # [nq, T, S]
        mask = torch.arange(S)[None, :] > pos[:, None]                  # [T, S]
        scores = scores.masked_fill(mask[None], float("-inf"))
        p = torch.softmax(scores, dim=-1)
        attn = torch.einsum("hts,hsd->thd", p, V).reshape(T, d.q_size)
        o = attn @ W["o_proj"].T + res
        n2 = rms_norm(o, W["post_attention_layernorm"], d.rms_eps)
        m = torch.nn.functional.silu(n2 @ W["gate_proj"].T) * (n2 @ W["up_proj"].T)
        h = m @ W["down_proj"].T + o
        return bf16r(h) if out_bf16 else h

    # ---- backbone ----------------------------------------------------------------------
    def backbone_forward(self, x_bf16: torch.Tensor, positions) -> torch.Tensor:
        """Run tokens x [T, hidden] (bf16 values) at consecutive positions through the
        backbone; returns the final-RMSNorm fp32 hidden of every token [T, hidden]
        (fused_decode_tts.cu:728-831 for T = 1)."""
        h = bf16r(x_bf16.to(self.dt))
        for li, W in enumerate(self.bb.layers):
            h = self._layer(h, W, self.bk[li], self.bv[li], positions, kv_bf16=True, out_bf16=True)
        return rms_norm(h, self.bb.norm, self.d.rms_eps)

    def backbone_step(self, x_bf16: torch.Tensor) -> torch.Tensor:
        """decode_step_with_embedding (megakernel_backbone.py:230-267): one token at
        ``self.position``, then position += 1. Returns fp32 [hidden]."""
        out = self.backbone_forward(x_bf16.reshape(1, -1), [self.position])[0]
        self.position += 1
        return out

    def prefill(self, embeds_bf16: torch.Tensor) -> torch.Tensor:
        """Causal forward over the context [L, hidden] from position 0; returns the last
        token's normed hidden (generator.py:209-225 with the kernel's rounding points)."""
        self.reset_backbone()
        L = embeds_bf16.shape[0]
        out = self.backbone_forward(embeds_bf16, list(range(L)))
        self.position = L
        return out[-1]

    # ---- code predictor ----------------------------------------------------------------
    def cp_forward(self, x_bf16: torch.Tensor, positions) -> torch.Tensor:
        """Code-predictor layers on tokens [T, hidden] (bf16 inputs, fp32 hidden and KV,
        fused_decode_code_predictor.cu:565-668); returns final-normed fp32 [T, hidden]."""
        h = bf16r(x_bf16.to(self.dt))
        for li, W in enumerate(self.cp.layers):
            h = self._layer(h, W, self.ck[li], self.cv[li], positions, kv_bf16=False, out_bf16=False)
        return rms_norm(h, self.cp.norm, self.d.rms_eps)

    @staticmethod
    def head_logits(W: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
        """bf16(W @ bf16(h)) (generator.py:158,331,351)."""
        return bf16r(W @ bf16r(h.to(W.dtype)))

    def cp_chain(self, h_backbone: torch.Tensor, g0: int, do_sample=False, temperature=0.9,
                 top_k=50, seed=0, frame=0, stream=0, forced=None):
        """generator.py:309-354: groups 1..15 for one frame. Returns (tokens[15], logits list).
        ``forced`` (optional 15 ints) teacher-forces the tokens fed back (parity tests)."""
        self.reset_cp()
        x0 = bf16r(h_backbone.to(self.dt))
        x1 = self.codec_embedding[g0]
        h = self.cp_forward(torch.stack([x0, x1]), [0, 1])[-1]
        tokens, all_logits = [], []
        for g in range(15):
            if g > 0:
                prev = tokens[-1] if forced is None else forced[g - 1]
                h = self.cp_forward(self.cp_embed[g - 1][prev].reshape(1, -1), [g + 1])[0]
            logits = self.head_logits(self.cp_head[g], h)
            all_logits.append(logits)
            u = draw_u24(seed, frame, g + 1, stream) if do_sample else None
            tokens.append(sample_token(logits, do_sample, temperature, top_k, 1.0, None, u))
        return tokens, all_logits

    def combine(self, groups, extra_row: torch.Tensor) -> torch.Tensor:
        """generator.py:143-149,356-362: sequential bf16 adds of the 16 embeddings, then the
        trailing-text (or pad) row."""
        c = self.codec_embedding[groups[0]].clone()
        for i in range(15):
            c = bf16r(c + self.cp_embed[i][groups[i + 1]])
        return bf16r(c + bf16r(extra_row.to(self.dt)))

    def suppress_mask(self, eos: int):
        d = self.d
        m = torch.zeros(d.vocab, dtype=torch.bool)
        m[d.vocab - 1024:] = True
        m[eos] = False
        return m

    def generate(self, talker_input_embeds, trailing_text_hidden, tts_pad_embed, max_tokens=500,
                 do_sample=False, temperature=0.9, top_k=50, top_p=1.0, cp_do_sample=False,
                 cp_temperature=0.9, cp_top_k=50, min_new_tokens=2, repetition_penalty=1.0,
                 eos_token_id=None, seed=0, stream=0, forced_codes=None, record=None):
        """generator.py:77-176 for one utterance. Inputs are 2-D (leading batch dim of 1
        dropped): embeds [L, hidden], trailing [T, hidden], pad [hidden]. Returns the list of
        [16] frames. ``forced_codes`` (list of [16]) teacher-forces the fed-back tokens;
        ``record`` (dict) collects per-frame logits for parity tests."""
        eos = self.d.eos_token_id if eos_token_id is None else eos_token_id
        sup = self.suppress_mask(eos)
        h = self.prefill(talker_input_embeds)
        logits = self.head_logits(self.codec_head, h)
        logits[sup] = float("-inf")
        u = draw_u24(seed, 0, 0, stream) if do_sample else None
        g0 = sample_token(logits, do_sample, temperature, top_k, top_p,
                          eos if min_new_tokens > 0 else None, u)
        if record is not None:
            record.setdefault("g0_logits", []).append(logits)
        frames, hist = [], []
        T = trailing_text_hidden.shape[0]
        for step in range(max_tokens):
            if forced_codes is not None:
                if step >= len(forced_codes):
                    break
                g0_in = forced_codes[step][0]
            else:
                g0_in = g0
            if g0_in == eos:
                break
            hist.append(g0_in)
            forced = None if forced_codes is None else forced_codes[step][1:]
            toks, cpl = self.cp_chain(h, g0_in, cp_do_sample, cp_temperature, cp_top_k,
                                      seed, step, stream, forced)
            groups = [g0_in] + (toks if forced is None else list(forced))
            frames.append([g0] + toks if forced_codes is None else [g0] + toks)
            if record is not None:
                record.setdefault("cp_logits", []).append(cpl)
                record.setdefault("hidden", []).append(h)
            extra = trailing_text_hidden[step] if step < T else tts_pad_embed.reshape(-1)
            x = self.combine(groups, extra)
            h = self.backbone_step(x)
            logits = self.head_logits(self.codec_head, h)
            logits[sup] = float("-inf")
            logits = apply_repetition_penalty(logits, hist, repetition_penalty)
            u = draw_u24(seed, step + 1, 0, stream) if do_sample else None
            g0 = sample_token(logits, do_sample, temperature, top_k, top_p,
                              eos if step + 1 < min_new_tokens else None, u)
            if record is not None:
                record.setdefault("g0_logits", []).append(logits)
        return frames
