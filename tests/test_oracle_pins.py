"""Pins the CPU oracle (oracle/qtt_oracle.py) before it is trusted as the parity reference:

* Philox4x32-10 against the published Random123 known-answer vectors;
* mRoPE with equal (t, h, w) position ids against the reference's 1D tables
  (megakernel_backbone.py:389-398) and the section layout of rope_multimodal.cuh:26-54;
* decoder-layer math against transformers' Qwen3Model (the PyTorch forward the reference's
  talker and code predictor are built from) in fp32;
* sampler / combine / repetition penalty against literal restatements of the reference's
  torch code (generator.py:143-207,356-362) on bf16 tensors;
* reference-kernel golden vectors (tests/golden/ref_megakernel_golden.npz, produced on a B200
  by tests/golden/make_ref_golden.py from the reference's own CUDA kernels).
"""
import os

import numpy as np
import pytest
import torch

from oracle import qtt_oracle as O
from qwentts_turbo_b200.config import DEFAULT_DIMS, LAYER_TENSORS, frame_weight_bytes
from qwentts_turbo_b200.weights import rope_tables, synthetic_weights

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_megakernel_golden.npz")


# Random123 kat_vectors, philox4x32 with 10 rounds: counter, key -> output
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,out", PHILOX_KAT)
def test_philox_known_answers(ctr, key, out):
    assert O.philox4x32_10(ctr, key) == out


def test_frame_weight_bytes():
    # BASELINE: 880,934,912 + 6,291,456 + 15 * (157,311,488 + 4,194,304)
    assert frame_weight_bytes() == 3_309_813_248
    assert DEFAULT_DIMS.layer_bytes() == 31_461_888


@pytest.mark.parametrize("pos", [0, 1, 2, 7, 63, 255, 1000, 4095])
def test_mrope_equal_positions_is_1d_table(pos):
    cos, sin = rope_tables(4096)
    c, s = O.mrope_cos_sin(pos, pos, pos)
    assert torch.equal(c, cos[pos].float()) and torch.equal(s, sin[pos].float())


def test_mrope_section_layout():
    inv = torch.ones(64)
    ang = O.mrope_angles(1.0, 2.0, 3.0, inv, (24, 20, 20))[:64]
    assert int((ang == 1).sum()) == 24 and int((ang == 2).sum()) == 20 and int((ang == 3).sum()) == 20
    assert torch.equal(ang[60:], torch.ones(4))          # the tail frequencies are temporal
    assert ang[1] == 2 and ang[2] == 3 and ang[3] == 1   # T H W T ... interleave


def _hf_model(weights, prefix, n_layers):
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3Model
    d = DEFAULT_DIMS
    cfg = Qwen3Config(vocab_size=16, hidden_size=d.hidden, intermediate_size=d.intermediate,
                      num_hidden_layers=n_layers, num_attention_heads=d.n_q_heads,
                      num_key_value_heads=d.n_kv_heads, head_dim=d.head_dim, rms_norm_eps=d.rms_eps,
                      rope_parameters={"rope_type": "default", "rope_theta": d.rope_theta},
                      max_position_embeddings=8192, attn_implementation="eager")
    m = Qwen3Model(cfg).float().eval()
    attr = {"input_layernorm": "input_layernorm", "q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj",
            "v_proj": "self_attn.v_proj", "q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm",
            "o_proj": "self_attn.o_proj", "post_attention_layernorm": "post_attention_layernorm",
            "gate_proj": "mlp.gate_proj", "up_proj": "mlp.up_proj", "down_proj": "mlp.down_proj"}
    sd = {}
    for i in range(n_layers):
        for t in LAYER_TENSORS:
            sd[f"layers.{i}.{attr[t]}.weight"] = weights[f"{prefix}.layers.{i}.{t}"].float()
    sd["norm.weight"] = weights[f"{prefix}.norm"].float()
    sd["embed_tokens.weight"] = torch.zeros(16, d.hidden)
    m.load_state_dict(sd)
    return m


def test_oracle_layers_match_transformers_qwen3(small_weights):
    """fp32 hidden / fp32 KV path (the code predictor's) against HF Qwen3Model, causal, 6 tokens."""
    orc = O.Qwen3TTSOracle(small_weights, backbone_layers=2, cp_layers=2, max_seq=64, cp_max_seq=64,
                           exact_rope=True)
    g = torch.Generator().manual_seed(5)
    x = O.bf16r(torch.randn(6, 1024, generator=g))
    ours = orc.cp_forward(x, list(range(6)))
    m = _hf_model(small_weights, "cp", 2)
    with torch.no_grad():
        ref = m(inputs_embeds=x[None], position_ids=torch.arange(6)[None]).last_hidden_state[0]
    err = (ours - ref).abs().max().item()
    assert err < 2e-4 * max(1.0, ref.abs().max().item()), err


def test_oracle_decode_equals_prefill(small_weights):
    """Token-by-token decode gives the same result as the causal multi-token forward."""
    g = torch.Generator().manual_seed(6)
    x = O.bf16r(torch.randn(5, 1024, generator=g))
    a = O.Qwen3TTSOracle(small_weights, backbone_layers=2, cp_layers=2, max_seq=64)
    full = a.backbone_forward(x, list(range(5)))
    b = O.Qwen3TTSOracle(small_weights, backbone_layers=2, cp_layers=2, max_seq=64)
    steps = torch.stack([b.backbone_step(x[i]) for i in range(5)])
    # the hidden state is rounded to bf16 after every layer, so a different fp32 summation
    # order can move a value by one bf16 ulp (1/64 at |h| in [2, 4))
    assert (full - steps).abs().max().item() < 2e-2
    assert (a.bk[:, :, :5] - b.bk[:, :, :5]).abs().max() < 2e-2


def test_backbone_rounding_points(small_weights):
    orc = O.Qwen3TTSOracle(small_weights, backbone_layers=2, cp_layers=2, max_seq=64)
    g = torch.Generator().manual_seed(7)
    orc.backbone_step(O.bf16r(torch.randn(1024, generator=g)))
    kv = orc.bk[:, :, 0]
    assert torch.equal(kv, O.bf16r(kv))          # K stored as bf16 (fused_decode_tts.cu:271)
    assert torch.equal(orc.bv[:, :, 0], O.bf16r(orc.bv[:, :, 0]))


def _ref_sample(logits_bf16, do_sample, temperature, top_k, suppress_eos_id):
    """Literal restatement of generator.py:179-194 up to the multinomial (returns probs)."""
    logits = logits_bf16.clone()
    if suppress_eos_id is not None:
        logits[suppress_eos_id] = float("-inf")
    if not do_sample:
        return int(logits.argmax().item()), None
    scaled = logits / temperature
    if top_k > 0:
        topk_vals = torch.topk(scaled, min(top_k, scaled.size(-1)))[0]
        scaled[scaled < topk_vals[-1]] = float("-inf")
    return None, torch.softmax(scaled, dim=-1)


@pytest.mark.parametrize("seed", range(6))
def test_sampler_matches_reference_semantics(seed):
    g = torch.Generator().manual_seed(seed)
    logits = (torch.randn(3072, generator=g) * 0.7).to(torch.bfloat16)
    logits[3000:3010] = logits[5]          # ties
    eos = 2150
    a, _ = _ref_sample(logits, False, 0.9, 50, eos)
    assert O.sample_token(logits.float(), False, 0.9, 50, 1.0, eos) == a
    _, probs = _ref_sample(logits, True, 0.9, 50, eos)
    kept_ref = probs > 0
    # oracle: the kept set equals the reference's, and draws land only on kept ids
    picks = {O.sample_token(logits.float(), True, 0.9, 50, 1.0, eos, u24=u) for u in range(0, 1 << 24, 1 << 14)}
    assert all(bool(kept_ref[p]) for p in picks)
    assert len(picks) >= min(40, int(kept_ref.sum()))


def _ref_top_p_kept(logits_bf16, temperature, top_k, top_p):
    """Literal restatement of generator.py:188-205 up to the multinomial, on bf16 tensors as the
    reference runs it (the sort made stable: torch.sort leaves the order of equal values open):
    the set of ids with nonzero probability after top-k and top-p."""
    scaled = logits_bf16.clone() / temperature
    if top_k > 0:
        topk_vals = torch.topk(scaled, min(top_k, scaled.size(-1)))[0]
        scaled[scaled < topk_vals[-1]] = float("-inf")
    if top_p < 1.0:
        sorted_logits, sorted_idx = torch.sort(scaled, descending=True, stable=True)
        cumprobs = torch.cumsum(torch.softmax(sorted_logits, dim=-1), dim=-1)
        remove = cumprobs > top_p
        remove[1:] = remove[:-1].clone()
        remove[0] = False
        sorted_logits[remove] = float("-inf")
        scaled.scatter_(0, sorted_idx, sorted_logits)
    return torch.softmax(scaled, dim=-1) > 0


@pytest.mark.parametrize("seed,top_k,top_p", [(0, 50, 0.8), (1, 50, 0.5), (2, 0, 0.9), (3, 20, 0.3), (4, 0, 0.97)])
def test_top_p_matches_reference_semantics(seed, top_k, top_p):
    """The oracle's nucleus filter keeps exactly the reference's set of ids, and its draws land
    only there."""
    g = torch.Generator().manual_seed(seed)
    logits = (torch.randn(3072, generator=g) * 1.5).to(torch.bfloat16)
    kept_ref = _ref_top_p_kept(logits, 0.9, top_k, top_p)
    kept = torch.isfinite(O.filter_logits(logits.float(), 0.9, top_k, top_p))
    assert torch.equal(kept, kept_ref), (int(kept.sum()), int(kept_ref.sum()))
    picks = {O.sample_token(logits.float(), True, 0.9, top_k, top_p, None, u24=u) for u in range(0, 1 << 24, 1 << 14)}
    assert all(bool(kept_ref[p]) for p in picks)


def test_inverse_cdf_pick_edges():
    p = torch.tensor([0.0, 0.25, 0.0, 0.5, 0.25]).to(torch.bfloat16).float()
    assert O.inverse_cdf_pick(p, 0) == 1
    assert O.inverse_cdf_pick(p, (1 << 24) - 1) == 4
    assert O.inverse_cdf_pick(p, 1 << 23) == 3        # u = 0.5 -> cum 0.25 | 0.75
    counts = np.zeros(5)
    for u in range(0, 1 << 24, 1 << 12):
        counts[O.inverse_cdf_pick(p, u)] += 1
    np.testing.assert_allclose(counts / counts.sum(), p.numpy(), atol=1e-3)


def test_combine_is_sequential_bf16(small_weights):
    orc = O.Qwen3TTSOracle(small_weights, backbone_layers=2, cp_layers=2, max_seq=16)
    groups = [5] + list(range(100, 115))
    extra = torch.randn(1024).to(torch.bfloat16)
    # generator.py:356-362 then :147 on bf16 tensors
    c = small_weights["talker.codec_embedding"][groups[0]].clone()
    for i in range(15):
        c = c + small_weights[f"cp.codec_embedding.{i}"][groups[i + 1]]
    c = c + extra
    assert torch.equal(orc.combine(groups, extra.float()), c.float())


def test_repetition_penalty_matches_reference():
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(3072, generator=g).to(torch.bfloat16)
    hist = [7, 7, 100, 2500, 3]
    ref = logits.clone()
    prev = torch.tensor(hist, dtype=torch.long)
    scores = ref[prev]
    ref[prev] = torch.where(scores > 0, scores / 1.2, scores * 1.2)   # generator.py:163-167
    assert torch.equal(O.apply_repetition_penalty(logits.float(), hist, 1.2), ref.float())


@pytest.mark.skipif(not os.path.exists(GOLDEN), reason="reference-kernel golden vectors not generated yet")
def test_oracle_matches_reference_kernel_golden():
    """Outputs of the reference's own CUDA kernels (run on a B200 by
    tests/golden/make_ref_golden.py) vs the oracle on the same seeded inputs. The fp64 oracle
    (exact math at the reference's rounding points) reproduces the reference kernel's C1
    backbone step to < 1e-5 and its code-predictor steps to < 1e-5; the fp32 oracle differs by
    a bf16 flip cascade (0.038 max-abs), which is why the GPU tests use the fp64 oracle."""
    from qwentts_turbo_b200.workloads import c1_inputs
    z = np.load(GOLDEN)
    nb, nc, ctx = int(z["bb_layers"]), int(z["cp_layers"]), int(z["ctx"])
    w = synthetic_weights(backbone_layers=nb, cp_layers=nc)
    orc = O.Qwen3TTSOracle(w, backbone_layers=nb, cp_layers=nc, max_seq=512, dtype=torch.float64)
    k, v, emb = c1_inputs(nb, ctx, int(z["kv_seed"]))
    orc.set_kv_cache(k.double(), v.double())
    orc.position = ctx
    h = orc.backbone_step(emb.double())
    ref = torch.from_numpy(z["bb_hidden"]).double()
    assert (h - ref).abs().max().item() < 1e-5
    # code-predictor steps (reference kernel: one token per launch from position 0)
    orc.reset_cp()
    cp_in = torch.from_numpy(z["cp_emb"]).double()
    cp_ref = torch.from_numpy(z["cp_hidden"]).double()
    for i in range(cp_in.shape[0]):
        hi = orc.cp_forward(cp_in[i:i + 1], [i])[0]
        assert (hi - cp_ref[i]).abs().max().item() < 1e-5, i
