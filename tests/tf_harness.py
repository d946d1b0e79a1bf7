"""Teacher-forced frame comparison between the engine and the CPU oracle.

Free-running greedy sequences of two correct implementations diverge at the first near-tie,
so frame parity is measured the way the reference's own gate does it for early tokens
(tests/test_audio.py:281-324 compares the first g0 tokens): each frame starts both sides
from the SAME state -- the engine's backbone hidden, group-0 token, KV cache rows and
repetition history -- and compares what each produces for that frame:

* the 15 code-predictor logit vectors and tokens (the oracle runs the chain from the
  engine's hidden and group-0 token, feeding back the engine's tokens),
* the backbone step on the engine's combined embedding (same KV rows), the codec-head
  logits and the next group-0 token (greedy, or sampled with the same Philox draw from
  the engine's own logits, which isolates the device sampler).
"""
from __future__ import annotations

import torch

from oracle import qtt_oracle as O


ATOL, RTOL = 2e-2, 1e-2   # BASELINE.json north_star logits tolerance (atol / rtol)


def violation(a, b):
    """max over finite elements of |a - b| - (ATOL + RTOL |b|); <= 0 means within tolerance."""
    fin = torch.isfinite(b)
    return float(((a - b).abs() - (ATOL + RTOL * b.abs()))[fin].max())


def bf16_ulp(b):
    """Spacing of bf16 values at |b| (8 significant bits): the rounding quantum of a bf16 logit."""
    e = torch.floor(torch.log2(b.abs().clamp_min(2.0 ** -126)))
    return torch.exp2(e - 7)


def violation_ulp(a, b):
    """As violation(), with one more bf16 ulp of b allowed: both sides round their logits to
    bf16, so an fp32 difference far below the tolerance can still move a logit by one ulp."""
    fin = torch.isfinite(b)
    return float(((a - b).abs() - (ATOL + RTOL * b.abs() + bf16_ulp(b)))[fin].max())


def _compare_frame(orc, kv, h_e, g0, pos, step, codes, g0_next, cp_e, g0l_e, h_e2, trailing, pad, sp, sampling,
                   hist, sup, eos, peer=None):
    """One teacher-forced frame: the oracle runs from the engine's state before the frame
    (h_e, g0, KV rows), the engine's results are codes / g0_next / cp_e / g0l_e / h_e2. ``kv``:
    (k, v) of the engine's cache after the frame (its new row is copied into the oracle)."""
    rec = {"codes": codes, "g0_next": g0_next}
    # --- code predictor from the engine's state, fed back with the engine's tokens
    cp_do = sampling is not None and sampling.get("cp_do_sample", False)
    _, cp_o = orc.cp_chain(h_e, g0, forced=codes[1:])
    rec["cp_logits_err"] = max(float((cp_e[g] - cp_o[g].double()).abs().max()) for g in range(15))
    rec["cp_logits_viol"] = max(violation(cp_e[g], cp_o[g].double()) for g in range(15))
    cp_pred, cp_ties = [], []
    for g in range(15):
        if cp_do:   # sampled: same Philox draw on the ENGINE's logits (isolates the sampler)
            u = O.draw_u24(sampling["seed"], step, g + 1, sampling["stream"])
            cp_pred.append(O.sample_token(cp_e[g], True, sampling["cp_temperature"], sampling["cp_top_k"],
                                          1.0, None, u))
            cp_ties.append(None)
        else:       # greedy: argmax of the oracle's own logits
            lo = cp_o[g].double()
            cp_pred.append(O.argmax_first(lo))
            srt = torch.sort(lo, descending=True)[0]
            cp_ties.append(float(srt[0] - srt[1]))
    rec["cp_pred"] = cp_pred
    rec["cp_gap"] = cp_ties
    # --- backbone on the engine's combined input and KV rows
    extra = trailing[step] if step < trailing.shape[0] else pad
    x = orc.combine(codes, extra.to(orc.dt))
    orc.position = pos
    h_o = orc.backbone_step(x)
    rec["h_rel"] = float((h_e2 - h_o).norm() / h_o.norm())
    lo = orc.head_logits(orc.codec_head, h_o).double()
    rec["g0_logits_err"] = float((g0l_e - lo).abs().max())
    rec["g0_logits_viol"] = violation(g0l_e, lo)
    rec["g0_logits_viol_ulp"] = violation_ulp(g0l_e, lo)
    if peer is not None:
        # another implementation's backbone step on the same input and KV rows (the reference's
        # own kernel): how far its codec-head logits land from the exact math
        h_p = peer(x, pos, kv).to(orc.dt)
        lp = bf16_logits(orc.codec_head, h_p)
        rec["peer_g0_logits_err"] = float((lp - lo).abs().max())
        rec["peer_g0_logits_viol"] = violation(lp, lo)
    # --- next group 0: greedy from the oracle's logits; sampled from the ENGINE's logits
    min_new = sp.min_new_tokens
    mask_eos = eos if step + 1 < min_new else None
    if sampling is None:
        l2 = lo.clone()
        l2[sup] = float("-inf")
        l2 = O.apply_repetition_penalty(l2, hist, sp.repetition_penalty)
        rec["g0_pred"] = O.sample_token(l2, False, 0.9, 50, 1.0, mask_eos)
        srt = torch.sort(l2[torch.isfinite(l2)], descending=True)[0]
        rec["g0_gap"] = float(srt[0] - srt[1])
    else:
        l2 = g0l_e.clone()
        l2[sup] = float("-inf")
        l2 = O.apply_repetition_penalty(l2, hist, sampling["repetition_penalty"])
        u = O.draw_u24(sampling["seed"], step + 1, 0, sampling["stream"])
        rec["g0_pred"] = O.sample_token(l2, True, sampling["temperature"], sampling["top_k"],
                                        sampling.get("top_p", 1.0), mask_eos, u)
        rec["g0_gap"] = None
    # --- keep the oracle's cache identical to the engine's
    kc, vc = kv
    orc.bk[:, :, pos] = kc[:, :, pos].cpu().to(orc.dt)
    orc.bv[:, :, pos] = vc[:, :, pos].cpu().to(orc.dt)
    return rec


def bf16_logits(W, h):
    """Codec-head logits as the reference computes them: bf16 values of W @ bf16(h)."""
    return O.Qwen3TTSOracle.head_logits(W, h).double()


def run_teacher_forced(eng, orc, embeds, trailing, pad, sp, n_frames, sampling=None, peer=None):
    """Returns a list of per-frame dicts. ``sampling``: None for greedy, else dict(temperature,
    top_k, repetition_penalty, seed, stream, cp_temperature, cp_top_k, cp_do_sample,
    min_new_tokens). ``peer(x, pos, (k, v))``: optional second implementation of the backbone
    step, run on each frame's combined input x at position pos over the engine's KV rows; its
    codec-head logits are compared with the exact math as well (``peer_g0_logits_*``)."""
    eng.prefill(0, embeds.cuda(), sp)
    st = eng.state(0)
    P = st["position"]
    kc, vc = eng.kv(0)
    orc.reset_backbone()
    orc.set_kv_cache(kc[:, :, :P].cpu().to(orc.dt), vc[:, :, :P].cpu().to(orc.dt))
    cp_dbg = torch.zeros(15, orc.d.cp_vocab, dtype=torch.float32, device="cuda")
    g0_dbg = torch.zeros(orc.d.vocab, dtype=torch.float32, device="cuda")
    eng.set_debug_outputs(cp_dbg, g0_dbg)
    eos = orc.d.eos_token_id if sampling is None else sampling.get("eos", orc.d.eos_token_id)
    sup = orc.suppress_mask(eos)
    hist = []
    out = []
    try:
        for _ in range(n_frames):
            st = eng.state(0)
            pos, g0, step = st["position"], st["g0"], st["frames"]
            h_e = eng.hidden(0).cpu().to(orc.dt)
            eng.frames(0, 1, trailing.cuda(), pad.cuda(), sp)
            eng.check()
            codes = eng.codes(0)[step].cpu().tolist()
            g0_next = eng.state(0)["g0"]
            hist.append(g0)
            out.append(_compare_frame(orc, eng.kv(0), h_e, g0, pos, step, codes, g0_next, cp_dbg.cpu().double(),
                                      g0_dbg.cpu().double(), eng.hidden(0).cpu().to(orc.dt), trailing, pad, sp,
                                      sampling, hist, sup, eos, peer))
    finally:
        eng.set_debug_outputs(None, None)
    return out


def run_teacher_forced_batch(eng, orc, embeds, trailing, pads, sp, n_frames, sampling=None, check=None,
                             prefill=True, peer=None):
    """The same for the batched path: utterances 0..B-1 of ``eng`` advance together through
    qtt_batch_frames; each utterance in ``check`` (default: all) is compared with the oracle
    holding that utterance's own KV cache (one oracle, its caches swapped per utterance).
    Returns one list of per-frame dicts per checked utterance, in ``check`` order. With
    ``prefill=False`` the caller has already prefilled the utterances."""
    B = len(embeds)
    check = list(range(B)) if check is None else list(check)
    if prefill:
        eng.batch_prefill([e.cuda() for e in embeds], sp)
    eng.check()
    caches = {}
    for s in check:
        P = eng.state(s)["position"]
        kc, vc = eng.kv(s)
        orc.reset_backbone()
        orc.set_kv_cache(kc[:, :, :P].cpu().to(orc.dt), vc[:, :, :P].cpu().to(orc.dt))
        caches[s] = (orc.bk, orc.bv)
    d = orc.d
    cp_dbg = torch.zeros(B, 15, d.cp_vocab, dtype=torch.float32, device="cuda")
    g0_dbg = torch.zeros(B, d.vocab, dtype=torch.float32, device="cuda")
    eng.batch_set_debug_outputs(cp_dbg, g0_dbg)
    eos = d.eos_token_id if sampling is None else sampling.get("eos", d.eos_token_id)
    sup = orc.suppress_mask(eos)
    hists = {s: [] for s in check}
    out = {s: [] for s in check}
    tr = [None if t is None else t.cuda() for t in trailing]
    pd = [x.cuda() for x in pads]
    try:
        for _ in range(n_frames):
            before = {}
            for s in check:
                st = eng.state(s)
                before[s] = (st["position"], st["g0"], st["frames"], eng.hidden(s).cpu().to(orc.dt))
            eng.batch_frames(1, tr, pd, sp)
            eng.check()
            for s in check:
                pos, g0, step, h_e = before[s]
                codes = eng.codes(s)[step].cpu().tolist()
                g0_next = eng.state(s)["g0"]
                hists[s].append(g0)
                orc.bk, orc.bv = caches[s]
                smp = None if sampling is None else dict(sampling, stream=sampling["stream"] + s)
                out[s].append(_compare_frame(orc, eng.kv(s), h_e, g0, pos, step, codes, g0_next,
                                             cp_dbg[s].cpu().double(), g0_dbg[s].cpu().double(),
                                             eng.hidden(s).cpu().to(orc.dt), trailing[s], pads[s], sp, smp,
                                             hists[s], sup, eos, peer))
    finally:
        eng.batch_set_debug_outputs(None, None)
    return [out[s] for s in check]
