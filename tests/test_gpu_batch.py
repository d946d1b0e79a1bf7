"""Batched decode (qtt_batch_prefill / qtt_batch_frames): several utterances advance together,
every projection a tcgen05 GEMM over bf16 hi/lo activation planes. Checked against the fp64
oracle the same way as the batch-1 engine (tests/tf_harness.py): each frame of each utterance
starts the oracle from the engine's state for that utterance, and the tokens (ties excepted),
the code-predictor and codec-head logits (atol 2e-2 / rtol 1e-2) and the backbone hidden must
agree. Also: batched prefill vs the oracle's causal prefill, batched vs batch-1 engine codes,
and the argument checks."""
import pytest
import torch

from oracle import qtt_oracle as O
from qwentts_turbo_b200 import _lib
from qwentts_turbo_b200.engine import DeviceModel, Engine, sampling_struct
from qwentts_turbo_b200.workloads import c3_inputs
from tests.tf_harness import run_teacher_forced_batch

pytestmark = pytest.mark.gpu

F64 = torch.float64
TIE_TOL = 4e-2     # two bf16 ulps at |logit| in [2, 4)
HID_REL = 1.5e-2   # final-normed hidden ||a - b|| / ||b|| (allows one bf16 flip cascade)


def _greedy_sp(**kw):
    base = dict(do_sample=False, min_new_tokens=10_000)
    base.update(kw)
    return sampling_struct(**base)


def _frame_stats(recs, greedy=True):
    full, bad = 0, []
    for f, r in enumerate(recs):
        ok = True
        for g in range(15):
            if r["codes"][g + 1] != r["cp_pred"][g]:
                ok = False
                if not greedy or r["cp_gap"][g] > TIE_TOL:
                    bad.append((f, g + 1, r["codes"][g + 1], r["cp_pred"][g], r["cp_gap"][g]))
        if r["g0_next"] != r["g0_pred"]:
            ok = False
            if not greedy or r["g0_gap"] > TIE_TOL:
                bad.append((f, 0, r["g0_next"], r["g0_pred"], r["g0_gap"]))
        full += ok
    return full, bad


def _inputs(ctxs, n_trailing, seed):
    out = [c3_inputs(ctx=c, n_trailing=n_trailing, seed=seed + i) for i, c in enumerate(ctxs)]
    return [o[0] for o in out], [o[1] for o in out], [o[2] for o in out]


@pytest.fixture(scope="module")
def dev_small(small_weights):
    return DeviceModel(small_weights, rope_rows=1024, backbone_layers=2, cp_layers=2)


@pytest.fixture(scope="module")
def orc_small(small_weights):
    return O.Qwen3TTSOracle(small_weights, backbone_layers=2, cp_layers=2, max_seq=512, dtype=F64)


def test_batch_prefill_matches_oracle(dev_small, orc_small):
    """Uneven contexts in one batch: each utterance's decode state equals the oracle's causal
    prefill of its own context."""
    embeds, _, _ = _inputs([9, 23, 40], 0, 31)
    eng = Engine(dev_small, max_streams=3, max_seq=512, max_frames=16)
    try:
        eng.batch_prefill([e.cuda() for e in embeds], _greedy_sp())
        eng.check()
        for s, e in enumerate(embeds):
            ref = orc_small.prefill(e.to(F64))
            got = eng.hidden(s).cpu().to(F64)
            assert eng.state(s)["position"] == e.shape[0]
            rel = float((got - ref).norm() / ref.norm())
            assert rel <= HID_REL, f"utterance {s}: rel {rel:.3g}"
    finally:
        eng.close()


def test_prefill_tc_matches_oracle(dev_small, orc_small):
    """Tensor-core prefill in chunks of up to 128 positions (contexts of 9, 150 and 300 positions:
    one to three chunks): the decode state equals the oracle's causal prefill, the cached K/V rows
    equal the oracle's up to bf16 rounding, and the first group-0 token equals the token-by-token
    prefill's unless the top two logits are within two bf16 ulps."""
    embeds, _, _ = _inputs([9, 150, 300], 0, 61)
    sp = _greedy_sp()
    eng = Engine(dev_small, max_streams=2, max_seq=512, max_frames=16)
    try:
        for e in embeds:
            L = e.shape[0]
            eng.prefill_tc(0, e.cuda(), sp)
            eng.check()
            ref = orc_small.prefill(e.to(F64))
            assert eng.state(0)["position"] == L
            got = eng.hidden(0).cpu().to(F64)
            rel = float((got - ref).norm() / ref.norm())
            assert rel <= HID_REL, f"L={L}: hidden rel {rel:.3g}"
            k, v = eng.kv(0)
            for a, b in ((k, orc_small.bk), (v, orc_small.bv)):
                a = a[:, :, :L].cpu().to(F64)
                b = b[:, :, :L]
                krel = float((a - b).norm() / b.norm())
                assert krel <= HID_REL, f"L={L}: cache rel {krel:.3g}"
            g0_tc = eng.state(0)["g0"]
            eng.prefill(1, e.cuda(), sp)
            eng.check()
            lo = orc_small.head_logits(orc_small.codec_head, ref).double()
            lo[orc_small.suppress_mask(orc_small.d.eos_token_id)] = float("-inf")
            top = torch.sort(lo, descending=True)[0]
            if float(top[0] - top[1]) > TIE_TOL:
                assert g0_tc == eng.state(1)["g0"], f"L={L}"
    finally:
        eng.close()


def test_batch_small_teacher_forced(dev_small, orc_small):
    """2+2-layer model with random norm weights, 3 utterances of different contexts, greedy with
    repetition penalty, 8 frames (trailing rows, then the pad row)."""
    embeds, trailing, pads = _inputs([17, 30, 41], 5, 21)
    eng = Engine(dev_small, max_streams=3, max_seq=512, max_frames=16)
    try:
        recs = run_teacher_forced_batch(eng, orc_small, embeds, trailing, pads, _greedy_sp(repetition_penalty=1.3), 8)
    finally:
        eng.close()
    for s, r in enumerate(recs):
        full, bad = _frame_stats(r)
        assert not bad, (s, bad)
        assert full >= len(r) - 1, (s, full)
        assert max(x["cp_logits_viol"] for x in r) <= 0
        assert max(x["g0_logits_viol"] for x in r) <= 0
        assert max(x["h_rel"] for x in r) <= HID_REL


def test_batch_kv_in_attention_path(dev_small, orc_small):
    """The path of GPUs whose clusters hold 2 CTAs (q/k norms, RoPE and the new K/V rows in the
    attention stage rather than the QKV epilogue; forced by the qtt_set_debug_kv_in_attention test
    hook): the same teacher-forced frames and a tensor-core prefill against the oracle."""
    embeds, trailing, pads = _inputs([17, 30, 41], 5, 21)
    eng = Engine(dev_small, max_streams=3, max_seq=512, max_frames=16)
    try:
        _lib.check(eng.lib.qtt_set_debug_kv_in_attention(eng.h, 1), "qtt_set_debug_kv_in_attention")
        recs = run_teacher_forced_batch(eng, orc_small, embeds, trailing, pads, _greedy_sp(repetition_penalty=1.3), 6)
        for s, r in enumerate(recs):
            full, bad = _frame_stats(r)
            assert not bad, (s, bad)
            assert full >= len(r) - 1, (s, full)
            assert max(x["h_rel"] for x in r) <= HID_REL
        e = _inputs([150], 0, 61)[0][0]
        eng.prefill_tc(0, e.cuda(), _greedy_sp())
        eng.check()
        ref = orc_small.prefill(e.to(F64))
        got = eng.hidden(0).cpu().to(F64)
        assert float((got - ref).norm() / ref.norm()) <= HID_REL
    finally:
        eng.lib.qtt_set_debug_kv_in_attention(eng.h, 0)
        eng.close()


def test_batch_sampling_teacher_forced(dev_small, orc_small):
    """Temperature / top-k / repetition penalty with per-utterance Philox streams, code predictor
    sampled too: each utterance's picks equal the oracle sampler's on the engine's logits."""
    embeds, trailing, pads = _inputs([20, 33], 4, 41)
    cfg = dict(temperature=0.9, top_k=50, repetition_penalty=1.2, seed=77, stream=5, cp_do_sample=True,
               cp_temperature=0.9, cp_top_k=50)
    sp = sampling_struct(do_sample=True, temperature=0.9, top_k=50, repetition_penalty=1.2, min_new_tokens=10_000,
                         cp_do_sample=True, cp_temperature=0.9, cp_top_k=50, seed=77, philox_stream=5)
    eng = Engine(dev_small, max_streams=2, max_seq=512, max_frames=16)
    try:
        recs = run_teacher_forced_batch(eng, orc_small, embeds, trailing, pads, sp, 5, sampling=cfg)
    finally:
        eng.close()
    for s, r in enumerate(recs):
        _, bad = _frame_stats(r, greedy=False)
        assert len(bad) <= 1, (s, bad)
        assert max(x["cp_logits_viol"] for x in r) <= 0


def test_batch_top_p_teacher_forced(dev_small, orc_small):
    """Nucleus sampling in the batched path (one CTA per utterance runs the sampler): each
    utterance's group-0 picks equal the oracle sampler's on the engine's logits."""
    embeds, trailing, pads = _inputs([15, 28], 4, 71)
    cfg = dict(temperature=0.9, top_k=50, top_p=0.7, repetition_penalty=1.2, seed=5, stream=1, cp_do_sample=False)
    sp = sampling_struct(do_sample=True, temperature=0.9, top_k=50, top_p=0.7, repetition_penalty=1.2,
                         min_new_tokens=10_000, seed=5, philox_stream=1)
    eng = Engine(dev_small, max_streams=2, max_seq=512, max_frames=16)
    try:
        recs = run_teacher_forced_batch(eng, orc_small, embeds, trailing, pads, sp, 5, sampling=cfg)
    finally:
        eng.close()
    for s, r in enumerate(recs):
        bad = [(f, x["g0_next"], x["g0_pred"]) for f, x in enumerate(r) if x["g0_next"] != x["g0_pred"]]
        assert len(bad) <= 1, (s, bad)


def test_batch_matches_batch1_engine(dev_small):
    """Free-running greedy codes of the batched path equal the batch-1 engine's on the same
    utterances until the first near-tie (checked over the first 2 frames)."""
    embeds, trailing, pads = _inputs([12, 25], 3, 51)
    sp = _greedy_sp()
    e1 = Engine(dev_small, max_streams=1, max_seq=512, max_frames=16)
    ref = []
    try:
        for s in range(2):
            e1.prefill(0, embeds[s].cuda(), sp)
            e1.frames(0, 2, trailing[s].cuda(), pads[s].cuda(), sp)
            e1.check()
            ref.append(e1.codes(0)[:2].cpu())
    finally:
        e1.close()
    eb = Engine(dev_small, max_streams=2, max_seq=512, max_frames=16)
    try:
        eb.batch_prefill([e.cuda() for e in embeds], sp)
        eb.batch_frames(2, [t.cuda() for t in trailing], [x.cuda() for x in pads], sp)
        eb.check()
        same = sum(int((eb.codes(s)[:2].cpu() == ref[s]).sum()) for s in range(2))
    finally:
        eb.close()
    assert same >= 60, f"{same}/64 codes equal"


def test_batch_last_codes(dev_small):
    """qtt_batch_last_codes gathers each stream's latest frame (-1s before the first frame), the
    rows a serving loop copies to the host once per batched frame."""
    embeds, trailing, pads = _inputs([12, 25, 19], 4, 61)
    sp = _greedy_sp()
    eng = Engine(dev_small, max_streams=3, max_seq=512, max_frames=16)
    try:
        eng.batch_prefill([e.cuda() for e in embeds], sp)
        assert torch.equal(eng.batch_last_codes(3).cpu(), torch.full((3, 16), -1, dtype=torch.int32))
        tr, pd = [t.cuda() for t in trailing], [x.cuda() for x in pads]
        for f in range(3):
            eng.batch_frames(1, tr, pd, sp)
            got = eng.batch_last_codes(3).cpu()
            eng.check()
            want = torch.stack([eng.codes(s)[f].cpu() for s in range(3)])
            assert torch.equal(got, want), f
        assert torch.equal(eng.batch_last_codes(2).cpu(), want[:2])   # a prefix of the streams
    finally:
        eng.close()


def _batch_run(dev, embeds, trailing, pads, sp, n, debug):
    B = len(embeds)
    eng = Engine(dev, max_streams=B, max_seq=512, max_frames=16)
    try:
        if debug:   # the debug logit outputs change the heads' timing, not their results
            cp = torch.zeros(B, 15, 2048, dtype=torch.float32, device="cuda")
            g0 = torch.zeros(B, 3072, dtype=torch.float32, device="cuda")
            eng.batch_set_debug_outputs(cp, g0)
        eng.batch_prefill([e.cuda() for e in embeds], sp)
        tr, pd = [t.cuda() for t in trailing], [x.cuda() for x in pads]
        for _ in range(n):   # one launch per frame, state read back in between as a caller would
            eng.batch_frames(1, tr, pd, sp)
            _ = [eng.state(s) for s in range(B)]
        eng.check()
        return [eng.codes(s)[:n].cpu() for s in range(B)], [eng.hidden(s).cpu() for s in range(B)]
    finally:
        eng.batch_set_debug_outputs(None, None)
        eng.close()


def test_batch_runs_bit_identical(dev_small):
    """Two runs of the same frames give bit-identical codes and hidden states, with and without
    the debug outputs: every cross-CTA sum has a fixed order and every stage reads only data
    published before its barrier (a stale read shows up here as a difference)."""
    embeds, trailing, pads = _inputs([17, 30, 41], 5, 21)
    sp = _greedy_sp(repetition_penalty=1.3)
    a = _batch_run(dev_small, embeds, trailing, pads, sp, 4, False)
    b = _batch_run(dev_small, embeds, trailing, pads, sp, 4, False)
    c = _batch_run(dev_small, embeds, trailing, pads, sp, 4, True)
    for s in range(3):
        for other in (b, c):
            assert torch.equal(a[0][s], other[0][s]), s
            assert torch.equal(a[1][s], other[1][s]), s


def test_batch_eos_stops_one_utterance(dev_small):
    """EOS in the batched path: utterance 0 stops at the first frame whose group-0 token is the
    EOS id (as generator.py:125-127), its row goes idle, and the other utterance's codes are the
    same as in a run without that EOS (as long as its own tokens do not hit the id)."""
    embeds, trailing, pads = _inputs([20, 35], 4, 91)
    base = _greedy_sp()
    eng = Engine(dev_small, max_streams=2, max_seq=512, max_frames=16)
    try:
        ed, td, pd = [e.cuda() for e in embeds], [t.cuda() for t in trailing], [x.cuda() for x in pads]
        eng.batch_prefill(ed, base)
        eng.batch_frames(6, td, pd, base)
        eng.check()
        ref = [eng.codes(s)[:6].cpu().tolist() for s in range(2)]
        eos = ref[0][3][0]   # below the suppressed band: the logit masks stay the same (see the batch-1 test)
        stop0 = next(i for i in range(4) if ref[0][i][0] == eos)
        stop1 = next((i for i in range(6) if ref[1][i][0] == eos), 6)
        sp = sampling_struct(do_sample=False, min_new_tokens=0, eos_token_id=eos)
        eng.batch_prefill(ed, sp)
        eng.batch_frames(6, td, pd, sp)
        eng.check()
        st = eng.batch_states(2)
        assert st[0][1] == stop0 and st[0][2] == eos
        assert st[1][1] == stop1
        assert eng.codes(0)[:stop0].cpu().tolist() == ref[0][:stop0]
        assert eng.codes(1)[:stop1].cpu().tolist() == ref[1][:stop1]
    finally:
        eng.close()


def test_batch_argument_errors(dev_small):
    eng = Engine(dev_small, max_streams=2, max_seq=64, max_frames=4)
    try:
        e = torch.zeros(8, 1024, dtype=torch.bfloat16, device="cuda")
        with pytest.raises(_lib.QTTError):
            eng.batch_prefill([e, e, e], _greedy_sp())          # more utterances than streams
        with pytest.raises(_lib.QTTError):
            eng.batch_prefill([torch.zeros(64, 1024, dtype=torch.bfloat16, device="cuda")], _greedy_sp())  # >= max_seq
    finally:
        eng.close()
