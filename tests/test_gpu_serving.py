"""Continuous batching on the GPU (``qwentts_turbo_b200.serving``): utterances join freed slots of a
running batch (tensor-core prefill into the slot) and leave at their own frame limits. Each one's
codes must equal the same utterance decoded alone by the batched path with the same Philox
stream, bit for bit, greedy and sampled: an utterance's rows of every GEMM, its norms, its
sampler and its code-predictor attention never mix with other rows, and at these context sizes
(a batch total below 16 positions per warp and KV head) the backbone attention cuts every row
into chunks of 16 positions whatever the batch holds."""
import pytest
import torch

from qwentts_turbo_b200.engine import DeviceModel, Engine, sampling_struct
from qwentts_turbo_b200.serving import ContinuousBatcher, Utterance
from qwentts_turbo_b200.workloads import c3_inputs

pytestmark = pytest.mark.gpu

CTXS = [12, 40, 25, 33, 18, 50, 9]
LIMITS = [3, 7, 2, 5, 4, 3, 6]


@pytest.fixture(scope="module")
def dev_small(small_weights):
    return DeviceModel(small_weights, rope_rows=1024, backbone_layers=2, cp_layers=2)


def _utts():
    out = []
    for i, (c, lim) in enumerate(zip(CTXS, LIMITS)):
        e, t, p = c3_inputs(ctx=c, n_trailing=4, seed=70 + i)
        out.append(Utterance(e.cuda(), t.cuda(), p.cuda(), lim, 1000 + 3 * i))
    return out


def _alone(dev, u, sp):
    eng = Engine(dev, max_streams=1, max_seq=512, max_frames=16)
    try:
        eng.set_stream_params(0, u.philox_stream, u.max_frames)
        eng.prefill_tc(0, u.embeds, sp)
        eng.batch_frames(u.max_frames + 2, [u.trailing], [u.pad], sp)   # the limit stops it
        eng.check()
        n = eng.state(0)["frames"]
        return eng.codes(0)[:n].cpu()
    finally:
        eng.close()


def _continuous(dev, utts, sp, slots, chunk):
    eng = Engine(dev, max_streams=slots, max_seq=512, max_frames=16)
    try:
        cb = ContinuousBatcher(eng, sp, chunk=chunk)
        uids = [cb.submit(u) for u in utts]
        done = cb.run()
        eng.check()
        return [done[i] for i in uids], cb
    finally:
        eng.close()


@pytest.mark.parametrize("sampled", [False, True])
def test_continuous_equals_alone(dev_small, sampled):
    sp = (sampling_struct(do_sample=True, temperature=0.9, top_k=50, repetition_penalty=1.2, min_new_tokens=10_000)
          if sampled else sampling_struct(do_sample=False, repetition_penalty=1.3, min_new_tokens=10_000))
    utts = _utts()
    got, cb = _continuous(dev_small, utts, sp, slots=3, chunk=2)
    assert cb.launches > len(utts)            # slots were refilled while others kept running
    for u, f in zip(utts, got):
        assert f.reason == "limit"
        ref = _alone(dev_small, u, sp)
        assert ref.shape == (u.max_frames, 16)
        assert torch.equal(f.codes.cpu(), ref), (f.uid, f.codes.cpu(), ref)


def test_continuous_independent_of_slot_count_and_chunk(dev_small):
    sp = sampling_struct(do_sample=True, temperature=0.9, top_k=50, repetition_penalty=1.2, min_new_tokens=10_000)
    utts = _utts()
    a, _ = _continuous(dev_small, utts, sp, slots=2, chunk=3)
    b, _ = _continuous(dev_small, utts, sp, slots=4, chunk=1)
    for x, y in zip(a, b):
        assert torch.equal(x.codes.cpu(), y.codes.cpu()), x.uid
