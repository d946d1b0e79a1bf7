"""Host logic of the continuous batcher (``qwentts_turbo_b200.serving``) against a fake engine that
follows the batched path's stream contract: a stream makes a frame while it has not reached EOS,
is below its frame limit (``qtt_set_stream_params``; < 0 parks it) and has room in its cache; its
codes depend only on its Philox stream and frame index."""
import torch

from qwentts_turbo_b200.serving import ContinuousBatcher, Utterance

EOS = 2150


class _Sp:
    eos_token_id = EOS


class FakeEngine:
    def __init__(self, max_streams, max_frames=64, max_seq=1000, eos_after=None):
        self.max_streams, self.max_frames, self.max_seq = max_streams, max_frames, max_seq
        self.device = torch.device("cpu")
        self.eos_after = eos_after or {}        # philox stream -> frames before EOS
        self.params = [(-1, 0)] * max_streams
        self.st = [[0, 0, 0, 0] for _ in range(max_streams)]   # position, frames, g0, done
        self.cb = torch.full((max_streams, max_frames, 16), -1, dtype=torch.int32)
        self.philox = [0] * max_streams
        self.frame_calls = []                   # B of every batched frame call
        self.prefills = []

    def _limit(self, s):
        lim = self.params[s][1]
        return 0 if lim < 0 else (min(lim, self.max_frames) if lim > 0 else self.max_frames)

    def set_stream_params(self, s, philox, limit):
        self.params[s] = (philox, limit)

    def prefill_tc(self, s, embeds, sp, stream=None):
        self.philox[s] = self.params[s][0]
        first = EOS if self.eos_after.get(self.philox[s]) == 0 else 7
        self.st[s] = [embeds.shape[0], 0, first, 0]
        self.prefills.append(s)

    def batch_frames(self, n, trailing, pads, sp, stream=None):
        B = len(pads)
        assert len(trailing) == B and all(p is not None for p in pads)
        self.frame_calls.append(B)
        for _ in range(n):
            for s in range(B):
                pos, fr, g0, done = self.st[s]
                if done or g0 == EOS or fr >= self._limit(s) or pos >= self.max_seq - 1:
                    continue
                self.cb[s, fr] = self.philox[s] * 1000 + fr
                fr += 1
                g0 = EOS if self.eos_after.get(self.philox[s]) == fr else 7
                self.st[s] = [pos + 1, fr, g0, int(g0 == EOS)]

    def batch_states(self, B, stream=None):
        return [list(x) for x in self.st[:B]]

    def codes(self, s):
        return self.cb[s]


def _utt(L, limit=0, philox=-1):
    return Utterance(torch.zeros(L, 1024, dtype=torch.bfloat16), None, torch.zeros(1024, dtype=torch.bfloat16),
                     limit, philox)


def _expect(philox, n):
    return (philox * 1000 + torch.arange(n, dtype=torch.int32))[:, None].expand(n, 16)


def test_every_utterance_decoded_with_its_own_limit():
    eng = FakeEngine(3)
    cb = ContinuousBatcher(eng, _Sp(), chunk=4)
    limits = [5, 17, 3, 9, 1, 12, 8]
    uids = [cb.submit(_utt(10 + i, lim)) for i, lim in enumerate(limits)]
    done = cb.run()
    assert sorted(done) == uids
    for uid, lim in zip(uids, limits):
        f = done[uid]
        assert f.reason == "limit"
        assert torch.equal(f.codes, _expect(uid, lim))   # default Philox stream = submission index
    assert len(eng.prefills) == len(limits)
    assert max(eng.frame_calls) <= 3


def test_freed_slots_are_refilled_in_fifo_order():
    eng = FakeEngine(2)
    cb = ContinuousBatcher(eng, _Sp(), chunk=2)
    for lim in (2, 8, 2, 2):
        cb.submit(_utt(5, lim))
    cb.step()                     # uid 0 (slot 0) ends after 2 frames, uid 1 keeps running
    assert cb.slot_uid == [None, 1]
    cb.step()                     # uid 2 takes slot 0
    assert eng.prefills == [0, 1, 0]
    assert cb.slot_uid == [None, 1]
    cb.step()
    assert eng.prefills == [0, 1, 0, 0] and cb.slot_uid[1] == 1


def test_eos_and_explicit_philox_streams():
    eng = FakeEngine(4, eos_after={100: 3, 101: 0, 102: 6})
    cb = ContinuousBatcher(eng, _Sp(), chunk=5)
    a = cb.submit(_utt(4, 0, 100))
    b = cb.submit(_utt(4, 0, 101))   # EOS as the first token: no frames (generator.py breaks at once)
    c = cb.submit(_utt(4, 4, 102))   # the limit comes before EOS
    done = cb.run()
    assert done[a].reason == "eos" and torch.equal(done[a].codes, _expect(100, 3))
    assert done[b].reason == "eos" and done[b].codes.shape == (0, 16)
    assert done[c].reason == "limit" and torch.equal(done[c].codes, _expect(102, 4))


def test_full_context_ends_the_utterance():
    eng = FakeEngine(1, max_seq=12)
    cb = ContinuousBatcher(eng, _Sp(), chunk=3)
    u = cb.submit(_utt(8))
    f = cb.run()[u]
    assert f.reason == "context" and f.codes.shape[0] == 3    # positions 8, 9, 10 fit below max_seq - 1


def test_parked_slots_make_no_frames():
    eng = FakeEngine(4)
    cb = ContinuousBatcher(eng, _Sp(), chunk=2)
    cb.submit(_utt(3, 6))
    cb.run()
    assert all(s[1] == 0 for s in eng.st[1:])
    assert eng.frame_calls and max(eng.frame_calls) == 1    # only slot 0 is passed to the launches


def test_static_policy_waits_for_the_whole_batch():
    eng = FakeEngine(2)
    cb = ContinuousBatcher(eng, _Sp(), chunk=2, policy="static")
    for lim in (2, 6, 2):
        cb.submit(_utt(5, lim))
    cb.step()
    cb.step()                     # slot 0 is free, but uid 1 still runs: no refill
    assert eng.prefills == [0, 1] and cb.slot_uid == [None, 1]
    done = cb.run()
    assert eng.prefills == [0, 1, 0] and torch.equal(done[2].codes, _expect(2, 2))
