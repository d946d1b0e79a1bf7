"""Continuous batching of utterances over the batched decode path.

The reference decodes one utterance per ``generate`` call (``generator.py:77-176``): prefill of the
context, then frames until group 0 samples EOS (``generator.py:125-127``) or ``max_new_tokens``
frames were made. Serving many utterances on one GPU, the batched kernel advances up to 64 engine
streams ("slots") per launch, and utterances end at different frames. ``ContinuousBatcher`` keeps
the slots busy: after every chunk of frames it reads all slots' states with one device-to-host
copy, hands out the codes of the utterances that ended, and gives each freed slot the next queued
utterance (tensor-core prefill of its context into that slot) while the other slots keep their
state. Each utterance draws from its own Philox stream and has its own frame limit
(``qtt_set_stream_params``), so its codes do not depend on its slot or on when it joined. Its
arithmetic is its own except in one place: the backbone attention cuts each utterance's context
into chunks of 16 positions until the batch's total context exceeds 16 positions per warp and KV
head, and above that sizes the chunks for the whole batch, which reorders the softmax's partial
sums (a last-bit difference, which can flip a near-tie).
"""
from __future__ import annotations

import collections
import ctypes
from dataclasses import dataclass

import torch


def _with_stream(sp, philox: int):
    """Copy of a qtt_sampling struct with another Philox stream."""
    out = type(sp)()
    ctypes.pointer(out)[0] = sp
    out.philox_stream = philox
    return out


@dataclass
class Utterance:
    """One request: the reference's ``generate`` arguments for one utterance.

    embeds: bf16 [L, 1024] context (``inputs_embeds``); trailing: bf16 [T, 1024] text rows added
    to frames 0..T-1 or None; pad: bf16 [1024] added after them (``tts_pad_embed``); max_frames:
    frame limit (``max_new_tokens``; 0 = the engine's max_frames); philox_stream: Philox stream of
    the utterance's draws (-1: its submission index)."""
    embeds: torch.Tensor
    trailing: torch.Tensor | None
    pad: torch.Tensor
    max_frames: int = 0
    philox_stream: int = -1


@dataclass
class Finished:
    uid: int
    codes: torch.Tensor        # int32 [frames, 16] on the engine's device
    reason: str                # "eos", "limit" or "context" (the KV cache or RoPE table is full)


class ContinuousBatcher:
    """FIFO continuous batching over engine streams 0..slots-1.

    engine: an ``Engine`` (or anything with its batched methods); sampling: the ``qtt_sampling``
    of every launch; chunk: frames per batched call between two state reads (a slot freed inside
    a chunk idles for the rest of it); policy: "continuous" refills a slot as soon as it is free,
    "static" only once every slot is free (request-level batching, the comparison point);
    prefill: "tensor_core" (qtt_prefill_tc, chunks of up to 128 positions per launch) or
    "tokenwise" (qtt_prefill, the batch-1 kernel token by token) for each joining utterance."""

    def __init__(self, engine, sampling, slots: int | None = None, chunk: int = 4, stream=None,
                 policy: str = "continuous", prefill: str = "tensor_core"):
        self.eng = engine
        self.sp = sampling
        self.slots = min(64, engine.max_streams) if slots is None else slots
        if not 1 <= self.slots <= min(64, engine.max_streams):
            raise ValueError(f"slots must be in [1, {min(64, engine.max_streams)}]")
        if chunk < 1:
            raise ValueError("chunk must be >= 1")
        if policy not in ("continuous", "static"):
            raise ValueError("policy must be 'continuous' or 'static'")
        if prefill not in ("tensor_core", "tokenwise"):
            raise ValueError("prefill must be 'tensor_core' or 'tokenwise'")
        self.prefill = prefill
        self.policy = policy
        self.chunk = chunk
        self.stream = stream
        self.queue: collections.deque = collections.deque()
        self.slot_uid = [None] * self.slots       # uid of the utterance in each slot
        self.slot_utt = [None] * self.slots
        self.slot_limit = [0] * self.slots
        self.slot_frames = [0] * self.slots
        self.next_uid = 0
        dev = engine.device
        self._zero_pad = torch.zeros(1024, dtype=torch.bfloat16, device=dev)
        for s in range(self.slots):
            engine.set_stream_params(s, -1, -1)   # parked until an utterance arrives
        self.launches = 0                         # batched frame calls and prefills issued

    def submit(self, utt: Utterance) -> int:
        uid = self.next_uid
        self.next_uid += 1
        self.queue.append((uid, utt))
        return uid

    def busy(self) -> int:
        return sum(u is not None for u in self.slot_uid)

    def pending(self) -> int:
        return len(self.queue) + self.busy()

    def _admit(self, s: int, uid: int, utt: Utterance):
        dev = self.eng.device
        limit = utt.max_frames if utt.max_frames > 0 else self.eng.max_frames
        limit = min(limit, self.eng.max_frames)
        philox = utt.philox_stream if utt.philox_stream >= 0 else uid
        utt = Utterance(utt.embeds.to(dev, torch.bfloat16).contiguous(),
                        None if utt.trailing is None or utt.trailing.shape[0] == 0
                        else utt.trailing.to(dev, torch.bfloat16).contiguous(),
                        utt.pad.to(dev, torch.bfloat16).reshape(1024).contiguous(), limit, philox)
        self.eng.set_stream_params(s, philox, limit)
        if self.prefill == "tensor_core":
            self.eng.prefill_tc(s, utt.embeds, self.sp, self.stream)
        else:   # the first token's draw uses the launch's Philox stream: the utterance's own
            self.eng.prefill(s, utt.embeds, _with_stream(self.sp, philox), self.stream)
        self.launches += 1
        self.slot_uid[s], self.slot_utt[s], self.slot_limit[s], self.slot_frames[s] = uid, utt, limit, -1

    def _release(self, s: int):
        self.eng.set_stream_params(s, -1, -1)
        self.slot_uid[s] = self.slot_utt[s] = None

    def step(self) -> list:
        """Fill free slots from the queue, run one chunk of frames, return the utterances that
        ended (``Finished``)."""
        refill = self.policy == "continuous" or self.busy() == 0
        for s in range(self.slots):
            if not self.queue or not refill:
                break
            if self.slot_uid[s] is None:
                uid, utt = self.queue.popleft()
                self._admit(s, uid, utt)
        occupied = [s for s in range(self.slots) if self.slot_uid[s] is not None]
        if not occupied:
            return []
        B = occupied[-1] + 1
        trailing = [None if self.slot_utt[s] is None else self.slot_utt[s].trailing for s in range(B)]
        pads = [self._zero_pad if self.slot_utt[s] is None else self.slot_utt[s].pad for s in range(B)]
        self.eng.batch_frames(self.chunk, trailing, pads, self.sp, self.stream)
        self.launches += 1
        states = self.eng.batch_states(B, self.stream)
        out = []
        eos = self.sp.eos_token_id
        for s in occupied:
            _, frames, g0, done = states[s]
            reason = None
            if done or g0 == eos:
                reason = "eos"
            elif frames >= self.slot_limit[s]:
                reason = "limit"
            elif frames == self.slot_frames[s]:
                reason = "context"   # no progress over a whole chunk: the stream's cache is full
            self.slot_frames[s] = frames
            if reason is not None:
                out.append(Finished(self.slot_uid[s], self._codes(s, frames), reason))
                self._release(s)
        return out

    def _codes(self, s: int, frames: int) -> torch.Tensor:
        """Copy of slot s's codes, made on the batcher's stream so that it precedes the next
        utterance's frames in that slot."""
        c = self.eng.codes(s)[:frames]
        if self.stream is None:
            return c.clone()
        with torch.cuda.stream(self.stream):
            return c.clone()

    def run(self) -> dict:
        """Decode everything submitted; returns {uid: Finished}."""
        done = {}
        while self.pending():
            for f in self.step():
                done[f.uid] = f
        return done
