"""NativeTTSGenerator with the API of the reference's ``qwentts_turbo/generator.py``.

The reference's decode loop (generator.py:125-174) runs in Python with ~16 device->host syncs
per frame. Here one call of ``qtt_frames`` runs whole frames on the device: code-predictor
chain (15 weight sweeps), 16-embedding combine, trailing-text add, backbone step, codec head,
suppression, repetition penalty, EOS gate and sampling, then the next frame. The host only
checks for EOS every ``frame_chunk`` frames.

Batches: ``generate`` takes B-leading inputs. B = 1 runs on the batch-1 engine (qtt_frames, one
persistent kernel per frame of one utterance); B > 1 runs all utterances together on the batched
engine (qtt_batch_frames: one launch per frame of up to ``max_batch`` utterances, projections on
tcgen05 tensor cores) through ``serving.ContinuousBatcher``, each utterance with its own Philox
stream (its index b, as a B = 1 call for that utterance would use) and frame limit, stopping at
its own EOS.

Backends: only ``"megakernel"`` (the sm_100a engine) exists; there is no PyTorch/CPU path.
Prefill: the reference runs the HF talker over the context (generator.py:209-225) and copies its
cache into the megakernel (generator.py:245-257). Here ``prefill="tensor_core"`` (default) runs the
context through ``qtt_prefill_tc`` (chunks of up to 128 positions per launch, tcgen05 GEMMs, K/V
written straight into the engine's cache); ``prefill="tokenwise"`` runs it token by token
through the batch-1 decode kernel (same layer math, causal).
"""
from __future__ import annotations

import torch

from . import engine as _engine
from .checkpoint import eos_from_model, load_qwen_tts, weights_from_model
from .config import DEFAULT_DIMS, ModelDims
from .serving import ContinuousBatcher, Utterance

DEFAULT_MODEL_PATH = "Qwen/Qwen3-TTS-12Hz-0.6B-Base"


class NativeTTSGenerator:
    """Frame loop on the device. ``weights`` (dict, see qwentts_turbo_b200.weights) replaces
    checkpoint loading when given; otherwise ``model`` / ``model_path`` as in the reference."""

    def __init__(self, model_path=None, model=None, backend="megakernel", cp_backend="megakernel",
                 weights: dict | None = None, dims: ModelDims = DEFAULT_DIMS, max_seq_len: int = 4096,
                 max_frames: int = 4096, device: int = 0, frame_chunk: int = 32, prefill: str = "tensor_core",
                 max_batch: int = 8):
        if prefill not in ("tensor_core", "tokenwise"):
            raise ValueError("prefill must be 'tensor_core' or 'tokenwise'")
        self.prefill = prefill
        if backend != "megakernel" or cp_backend != "megakernel":
            raise ValueError("qwentts_turbo_b200 only has the sm_100a engine: use backend='megakernel', "
                             "cp_backend='megakernel'")
        self.backend, self.cp_backend = backend, cp_backend
        if weights is None:
            if model is None:
                model = load_qwen_tts(model_path or DEFAULT_MODEL_PATH)
            weights = weights_from_model(model)
            eos = eos_from_model(model, dims.eos_token_id)
            dims = ModelDims(**{**dims.__dict__, "eos_token_id": eos})
        nb = sum(1 for k in weights if k.startswith("talker.layers.") and k.endswith(".q_proj"))
        nc = sum(1 for k in weights if k.startswith("cp.layers.") and k.endswith(".q_proj"))
        self.dims = dims
        self.model = _engine.DeviceModel(weights, dims, device=device, rope_rows=max_seq_len,
                                         backbone_layers=nb, cp_layers=nc)
        self.engine = _engine.Engine(self.model, max_streams=1, max_seq=max_seq_len, max_frames=max_frames)
        self.max_seq_len, self.max_frames = max_seq_len, max_frames
        if not 1 <= max_batch <= 64:
            raise ValueError("max_batch must be in [1, 64]")
        self.max_batch = max_batch
        self._bengine = None   # batched engine, created by the first call with B > 1
        self.eos_token_id = dims.eos_token_id
        self.vocab_size = dims.vocab
        self.frame_chunk = frame_chunk
        self.device = torch.device("cuda", device)

    def generate(self, talker_input_embeds, attention_mask, trailing_text_hidden, tts_pad_embed, max_tokens=500,
                 do_sample=False, temperature=0.9, top_k=50, top_p=1.0, cp_do_sample=False, cp_temperature=0.9,
                 cp_top_k=50, min_new_tokens=2, repetition_penalty=1.0, seed: int = 0, batched: bool | None = None):
        """Arguments as generator.py:77-81 plus ``seed`` (Philox key of the sampler). Inputs may
        carry a leading batch dim B >= 1; each utterance keeps only its attention-mask-valid
        tokens. B > 1 (or ``batched=True``) decodes the utterances together on the batched engine;
        utterance b draws from Philox stream b either way. Returns a list of [16] code lists
        (B = 1) or a list of such lists (B > 1)."""
        if max_tokens > self.engine.max_frames:
            raise ValueError(f"max_tokens {max_tokens} > engine max_frames {self.engine.max_frames}")
        embeds = talker_input_embeds if talker_input_embeds.dim() == 3 else talker_input_embeds.unsqueeze(0)
        B = embeds.shape[0]
        trailing = trailing_text_hidden if trailing_text_hidden.dim() == 3 else trailing_text_hidden.unsqueeze(0)
        pad = tts_pad_embed.reshape(-1, self.dims.hidden)
        items = []
        for b in range(B):
            e = embeds[b]
            if attention_mask is not None:
                m = attention_mask.reshape(B, -1)[b].to(torch.bool).to(e.device)
                e = e[m]
            e = e.to(self.device, torch.bfloat16).contiguous()
            tr = trailing[min(b, trailing.shape[0] - 1)].to(self.device, torch.bfloat16).contiguous()
            pd = pad[min(b, pad.shape[0] - 1)].to(self.device, torch.bfloat16).contiguous()
            items.append((e, tr, pd))

        def sampling(stream):
            return _engine.sampling_struct(do_sample, temperature, top_k, top_p, cp_do_sample, cp_temperature,
                                           cp_top_k, min_new_tokens, repetition_penalty, self.eos_token_id, seed,
                                           philox_stream=stream, dims=self.dims)

        if batched is None:
            batched = B > 1
        if not batched:
            results = [self._run_one(e, tr, pd, sampling(b), max_tokens) for b, (e, tr, pd) in enumerate(items)]
        else:
            results = self._run_batched(items, sampling(0), max_tokens)
        return results[0] if B == 1 else results

    def _batched_engine(self, n: int):
        if self._bengine is None or self._bengine.max_streams < n:
            if self._bengine is not None:
                self._bengine.close()
            self._bengine = _engine.Engine(self.model, max_streams=n, max_seq=self.max_seq_len,
                                           max_frames=self.max_frames)
        return self._bengine

    def _run_batched(self, items, sp, max_tokens):
        """All utterances on the batched engine: up to max_batch at a time in engine streams,
        a freed stream taking the next utterance (continuous batching)."""
        eng = self._batched_engine(min(len(items), self.max_batch))
        cb = ContinuousBatcher(eng, sp, slots=min(len(items), self.max_batch), chunk=max(1, min(self.frame_chunk, max_tokens)),
                               prefill=self.prefill)
        for b, (e, tr, pd) in enumerate(items):
            cb.submit(Utterance(e, tr, pd, max_frames=max_tokens, philox_stream=b))
        done = cb.run()
        eng.check()
        return [done[b].codes.cpu().tolist() for b in range(len(items))]

    def _run_one(self, embeds, trailing, pad, sp, max_tokens):
        eng = self.engine
        if self.prefill == "tensor_core":
            eng.prefill_tc(0, embeds, sp)
        else:
            eng.prefill(0, embeds, sp)
        produced, st = 0, None
        while produced < max_tokens:
            n = min(self.frame_chunk, max_tokens - produced)
            eng.frames(0, n, trailing, pad, sp)
            produced += n
            st = eng.state(0)
            if st["done"]:
                break
        eng.check()
        nfr = st["frames"] if st is not None else 0
        return eng.codes(0)[:nfr].cpu().tolist()
