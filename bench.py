#!/usr/bin/env python
"""Benchmark of the Qwen3-TTS per-frame decode on B200.

Default workload ("C4"; per GPU of configs[4], "C5"): 64 independent
utterances per GPU decoded together by the batched engine (qtt_batch_frames: one launch per
frame of all 64, projections on tcgen05 tensor cores). Random-init bf16 weights (seed 0
backbone / seed 1 code predictor), prefill contexts ~ U[100, 400] tokens of N(0,1) embeddings,
64 trailing-text rows, temperature 0.9 / top-k 50 / repetition penalty 1.2 with a Philox stream
per utterance, code predictor greedy (the reference's default), EOS masked so that every
utterance decodes the same number of frames. One step = one frame of every utterance.

The batch-1 frame loop ("C3": 200-token context, greedy) is measured too and reported under
"bs1" (``--workload c3`` makes it the headline instead).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--workload c4|c3]

N > 1 runs under torchrun, one rank per GPU, each rank decoding its own utterances (weak
scaling, no collective on the decode path; codes are gathered to rank 0 afterwards). Rank 0
prints one JSON line. ``--impl reference`` times the reference algorithm on the host CPU cores
(the oracle port of the reference's PyTorch path, one utterance at a time).
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "codec_frames_per_s"
UNIT = "frames/s"
CTX = 200
N_TRAILING = 64
FALLBACK_HBM_GBS = 6650.0


CTX_LO, CTX_HI = 100, 400     # C4 prefill contexts
C5_CTX, C5_FRAMES = (100, 600), (200, 600)   # C5 contexts and frame counts per utterance
CTX_MID = (CTX_LO + CTX_HI) // 2


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("c4", "c3", "prefill", "c5"), default="c4")
    ap.add_argument("--batch", type=int, default=64, help="utterances per GPU (c4)")
    ap.add_argument("--bs1-steps", type=int, default=100, help="frames of the batch-1 side measurement (c4)")
    ap.add_argument("--serve-requests", type=int, default=128,
                    help="utterances per GPU of the continuous-batching measurement (c4; 0 = skip)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-c5", action="store_true", help="skip the C5 side measurement (c4)")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="skip the same-GPU timing of the reference's own kernels (oracle/_ref)")
    return ap.parse_args()


def workload_config(args):
    if args.workload == "c5":
        return {
            "workload": f"C5 per GPU: {args.batch} utterances decoded together, contexts U[{C5_CTX[0]},{C5_CTX[1]}], "
                        f"frame counts U[{C5_FRAMES[0]},{C5_FRAMES[1]}] (each utterance stops at its own count), "
                        "T 0.9 / top-k 50 / repetition 1.2 with a Philox stream per utterance, EOS masked",
            "model": "Qwen3-TTS-12Hz-0.6B (random-init bf16)",
            "global_batch": args.gpus * args.batch, "batch_per_gpu": args.batch,
            "ctx": f"U[{C5_CTX[0]},{C5_CTX[1]}]", "seq_len": C5_CTX[1] + C5_FRAMES[1],
            "parallelism": f"data parallel x{args.gpus} (independent utterances)" if args.gpus > 1 else "single GPU",
            "l2": "inputs larger than L2: 3.31 GB of weights + KV streamed per frame (L2 126 MB)",
        }
    if args.workload == "prefill":
        return {
            "workload": f"tensor-core backbone prefill of one {CTX}-position context per step (qtt_prefill_tc: "
                        "chunks of up to 128 positions per launch + the first group-0 token), greedy",
            "model": "Qwen3-TTS-12Hz-0.6B backbone (random-init bf16)",
            "global_batch": args.gpus, "batch_per_gpu": 1, "ctx": CTX, "seq_len": CTX,
            "parallelism": f"replicas x{args.gpus}" if args.gpus > 1 else "single GPU",
            "l2": "inputs larger than L2: 881 MB of backbone weights streamed per launch (L2 126 MB)",
        }
    if args.workload == "c3":
        return {
            "workload": "C3: bs1 frame loop (15-step code predictor + combine + 28-layer backbone step + codec "
                        "head + sampling), 200-token context, 64 trailing rows, greedy, EOS disabled",
            "model": "Qwen3-TTS-12Hz-0.6B (random-init bf16)",
            "global_batch": args.gpus,
            "batch_per_gpu": 1,
            "ctx": CTX,
            "seq_len": CTX + args.warmup + args.steps,
            "parallelism": f"replicas x{args.gpus}" if args.gpus > 1 else "single GPU",
            "l2": "inputs larger than L2: 3.31 GB of weights streamed per frame (L2 126 MB)",
        }
    return {
        "workload": f"C4/C5: {args.batch} utterances per GPU decoded together (one launch per frame of all: "
                    "15-step code predictor + combine + 28-layer backbone + codec head + sampling), prefill "
                    f"ctx ~ U[{CTX_LO},{CTX_HI}], 64 trailing rows, T 0.9 / top-k 50 / repetition 1.2 with a "
                    "Philox stream per utterance, code predictor greedy, EOS masked",
        "model": "Qwen3-TTS-12Hz-0.6B (random-init bf16)",
        "global_batch": args.gpus * args.batch,
        "batch_per_gpu": args.batch,
        "ctx": f"U[{CTX_LO},{CTX_HI}]",
        "seq_len": CTX_HI + args.warmup + args.steps,
        "parallelism": f"data parallel x{args.gpus} (independent utterances)" if args.gpus > 1 else "single GPU",
        "l2": "inputs larger than L2: 3.31 GB of weights + KV streamed per frame (L2 126 MB)",
    }


# ------------------------------------------------------------------------------------------
# clocks sampled with nvidia-smi during the timed region
# ------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: int):
        self.samples = []
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            sel = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.proc = subprocess.Popen(["nvidia-smi", "-i", sel, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                self.samples.append((time.time(), float(parts[0]), float(parts[1]),
                                     [n for n, v in zip(self.NAMES, parts[3:7]) if v.lower() == "active"]))
            except ValueError:
                pass

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0: float, t1: float):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        win = [s for s in self.samples if t0 <= s[0] <= t1]
        if not win:  # short timed region: take the samples closest to it
            win = sorted(self.samples, key=lambda s: min(abs(s[0] - t0), abs(s[0] - t1)))[:3]
        reasons = sorted({r for s in win for r in s[3]})
        return {"sm_mhz": statistics.median(s[1] for s in win), "sm_max_mhz": max(s[2] for s in win),
                "reasons": reasons, "samples": len(win)}


# ------------------------------------------------------------------------------------------
def measured_hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic_per_frame(algorithmic_bytes, name="qtt_decode_kernel_frame_c3.txt"):
    """DRAM bytes per launch of this run: the DRAM / algorithmic ratio of the committed ncu capture
    (one frame launch at an early position) times this run's algorithmic bytes per launch, since
    the KV part grows with the position. None when the summary is absent."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("dram_over_algorithmic:"):
                    return float(line.split(":", 1)[1].split()[0]) * algorithmic_bytes
    except OSError:
        pass
    return None


def cpu_frames_per_s(seconds: float, warmup: int = 1, max_frames: int | None = None, seed: int = 4,
                     sampled: bool = False, ctx: int = CTX):
    """Oracle (CPU port of the reference path) frames/s, all host threads: the C3 loop, or with
    ``sampled`` the C4 per-utterance loop (T 0.9 / top-k 50 / repetition 1.2, Philox draws)."""
    from oracle.qtt_oracle import Qwen3TTSOracle
    from qwentts_turbo_b200.weights import synthetic_weights
    from qwentts_turbo_b200.workloads import c3_inputs
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    w = synthetic_weights()
    embeds, trailing, pad = c3_inputs(ctx, N_TRAILING, seed)
    orc = Qwen3TTSOracle(w, max_seq=ctx + 2048)
    del w
    # the oracle's generate() loop, frame by frame, with a time budget
    from oracle import qtt_oracle as O
    eos = orc.d.eos_token_id
    sup = orc.suppress_mask(eos)
    h = orc.prefill(embeds)
    logits = orc.head_logits(orc.codec_head, h)
    logits[sup] = float("-inf")
    g0 = O.sample_token(logits, False, 0.9, 50, 1.0, eos)
    hist = [g0]
    t_start = None
    timed = 0
    step = 0
    while True:
        if step == warmup:
            t_start = time.perf_counter()
        toks, _ = orc.cp_chain(h, g0)
        groups = [g0] + toks
        extra = trailing[step] if step < trailing.shape[0] else pad
        h = orc.backbone_step(orc.combine(groups, extra))
        logits = orc.head_logits(orc.codec_head, h)
        logits[sup] = float("-inf")
        if sampled:
            logits = O.apply_repetition_penalty(logits, hist, 1.2)
            g0 = O.sample_token(logits, True, 0.9, 50, 1.0, eos, O.draw_u24(1234, step + 1, 0, 0))
        else:
            g0 = O.sample_token(logits, False, 0.9, 50, 1.0, None)
        hist.append(g0)
        step += 1
        if t_start is not None:
            timed += 1
            el = time.perf_counter() - t_start
            if el >= seconds or (max_frames is not None and timed >= max_frames):
                break
    el = time.perf_counter() - t_start
    return timed / el, cores, timed, el


def ref_gpu_baseline(dev: int, ctx: int = CTX, frames: int = 20, warmup: int = 3):
    """Same-GPU baseline leg, outside the product's timed regions: the reference's own decode
    kernels (fused_decode_tts.cu:834-890, fused_decode_code_predictor.cu:674-730), compiled from
    its sources into oracle/_ref by oracle/Makefile, on the C3 workload's shapes and the same
    random-init weights. Per frame one backbone step at position ctx + f and 15 code-predictor
    steps at positions 0..14, timed with CUDA events on this GPU. Kernels only: the reference's
    PyTorch code-predictor prefill, its 16 head GEMVs, sampling and combine glue are not counted,
    so the result is a lower bound of the reference's frame time. None when oracle/_ref is absent."""
    from oracle import ref_kernels
    if not ref_kernels.available():
        return None
    from qwentts_turbo_b200.megakernel_backbone import extract_backbone_weights
    from qwentts_turbo_b200.megakernel_code_predictor import extract_code_predictor_weights
    from qwentts_turbo_b200.weights import synthetic_weights
    torch.cuda.set_device(dev)
    w = synthetic_weights()
    max_seq = ctx + warmup + frames + 8
    bw = extract_backbone_weights(w, max_seq)
    cw = extract_code_predictor_weights(w, 64)
    del w
    tts = ref_kernels.RefDecoder("tts", bw["layer_weights"], bw["final_norm_weight"], bw["cos_table"],
                                 bw["sin_table"], bw["num_layers"], max_seq)
    cp = ref_kernels.RefDecoder("cp", cw["layer_weights"], cw["final_norm_weight"], cw["cos_table"],
                                cw["sin_table"], cw["num_layers"], 64)
    g = torch.Generator().manual_seed(4)
    tts.k[:, :, :ctx] = torch.randn(tts.k[:, :, :ctx].shape, generator=g).to(torch.bfloat16).cuda()
    tts.v[:, :, :ctx] = torch.randn(tts.v[:, :, :ctx].shape, generator=g).to(torch.bfloat16).cuda()
    x = torch.randn(1024, generator=g).to(torch.bfloat16).cuda()
    tts.position = ctx
    stream = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    bb_ms, cp_ms = [], []
    for f in range(warmup + frames):
        ev[0].record(stream)
        tts.step(x)
        ev[1].record(stream)
        cp.position = 0
        for _ in range(15):
            cp.step(x)
        ev[2].record(stream)
        torch.cuda.synchronize()
        if f >= warmup:
            bb_ms.append(ev[0].elapsed_time(ev[1]))
            cp_ms.append(ev[1].elapsed_time(ev[2]))
    b, c = statistics.median(bb_ms), statistics.median(cp_ms)
    return {"frame_ms": b + c, "backbone_step_ms": b, "cp_15_steps_ms": c, "frames": frames,
            "what": "the reference's own CUDA kernels (oracle/_ref, built from its sources for sm_100a) on this "
                    "GPU: one 28-layer backbone step at the C3 positions + 15 code-predictor steps per frame, "
                    "median of the timed frames; kernels only (its PyTorch prefill, heads, sampling and combine "
                    "glue excluded), a lower bound of its frame time"}


# ------------------------------------------------------------------------------------------
def cpu_sample_text(c4, timed, el, cores):
    if c4:
        return (f"{timed} frames of one utterance of the C4 loop (sampled, repetition 1.2) after a {CTX_MID}-token "
                f"prefill, the mean C4 context ({el:.1f} s, fp32 torch oracle on {cores} host threads; the CPU path "
                "decodes one utterance at a time, so its frames/s does not depend on the batch)")
    return (f"{timed} frames of the C3 loop after a {CTX}-token prefill ({el:.1f} s, fp32 torch oracle on "
            f"{cores} host threads)")


def run_reference(args, rank):
    if rank != 0:
        return
    budget = 60.0
    c4 = args.workload == "c4"
    fps, cores, timed, el = cpu_frames_per_s(budget, warmup=args.warmup, max_frames=args.steps,
                                             sampled=c4, ctx=CTX_MID if c4 else CTX)
    line = {
        "impl": "reference", "metric": METRIC, "value": fps, "unit": UNIT, "n_gpus": args.gpus, "steps": timed,
        "warmup": args.warmup, "ms_per_step": 1000.0 * el / timed, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args),
        "cpu_baseline": {"value": fps, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": cpu_sample_text(c4, timed, el, cores)},
        "e2e": {"value": fps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_c3(args, rank, world, local_rank, K, W):
    """Batch-1 frame loop; returns rank 0's JSON fields (None on other ranks)."""
    import torch.distributed as dist

    from qwentts_turbo_b200 import _lib
    from qwentts_turbo_b200.config import frame_weight_bytes, kv_read_bytes_per_frame
    from qwentts_turbo_b200.dist import gather_codes, max_over_ranks
    from qwentts_turbo_b200.engine import DeviceModel, Engine, sampling_struct
    from qwentts_turbo_b200.weights import synthetic_weights
    from qwentts_turbo_b200.workloads import c3_inputs

    dev = local_rank
    torch.cuda.set_device(dev)
    max_seq = CTX + W + K + 8
    weights = synthetic_weights()
    dm = DeviceModel(weights, device=dev, rope_rows=max_seq)
    del weights
    eng = Engine(dm, max_streams=1, max_seq=max_seq, max_frames=W + K + 1)
    embeds, trailing, pad = c3_inputs(CTX, N_TRAILING, seed=4 + rank)
    embeds_d, trailing_d, pad_d = embeds.cuda(), trailing.cuda(), pad.cuda()
    sp = sampling_struct(do_sample=False, min_new_tokens=1 << 30)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()


    # ---- device-resident run: inputs already in HBM --------------------------------------
    eng.prefill(0, embeds_d, sp)
    eng.frames(0, W, trailing_d, pad_d, sp)
    eng.check()
    clocks = ClockSampler(dev)
    time.sleep(0.3)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    e0.record(stream)
    eng.frames(0, K, trailing_d, pad_d, sp)
    e1.record(stream)
    barrier()
    t1 = time.time()
    ms = max_over_ranks(e0.elapsed_time(e1))
    clocks.stop()
    eng.check()
    st = eng.state(0)
    assert st["frames"] == W + K and st["done"] == 0, st
    codes = eng.codes(0)[: W + K].clone()

    # ---- end to end through the C-ABI with host buffers ---------------------------------
    lib = _lib.load()
    trailing_h = trailing.pin_memory()
    pad_h = pad.pin_memory()
    row_d = torch.empty(1024, dtype=torch.bfloat16, device="cuda")
    codes_dev = eng.codes(0)
    codes_h = torch.empty(K, 16, dtype=torch.int32).pin_memory()
    sh = stream.cuda_stream
    spb = ctypes.byref(sp)

    def e2e_frame(step, out_row):
        src = trailing_h[step] if step < N_TRAILING else pad_h
        row_d.copy_(src, non_blocking=True)
        rc = lib.qtt_frames(eng.h, 0, 1, None, 0, row_d.data_ptr(), spb, sh)
        if rc != 0:
            raise _lib.QTTError(rc, "qtt_frames")
        if out_row is not None:
            out_row.copy_(codes_dev[step], non_blocking=True)

    eng.prefill(0, embeds_d, sp)
    for s in range(W):
        e2e_frame(s, None)
    eng.check()
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for f in range(K):
        e2e_frame(W + f, codes_h[f])
    e3.record(stream)
    barrier()
    ms_e2e = max_over_ranks(e2.elapsed_time(e3))
    eng.check()
    assert torch.equal(codes_h, codes[W:].cpu()), "e2e path produced different codes"

    # ---- gather codes to rank 0 (after timing; NCCL over NVLink) ---------------------------
    gathered = gather_codes(codes)
    n_codes = sum(g.shape[0] for g in gathered) if gathered is not None else 0

    if rank != 0:
        eng.close()
        return None
    eng.close()
    ref_gpu = None if args.no_ref_gpu else ref_gpu_baseline(dev)

    # ---- roofline -------------------------------------------------------------------------
    wbytes = frame_weight_bytes()
    kvb = [kv_read_bytes_per_frame(CTX + W + f) for f in range(K)]
    bytes_per_frame = wbytes + sum(kvb) / K
    frame_s = ms / 1000.0 / K
    achieved = bytes_per_frame / frame_s / 1e9
    peak, peak_src = measured_hbm_peak()
    traffic = ncu_traffic_per_frame(bytes_per_frame)
    value = world * K / (ms / 1000.0)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (random-init weights, seeded N(0,1) inputs)",
        "config": workload_config(args),
        "frame_latency_us": 1000.0 * ms / K,
        "rtf": (ms / K) / (1000.0 / 12.0),
        "hbm_gbs": achieved,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_src, "traffic": traffic,
                     "algorithmic_bytes_per_launch": bytes_per_frame,
                     "kernel": "qtt_decode_kernel (1 launch per frame)"},
        "e2e": {"value": world * K / (ms_e2e / 1000.0), "unit": UNIT, "h2d_bytes_per_step": 2048,
                "d2h_bytes_per_step": 64,
                "path": "qtt_frames C-ABI per frame: pinned H2D of the frame's text row, D2H of its 16 codes"},
        "gpu_launches": K,
        "clocks": clocks.summary(t0, t1),
        "codes_gathered": n_codes,
        "ref_gpu_baseline": ref_gpu,
    }
    return line


def run_c4(args, rank, world, local_rank, K, W):
    """Batched frame loop of args.batch utterances per GPU; returns rank 0's JSON fields."""
    import torch.distributed as dist

    from qwentts_turbo_b200 import _lib
    from qwentts_turbo_b200.config import frame_weight_bytes, kv_read_bytes_per_frame
    from qwentts_turbo_b200.dist import gather_codes, max_over_ranks
    from qwentts_turbo_b200.engine import DeviceModel, Engine, sampling_struct
    from qwentts_turbo_b200.weights import synthetic_weights
    from qwentts_turbo_b200.workloads import c4_inputs

    dev = local_rank
    torch.cuda.set_device(dev)
    B = args.batch
    max_seq = CTX_HI + W + K + 8
    weights = synthetic_weights()
    dm = DeviceModel(weights, device=dev, rope_rows=max_seq)
    del weights
    eng = Engine(dm, max_streams=B, max_seq=max_seq, max_frames=W + K + 1)
    ctx, embeds, trailing, pads = c4_inputs(B, CTX_LO, CTX_HI, N_TRAILING, seed=4 + rank)
    embeds_d = [e.cuda() for e in embeds]
    trailing_d = [t.cuda() for t in trailing]
    pads_d = [x.cuda() for x in pads]
    sp = sampling_struct(do_sample=True, temperature=0.9, top_k=50, repetition_penalty=1.2,
                         min_new_tokens=1 << 30, seed=1234 + rank)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident run: inputs already in HBM --------------------------------------
    eng.batch_prefill(embeds_d, sp)
    eng.batch_frames(W, trailing_d, pads_d, sp)
    eng.check()
    clocks = ClockSampler(dev)
    time.sleep(0.3)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    e0.record(stream)
    eng.batch_frames(K, trailing_d, pads_d, sp)
    e1.record(stream)
    barrier()
    t1 = time.time()
    ms = max_over_ranks(e0.elapsed_time(e1))
    clocks.stop()
    eng.check()
    for s in range(B):
        st = eng.state(s)
        assert st["frames"] == W + K and st["done"] == 0, (s, st)
    codes = torch.stack([eng.codes(s)[: W + K].clone() for s in range(B)])   # [B, W+K, 16]

    # ---- end to end through the C-ABI with host buffers: per frame the B text rows H2D from
    # pinned memory, one qtt_batch_frames call, the B code rows D2H ------------------------
    lib = _lib.load()
    rows_h = torch.empty(K, B, 1024, dtype=torch.bfloat16).pin_memory()
    for f in range(K):
        for s in range(B):
            step = W + f
            rows_h[f, s] = trailing[s][step] if step < N_TRAILING else pads[s]
    rows_d = torch.empty(B, 1024, dtype=torch.bfloat16, device="cuda")
    codes_devs = [eng.codes(s) for s in range(B)]
    codes_h = torch.empty(K, B, 16, dtype=torch.int32).pin_memory()
    frame_codes_d = torch.empty(B, 16, dtype=torch.int32, device="cuda")
    sh = stream.cuda_stream
    spb = ctypes.byref(sp)
    no_trail = (ctypes.c_void_p * B)()
    zeros = (ctypes.c_int * B)(*([0] * B))
    row_ptrs = (ctypes.c_void_p * B)(*[rows_d[s].data_ptr() for s in range(B)])

    eng.batch_prefill(embeds_d, sp)
    eng.batch_frames(W, trailing_d, pads_d, sp)
    eng.check()
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for f in range(K):
        rows_d.copy_(rows_h[f], non_blocking=True)
        rc = lib.qtt_batch_frames(eng.h, B, 1, no_trail, zeros, row_ptrs, spb, sh)
        if rc != 0:
            raise _lib.QTTError(rc, "qtt_batch_frames")
        # the frame's codes of all B utterances: one gather (qtt_batch_last_codes), one D2H copy
        rc = lib.qtt_batch_last_codes(eng.h, B, frame_codes_d.data_ptr(), sh)
        if rc != 0:
            raise _lib.QTTError(rc, "qtt_batch_last_codes")
        codes_h[f].copy_(frame_codes_d, non_blocking=True)
    # the run's codes of every rank to rank 0 (NCCL all-gather over NVLink; one rank: a copy)
    gathered = gather_codes(torch.stack([codes_devs[s][W:W + K] for s in range(B)]).reshape(-1, 16))
    e3.record(stream)
    barrier()
    ms_e2e = max_over_ranks(e2.elapsed_time(e3))
    eng.check()
    assert torch.equal(codes_h, codes[:, W:].permute(1, 0, 2).cpu()), "e2e path produced different codes"
    n_codes = sum(x.shape[0] for x in gathered) if gathered is not None else 0
    if rank != 0:
        eng.close()
        return None

    # ---- roofline: weights once per frame for the batch + every utterance's KV ----------
    wbytes = frame_weight_bytes()
    kv = sum(kv_read_bytes_per_frame(ctx[s] + W + f) for s in range(B) for f in range(K)) / K
    bytes_per_frame = wbytes + kv
    frame_s = ms / 1000.0 / K
    achieved = bytes_per_frame / frame_s / 1e9
    peak, peak_src = measured_hbm_peak()
    # tensor work: every weight element meets every token's hi and lo operand (2 x 2 FLOP)
    tflops = 4.0 * (wbytes / 2) * B / frame_s / 1e12
    bstream_bytes = 80   # sizeof(qtt::BStream), copied H2D by every qtt_batch_frames call
    line = {
        "metric": METRIC, "value": world * B * K / (ms / 1000.0), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (random-init weights, seeded N(0,1) inputs)",
        "config": workload_config(args),
        "frames_per_s_per_gpu": B * K / (ms / 1000.0),
        "batch_frame_ms": ms / K,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_src, "traffic": ncu_traffic_per_frame(bytes_per_frame, "qtt_batch_kernel_frame_c4.txt"),
                     "algorithmic_bytes_per_launch": bytes_per_frame,
                     "tensor_tflops": tflops,
                     "kernel": "qtt_batch_kernel (1 launch per frame of all utterances)"},
        "e2e": {"value": world * B * K / (ms_e2e / 1000.0), "unit": UNIT,
                "h2d_bytes_per_step": B * 2048 + B * bstream_bytes, "d2h_bytes_per_step": B * 64,
                "path": "qtt_batch_frames C-ABI per frame: pinned H2D of the B text rows; the B code rows gathered "
                        "by qtt_batch_last_codes and read back with one D2H copy; "
                        "the run's codes of all ranks gathered to rank 0 at the end (NCCL all-gather)"},
        "gpu_launches": K,
        "clocks": clocks.summary(t0, t1),
        "codes_gathered": n_codes,
    }
    eng.close()
    return line


def run_serving(args, rank, world, local_rank):
    """Continuous batching (qwentts_turbo_b200.serving) of args.serve_requests utterances per GPU
    with uneven lengths (contexts U[CTX_LO, CTX_HI], frame limits U[50, 300], sampled as C4) on
    args.batch slots, against static batching of the same utterances (a batch is refilled only
    once all of its utterances ended). Every joining utterance is prefilled with the tensor-core
    prefill in its slot; the device-timed region covers the prefills, the frames and the host's
    scheduling between chunks. Returns useful codec frames/s (whole job) of both policies."""
    import torch.distributed as dist

    from qwentts_turbo_b200.dist import max_over_ranks
    from qwentts_turbo_b200.engine import DeviceModel, Engine, sampling_struct
    from qwentts_turbo_b200.serving import ContinuousBatcher, Utterance
    from qwentts_turbo_b200.weights import synthetic_weights

    dev = local_rank
    torch.cuda.set_device(dev)
    n, B, chunk = args.serve_requests, args.batch, 4
    lim_lo, lim_hi = 50, 300
    max_seq = CTX_HI + lim_hi + 8
    dm = DeviceModel(synthetic_weights(), device=dev, rope_rows=max_seq)
    eng = Engine(dm, max_streams=B, max_seq=max_seq, max_frames=lim_hi)
    g = torch.Generator().manual_seed(40 + rank)
    ctx = torch.randint(CTX_LO, CTX_HI + 1, (n,), generator=g).tolist()
    lims = torch.randint(lim_lo, lim_hi + 1, (n,), generator=g).tolist()
    utts = [Utterance(torch.randn(L, 1024, generator=g).to(torch.bfloat16).cuda(),
                      torch.randn(N_TRAILING, 1024, generator=g).to(torch.bfloat16).cuda(),
                      torch.randn(1024, generator=g).to(torch.bfloat16).cuda(), lim, 100_000 * rank + i)
            for i, (L, lim) in enumerate(zip(ctx, lims))]
    sp = sampling_struct(do_sample=True, temperature=0.9, top_k=50, repetition_penalty=1.2,
                         min_new_tokens=1 << 30, seed=1234 + rank)
    stream = torch.cuda.current_stream()

    def timed(policy, items):
        cb = ContinuousBatcher(eng, sp, slots=B, chunk=chunk, policy=policy)
        for u in items:
            cb.submit(u)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        done = cb.run()
        e1.record(stream)
        torch.cuda.synchronize()
        eng.check()
        frames = sum(f.codes.shape[0] for f in done.values())
        assert frames == sum(u.max_frames for u in items), "an utterance ended before its frame limit"
        return max_over_ranks(e0.elapsed_time(e1)), frames, cb.launches

    timed("continuous", utts[:min(n, 8)])      # warm-up (first launches, allocations)
    ms_c, frames, launches_c = timed("continuous", utts)
    ms_s, _, launches_s = timed("static", utts)
    eng.close()
    if rank != 0:
        return None
    return {"workload": f"{n} utterances per GPU, contexts U[{CTX_LO},{CTX_HI}], frame limits U[{lim_lo},{lim_hi}], "
                        f"sampled (T 0.9, top-k 50, repetition 1.2), {B} slots, {chunk} frames per state read",
            "frames": frames * world, "continuous_frames_per_s": world * frames / (ms_c / 1000.0),
            "static_frames_per_s": world * frames / (ms_s / 1000.0), "continuous_s": ms_c / 1000.0,
            "static_s": ms_s / 1000.0, "calls_continuous": launches_c, "calls_static": launches_s,
            "prefill": "qtt_prefill_tc of each joining utterance in its slot (inside the timed region)"}


def run_prefill(args, rank, world, local_rank, K, W):
    """Tensor-core prefill (qtt_prefill_tc) of a CTX-position context, one utterance per step;
    returns rank 0's JSON fields (metric: context positions per second)."""
    import torch.distributed as dist

    from qwentts_turbo_b200.config import DEFAULT_DIMS
    from qwentts_turbo_b200.dist import max_over_ranks
    from qwentts_turbo_b200.engine import DeviceModel, Engine, sampling_struct
    from qwentts_turbo_b200.weights import synthetic_weights
    from qwentts_turbo_b200.workloads import c3_inputs

    dev = local_rank
    torch.cuda.set_device(dev)
    L = CTX
    dm = DeviceModel(synthetic_weights(), device=dev, rope_rows=L + 16)
    eng = Engine(dm, max_streams=1, max_seq=L + 16, max_frames=4)
    embeds, _, _ = c3_inputs(L, 1, 4 + rank)
    emb_h = embeds.pin_memory()
    emb_d = embeds.cuda()
    sp = sampling_struct(do_sample=False, min_new_tokens=100)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(W):
        eng.prefill_tc(0, emb_d, sp)
    eng.check()
    ref_g0 = eng.state(0)["g0"]
    clocks = ClockSampler(dev)
    time.sleep(0.3)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    e0.record(stream)
    for _ in range(K):
        eng.prefill_tc(0, emb_d, sp)
    e1.record(stream)
    barrier()
    t1 = time.time()
    ms = max_over_ranks(e0.elapsed_time(e1))
    clocks.stop()
    eng.check()
    # end to end: the context from pinned host memory, the prefill, the first token read back
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(K):
        emb_d.copy_(emb_h, non_blocking=True)
        eng.prefill_tc(0, emb_d, sp, stream)
        assert eng.state(0, stream)["g0"] == ref_g0, "e2e prefill gave another first token"
    e3.record(stream)
    barrier()
    ms_e2e = max_over_ranks(e2.elapsed_time(e3))
    eng.close()
    if rank != 0:
        return None
    d = DEFAULT_DIMS
    row = 2 * 2 * d.n_kv_heads * d.head_dim * d.backbone_layers    # bf16 K + V of one position, all layers
    wb = d.backbone_layers * d.layer_bytes() + 2 * d.hidden         # backbone layers + final norm
    chunks = [(p0, min(128, L - p0)) for p0 in range(0, L, 128)]
    # per chunk launch: the weights once, the chunk's embeddings, its K/V rows written and the
    # cache rows [0, p0 + T) read once
    alg = [wb + T * 2 * d.hidden + T * row + (p0 + T) * row for p0, T in chunks]
    step_s = ms / 1000.0 / K
    achieved = sum(alg) / step_s / 1e9    # over the whole step (head launch and resets included)
    peak, peak_src = measured_hbm_peak()
    flops = sum(4.0 * (wb / 2) * T for _, T in chunks)   # hi and lo operand planes
    return {
        "metric": "prefill_positions_per_s", "value": world * L * K / (ms / 1000.0), "unit": "positions/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights, seeded N(0,1) context)", "config": workload_config(args),
        "prefill_ms_per_utterance": ms / K,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_src,
                     "traffic": ncu_traffic_per_frame(sum(alg) / len(alg), "qtt_batch_kernel_prefill_dense.txt"),
                     "algorithmic_bytes_per_launch": sum(alg) / len(alg),
                     "launches_per_step": len(chunks) + 1, "tensor_tflops": flops / step_s / 1e12,
                     "kernel": "qtt_batch_kernel, dense prefill program (achieved over the whole step: "
                               "the first-token launch and the stream reset are included)"},
        "e2e": {"value": world * L * K / (ms_e2e / 1000.0), "unit": "positions/s",
                "h2d_bytes_per_step": L * 2 * d.hidden + 80, "d2h_bytes_per_step": 16,
                "path": "pinned H2D of the context, qtt_prefill_tc, qtt_get_state (first token)"},
        "gpu_launches": K * (len(chunks) + 1),
        "clocks": clocks.summary(t0, t1),
    }


def run_c5(args, rank, world, local_rank):
    """C5 on each GPU: args.batch utterances with their own context
    lengths U[100,600] and frame counts U[200,600], decoded together until the last one reaches its
    count (the kernel stops each utterance at its own count, qtt_set_stream_params). One job per
    rank, timed on the device in three parts with CUDA events:
      prefill  contexts, text rows and pad rows H2D from pinned host memory + the tensor-core
               prefill of every utterance (qtt_prefill_tc into its stream),
      frames   one qtt_batch_frames call of max(count) frames,
      gather   every utterance's codes to rank 0 (NCCL all-gather over NVLink) and D2H there.
    value = useful frames of all ranks (the sum of the counts) / max over ranks of the frames part;
    e2e = the same frames / max over ranks of the whole job. Returns rank 0's fields."""
    import torch.distributed as dist

    from qwentts_turbo_b200.config import frame_weight_bytes, kv_read_bytes_per_frame
    from qwentts_turbo_b200.dist import gather_codes, max_over_ranks
    from qwentts_turbo_b200.engine import DeviceModel, Engine, sampling_struct
    from qwentts_turbo_b200.weights import synthetic_weights
    from qwentts_turbo_b200.workloads import c4_inputs

    dev = local_rank
    torch.cuda.set_device(dev)
    B = args.batch
    max_seq = C5_CTX[1] + C5_FRAMES[1] + 8
    dm = DeviceModel(synthetic_weights(), device=dev, rope_rows=max_seq)
    eng = Engine(dm, max_streams=B, max_seq=max_seq, max_frames=C5_FRAMES[1])
    ctx, embeds, trailing, pads = c4_inputs(B, C5_CTX[0], C5_CTX[1], N_TRAILING, seed=500 + rank)
    g = torch.Generator().manual_seed(600 + rank)
    counts = torch.randint(C5_FRAMES[0], C5_FRAMES[1] + 1, (B,), generator=g).tolist()
    # pinned host inputs and their device buffers (allocated before the timed region)
    emb_h = [e.pin_memory() for e in embeds]
    tr_h = [t.pin_memory() for t in trailing]
    pad_h = [x.pin_memory() for x in pads]
    emb_d = [torch.empty_like(e, device="cuda") for e in embeds]
    tr_d = [torch.empty_like(t, device="cuda") for t in trailing]
    pad_d = [torch.empty_like(x, device="cuda") for x in pads]
    sp = sampling_struct(do_sample=True, temperature=0.9, top_k=50, repetition_penalty=1.2,
                         min_new_tokens=1 << 30, seed=1234 + rank)
    stream = torch.cuda.current_stream()

    def job(n_frames=None):
        for a, b in zip(emb_d + tr_d + pad_d, emb_h + tr_h + pad_h):
            a.copy_(b, non_blocking=True)
        for s in range(B):
            eng.set_stream_params(s, 1000 * rank + s, counts[s])
            eng.prefill_tc(s, emb_d[s], sp)
        ev[1].record(stream)
        eng.batch_frames(max(counts) if n_frames is None else n_frames, tr_d, pad_d, sp)
        ev[2].record(stream)
        codes = torch.cat([eng.codes(s)[:counts[s]] for s in range(B)])
        got = gather_codes(codes)
        if got is not None:
            got = [x.cpu() for x in got]
        return got

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    job(args.warmup)      # warm-up: the same launches, a few frames
    eng.check()
    clocks = ClockSampler(dev)
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.time()
    ev[0].record(stream)
    got = job()
    ev[3].record(stream)
    torch.cuda.synchronize()
    t1 = time.time()
    clocks.stop()
    eng.check()
    st = eng.batch_states(B)
    assert [x[1] for x in st] == counts, "an utterance did not reach its frame count"
    t_pre = max_over_ranks(ev[0].elapsed_time(ev[1]))
    t_fr_local = ev[1].elapsed_time(ev[2])
    t_fr = max_over_ranks(t_fr_local)
    t_all = max_over_ranks(ev[0].elapsed_time(ev[3]))
    frames_local = sum(counts)
    frames_all = frames_local
    if world > 1:
        x = torch.tensor([frames_local], dtype=torch.int64, device="cuda")
        dist.all_reduce(x)
        frames_all = int(x.item())
    eng.close()
    if rank != 0:
        return None
    assert sum(c.shape[0] for c in got) == frames_all, "gathered codes"
    launches = max(counts)
    wbytes = frame_weight_bytes()
    kv = sum(kv_read_bytes_per_frame(ctx[s] + f) for s in range(B) for f in range(counts[s]))
    alg = (launches * wbytes + kv) / launches
    achieved = alg / (t_fr_local / 1000.0 / launches) / 1e9
    peak, peak_src = measured_hbm_peak()
    h2d = sum(2 * 1024 * (c + N_TRAILING + 1) for c in ctx) + 80 * B
    return {
        "workload": f"C5 per GPU: {B} utterances decoded together, contexts U[{C5_CTX[0]},{C5_CTX[1]}], frame counts "
                    f"U[{C5_FRAMES[0]},{C5_FRAMES[1]}] (each stops at its own count), T 0.9 / top-k 50 / repetition "
                    "1.2 with a Philox stream per utterance, EOS masked; codes gathered to rank 0",
        "metric": METRIC, "value": frames_all / (t_fr / 1000.0), "unit": UNIT, "n_gpus": world,
        "frames": frames_all, "launches_per_gpu": launches, "occupancy": frames_local / (B * launches),
        "ms_per_launch": t_fr / launches,
        "e2e": {"value": frames_all / (t_all / 1000.0), "unit": UNIT, "prefill_ms": t_pre, "frames_ms": t_fr,
                "job_ms": t_all, "h2d_bytes_per_gpu": h2d, "d2h_bytes": frames_all * 64,
                "path": "pinned H2D of every input, qtt_prefill_tc per utterance, one qtt_batch_frames call, NCCL "
                        "all-gather of the codes to rank 0 and D2H there"},
        "limiter": "the batch drains: a launch costs the same with fewer utterances running (the frame is "
                   "latency-bound), so useful frames per launch fall as utterances reach their counts; the "
                   "gather is a few MB over NVLink",
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_src, "algorithmic_bytes_per_launch": alg},
        "clocks": clocks.summary(t0, t1),
    }


def run_ours(args, rank, world, local_rank):
    if args.workload == "c5":
        c5 = run_c5(args, rank, world, local_rank)
        if c5 is not None:
            line = {k: c5[k] for k in ("metric", "value", "unit", "n_gpus")}
            line.update({"steps": c5["launches_per_gpu"], "warmup": args.warmup, "ms_per_step": c5["ms_per_launch"],
                         "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                         "data": "synthetic (random-init weights, seeded N(0,1) inputs)",
                         "config": workload_config(args), "e2e": c5["e2e"], "roofline": c5["roofline"],
                         "gpu_launches": c5["launches_per_gpu"] + args.batch * 2, "clocks": c5["clocks"],
                         "occupancy": c5["occupancy"], "limiter": c5["limiter"]})
            print(json.dumps(line), flush=True)
        return
    if args.workload == "prefill":
        line = run_prefill(args, rank, world, local_rank, args.steps, args.warmup)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if args.workload == "c3":
        line = run_c3(args, rank, world, local_rank, args.steps, args.warmup)
    else:
        line = run_c4(args, rank, world, local_rank, args.steps, args.warmup)
        if args.bs1_steps > 0:
            bs1 = run_c3(args, rank, world, local_rank, args.bs1_steps, min(args.warmup, 3))
            if line is not None:
                line["bs1"] = {"workload": "C3 (batch-1 frame loop, 200-token context, greedy)",
                               "frames_per_s": bs1["value"] / world, "frame_latency_us": bs1["frame_latency_us"],
                               "rtf": bs1["rtf"], "e2e_frames_per_s": bs1["e2e"]["value"] / world,
                               "hbm_frac": bs1["roofline"]["frac"], "steps": args.bs1_steps,
                               "ref_gpu_baseline": bs1["ref_gpu_baseline"]}
                if bs1["ref_gpu_baseline"] is not None:
                    line["bs1"]["ref_megakernel_frame_ms"] = bs1["ref_gpu_baseline"]["frame_ms"]
        if args.serve_requests > 0:
            serving = run_serving(args, rank, world, local_rank)
            if line is not None:
                line["serving"] = serving
        if not args.no_c5:
            c5 = run_c5(args, rank, world, local_rank)
            if line is not None:
                line["c5"] = c5
    if line is None:
        return
    if world == 1 and not args.no_cpu_baseline:
        c4 = args.workload == "c4"
        fps, cores, timed, el = cpu_frames_per_s(args.cpu_seconds, sampled=c4, ctx=CTX_MID if c4 else CTX)
        line["cpu_baseline"] = {"value": fps, "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": cpu_sample_text(c4, timed, el, cores)}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and args.impl == "ours":
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    args.gpus = world
    try:
        if args.impl == "reference":
            run_reference(args, rank)
        else:
            run_ours(args, rank, world, local_rank)
    except BaseException:
        if world > 1 and args.impl == "ours":
            # the other ranks may be waiting in a collective this rank never reaches: exit at once
            # (torchrun then stops them) instead of waiting in destroy_process_group
            import traceback
            traceback.print_exc()
            sys.stdout.flush()
            sys.stderr.flush()
            os._exit(1)
        raise
    if world > 1 and args.impl == "ours":
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
