"""qtt_backbone_step_noalloc: the backbone decode step for callers that must not allocate device
memory while decoding (a service that reserves its whole device memory budget at start-up, or a
host framework whose caching allocator owns the device memory). Its scratch is a fixed device
array inside libqtt.so instead of the drop-in launcher's per-stream cudaMalloc.

Checked through the C ABI against the existing entry point (launch_tts_decode_with_embedding)
on the same inputs for two calls in a row, with the parity tolerance of the other GPU tests
(atol 2e-2 / rtol 1e-2), and both against the fp64 CPU oracle of the same step. After each call
qtt_stream_check reads the fixed scratch's error word (a device-side timeout would show there),
and the device's free memory does not change across the second call. This file is collected
last so that a run stopping at the first failure has already run every other test; it also
passes on its own in a fresh process.
"""
import ctypes
import math

import pytest
import torch

from oracle import qtt_oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def test_noalloc_step_matches_dropin_launcher():
    from qwentts_turbo_b200 import _lib
    from qwentts_turbo_b200.megakernel_backbone import device_layer_table, extract_backbone_weights
    from qwentts_turbo_b200.weights import synthetic_weights
    from qwentts_turbo_b200.workloads import c1_inputs

    lib = _lib.load()
    torch.cuda.set_device(0)
    n_layers, ctx, max_seq = 4, 100, 512
    w = synthetic_weights(backbone_layers=n_layers, cp_layers=1, seed_backbone=21, seed_cp=22, norm_std=0.1)
    bw = extract_backbone_weights(w, max_seq)
    table = device_layer_table(bw["layer_weights"], n_layers)
    table_p = ctypes.cast(table.data_ptr(), ctypes.POINTER(_lib.TTSLayerWeights))
    k, v, _ = c1_inputs(n_layers=n_layers, ctx=ctx, seed=5)
    orc = O.Qwen3TTSOracle(w, backbone_layers=n_layers, cp_layers=1, max_seq=max_seq, dtype=torch.float64)
    orc.reset_backbone()
    orc.set_kv_cache(k.double(), v.double())
    caches = []
    for _ in range(2):   # [0]: existing entry point, [1]: no-alloc entry point
        kc = torch.zeros(n_layers, 8, max_seq, 128, dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros_like(kc)
        kc[:, :, :ctx] = k.cuda()
        vc[:, :, :ctx] = v.cuda()
        caches.append((kc, vc))
    g = torch.Generator().manual_seed(6)
    scale = ctypes.c_float(1.0 / math.sqrt(128.0))
    stream = torch.cuda.current_stream().cuda_stream
    embs = [torch.randn(1024, generator=g).to(torch.bfloat16).cuda() for _ in range(2)]
    results = [[(torch.full((1024,), float("nan"), dtype=torch.float32, device="cuda"),
                 torch.zeros(1024, dtype=torch.bfloat16, device="cuda")) for _ in range(2)] for _ in range(2)]
    for call in range(2):
        emb = embs[call]
        pos = ctx + call
        for which, (kc, vc) in enumerate(caches):
            out, hid = results[call][which]
            if which == 0:
                lib.launch_tts_decode_with_embedding(
                    emb.data_ptr(), table_p, bw["final_norm_weight"].data_ptr(), bw["cos_table"].data_ptr(),
                    bw["sin_table"].data_ptr(), kc.data_ptr(), vc.data_ptr(), hid.data_ptr(), None, None, None,
                    None, None, None, None, out.data_ptr(), n_layers, pos, pos + 1, max_seq, scale, stream)
                assert lib.qtt_last_launch_status() == 0
            else:
                torch.cuda.synchronize()
                free_before = torch.cuda.mem_get_info()[0]
                rc = lib.qtt_backbone_step_noalloc(
                    emb.data_ptr(), table_p, bw["final_norm_weight"].data_ptr(), bw["cos_table"].data_ptr(),
                    bw["sin_table"].data_ptr(), kc.data_ptr(), vc.data_ptr(), hid.data_ptr(), out.data_ptr(),
                    n_layers, pos, max_seq, scale, stream)
                assert rc == 0, _lib.STATUS.get(rc)
                # device-side errors of the step (from the fixed scratch's error word)
                assert lib.qtt_stream_check(stream) == 0
                if call == 1:   # the first call set the path up; the second allocates nothing
                    assert torch.cuda.mem_get_info()[0] == free_before
        torch.cuda.synchronize()
        (a, ha), (b, hb) = results[call]
        assert torch.isfinite(b).all()
        torch.testing.assert_close(b, a, atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(hb.float(), ha.float(), atol=ATOL, rtol=RTOL)
        # the new K/V rows agree as well
        torch.testing.assert_close(caches[1][0][:, :, pos].float(), caches[0][0][:, :, pos].float(),
                                   atol=ATOL, rtol=RTOL)
        # both against the fp64 oracle of the same step (final-normed hidden and codec-head logits)
        orc.position = pos
        ref = orc.backbone_step(emb.cpu().double())
        W = orc.codec_head
        l_ref = O.Qwen3TTSOracle.head_logits(W, ref)
        for got in (a, b):
            rel = float((got.cpu().double() - ref).norm() / ref.norm())
            assert rel <= 1.5e-2, f"call {call}: hidden rel-L2 {rel:.3g} from the oracle"
            torch.testing.assert_close(O.Qwen3TTSOracle.head_logits(W, got.cpu().double()), l_ref,
                                       atol=ATOL, rtol=RTOL)
        # keep the oracle's cache equal to the engine's (the row this step wrote)
        orc.bk[:, :, pos] = caches[1][0][:, :, pos].cpu().double()
        orc.bv[:, :, pos] = caches[1][1][:, :, pos].cpu().double()
    assert lib.qtt_stream_check(stream) == 0

    # beyond the fixed scratch's capacity: a clear error, nothing launched
    out = torch.zeros(1024, dtype=torch.float32, device="cuda")
    kc, vc = caches[1]
    rc = lib.qtt_backbone_step_noalloc(emb.data_ptr(), table_p, bw["final_norm_weight"].data_ptr(),
                                       bw["cos_table"].data_ptr(), bw["sin_table"].data_ptr(), kc.data_ptr(),
                                       vc.data_ptr(), None, out.data_ptr(), n_layers, 0, 1 << 20, scale, stream)
    assert rc == _lib.QTT_ERR_UNSUPPORTED
