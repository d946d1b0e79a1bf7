"""Generate tests/golden/ref_megakernel_golden.npz from the reference's OWN CUDA kernels
(hamza1brh/qwenTTS-turbo qwentts_turbo/csrc/*.cu, compiled for sm_100a by oracle/Makefile into
oracle/_ref/). Needs a GPU; run from the repo root:

    make -C oracle && python tests/golden/make_ref_golden.py <output.npz>

Inputs are regenerated from seeds on the CPU side of the test (qwentts_turbo_b200.workloads):
spec weights (seed 0 backbone, seed 1 code predictor), C1 KV cache + embedding (seed 2,
ctx 256, position 256), six code-predictor step embeddings N(0,1) (seed 9) at positions 0..5.
Stored: the reference kernels' fp32 final-normed outputs.
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import ref_kernels  # noqa: E402
from qwentts_turbo_b200.megakernel_backbone import extract_backbone_weights  # noqa: E402
from qwentts_turbo_b200.megakernel_code_predictor import extract_code_predictor_weights  # noqa: E402
from qwentts_turbo_b200.weights import synthetic_weights  # noqa: E402
from qwentts_turbo_b200.workloads import c1_inputs  # noqa: E402


def main(out_path):
    assert ref_kernels.available(), "build oracle/_ref first (make -C oracle)"
    w = synthetic_weights()
    k, v, emb = c1_inputs()
    bw = extract_backbone_weights(w, 512)
    tts = ref_kernels.RefDecoder("tts", bw["layer_weights"], bw["final_norm_weight"], bw["cos_table"],
                                 bw["sin_table"], 28, 512)
    tts.k[:, :, :256] = k.cuda()
    tts.v[:, :, :256] = v.cuda()
    tts.position = 256
    bb_hidden = tts.step(emb.cuda()).cpu().numpy()
    cw = extract_code_predictor_weights(w)
    cp = ref_kernels.RefDecoder("cp", cw["layer_weights"], cw["final_norm_weight"], cw["cos_table"],
                                cw["sin_table"], 5, 256)
    g = torch.Generator().manual_seed(9)
    cp_emb = torch.randn(6, 1024, generator=g).to(torch.bfloat16)
    cp_hidden = np.stack([cp.step(cp_emb[i].cuda()).cpu().numpy() for i in range(6)])
    torch.cuda.synchronize()
    np.savez_compressed(out_path, bb_layers=28, cp_layers=5, ctx=256, kv_seed=2, bb_hidden=bb_hidden,
                        cp_seed=9, cp_emb=cp_emb.float().numpy(), cp_hidden=cp_hidden)
    print("wrote", out_path, "bb |h| max", float(np.abs(bb_hidden).max()))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.path.dirname(__file__), "ref_megakernel_golden.npz"))
