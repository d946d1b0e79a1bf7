"""bench.py host logic without a GPU: every workload names its configuration, and the roofline
traffic figure is read from the committed ncu summaries."""
import argparse
import importlib.util
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("qtt_bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_every_workload_has_a_config():
    b = _bench()
    for w in ("c4", "c3", "prefill", "c5"):
        cfg = b.workload_config(argparse.Namespace(workload=w, gpus=2, batch=64, warmup=3, steps=10))
        assert cfg["workload"] and cfg["model"] and "parallelism" in cfg and "l2" in cfg
        assert cfg["global_batch"] in (2, 128)


def test_traffic_ratios_from_profiles():
    b = _bench()
    for name in ("qtt_decode_kernel_frame_c3.txt", "qtt_batch_kernel_frame_c4.txt",
                 "qtt_batch_kernel_prefill_dense.txt"):
        t = b.ncu_traffic_per_frame(1e9, name)
        assert t is not None and 1.0e9 <= t <= 1.3e9, (name, t)
    assert b.ncu_traffic_per_frame(1e9, "no_such_summary.txt") is None
