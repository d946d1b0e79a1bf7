"""Build libqtt.so in-tree for sm_100a with nvcc (no JIT cache, so the library travels with
the source tree).

Every build stamps the hash of its sources (``source_hash()``: csrc/*.cu, csrc/*.cuh and
include/qtt.h) into the library, exported as ``qtt_build_id()``, and writes it beside the library
(``libqtt.so.buildid``). The library is rebuilt whenever the sources' hash differs from the stamp,
and ``check_build_id()`` tells whether a prebuilt library matches the sources next to it.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(_HERE, "csrc")
SOURCES = ("qtt_kernel.cu", "qtt_api.cu", "qtt_noalloc.cu")
HEADERS = ("qtt_kernel.cuh", "qtt_device.cuh", "qtt_batch.cuh")
LIB = os.path.join(_HERE, "libqtt.so")
INCLUDE = os.path.join(os.path.dirname(_HERE), "include")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def source_hash() -> str:
    """16 hex digits of the SHA-256 over the library's sources (name and content, in order)."""
    h = hashlib.sha256()
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(INCLUDE, "qtt.h")]
    for d in deps:
        h.update(os.path.basename(d).encode())
        with open(d, "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


def _stamp_path() -> str:
    return LIB + ".buildid"


def _stale() -> bool:
    if not os.path.exists(LIB) or not os.path.exists(_stamp_path()):
        return True
    with open(_stamp_path()) as f:
        return f.read().strip() != source_hash()


def check_build_id(lib) -> None:
    """Raises RuntimeError when the loaded library (a ctypes handle) was not built from the
    sources in this tree."""
    got = lib.qtt_build_id().decode()
    want = source_hash()
    if got != want:
        raise RuntimeError(f"libqtt.so was built from other sources (build id {got}, sources {want}); "
                           "rebuild it with qwentts_turbo_b200.build.build_library(force=True)")


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/*.cu into qwentts_turbo_b200/libqtt.so (skipped when up to date)."""
    if not force and not _stale():
        return LIB
    bid = source_hash()
    cmd = ([_nvcc()] + NVCC_FLAGS + [f'-DQTT_BUILD_ID="{bid}"', "-I", INCLUDE] +
           [os.path.join(CSRC, s) for s in SOURCES] + ["-o", LIB + ".tmp"])
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(r.stdout + r.stderr)
    os.replace(LIB + ".tmp", LIB)
    with open(_stamp_path(), "w") as f:
        f.write(bid + "\n")
    return LIB


if __name__ == "__main__":
    build_library(force=True, verbose=True)
    print(LIB)
