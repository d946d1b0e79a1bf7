"""The C-ABI library builds for sm_100a, loads without a GPU, and exports every entry point
include/qtt.h declares (no compute calls here)."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qtt.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"\b((?:launch|qtt)_\w+)\s*\(", src)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib_path():
    from qwentts_turbo_b200.build import build_library
    return build_library()


def test_header_declares_reference_launchers():
    names = declared_functions()
    for n in ("launch_tts_decode_with_embedding", "launch_tts_decode", "launch_cp_decode_with_embedding"):
        assert n in names


def test_library_exports_every_declared_symbol(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing


def test_library_loads_and_binds(lib_path):
    from qwentts_turbo_b200 import _lib
    lib = _lib.load(lib_path)
    for n in declared_functions():
        assert hasattr(lib, n), n
    assert set(_lib.SIGNATURES) <= set(declared_functions())
    assert lib.qtt_status_string(0) == b"ok"
    assert lib.qtt_last_launch_status() == 0


def test_library_build_id_matches_sources(lib_path):
    """The library identifies the sources it was built from (a stale prebuilt library is
    detectable on any machine it travels to)."""
    from qwentts_turbo_b200 import _lib
    from qwentts_turbo_b200.build import check_build_id, source_hash
    lib = _lib.load(lib_path)
    assert lib.qtt_build_id().decode() == source_hash()
    check_build_id(lib)
