# SPDX-License-Identifier: Apache-2.0
"""CPU: the native libraries load and export every symbol the headers declare."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from gsa_b200 import _library

ROOT = Path(__file__).resolve().parents[1]
HEADERS = {"gsa_bvh": ROOT / "include" / "gsa_bvh.h", "reference_queries": ROOT / "include" / "reference_queries.h"}

# Symbols the reference binds (gsa/runtime.py:13-26, gsa/reference.py:11-14).
REFERENCE_SYMBOLS = {
    "gsa_bvh": {"build_bvh", "query_bvh", "query_ball_bvh", "free_bvh", "set_pool_mode", "pool_memory", "pool_reset_peak"},
    "reference_queries": {"ball", "nn3"},
}


def declared(header):
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return set(re.findall(r"^\s*int\s+(\w+)\s*\(", text, flags=re.M))


def exported(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


@pytest.mark.parametrize("name", sorted(HEADERS))
def test_headers_cover_reference_abi(name):
    assert REFERENCE_SYMBOLS[name] <= declared(HEADERS[name])


@pytest.mark.parametrize("name", sorted(HEADERS))
def test_library_exports_every_declared_symbol(name):
    lib = _library.load(name)
    syms = declared(HEADERS[name])
    assert syms
    for s in syms:
        assert hasattr(lib, s), s
    assert syms <= exported(_library.path(name))


def test_only_declared_symbols_are_exported():
    for name, header in HEADERS.items():
        assert exported(_library.path(name)) == declared(header), name


def test_test_variant_library_exports_same_abi():
    for name in ("gsa_bvh_walk", "gsa_bvh_ordered", "gsa_bvh_stack4", "gsa_bvh_cap8"):
        p = _library.path(name)
        assert p.is_file(), name
        assert exported(p) == declared(HEADERS["gsa_bvh"]), name


def test_pool_calls_without_gpu():
    lib = _library.load("gsa_bvh")
    lib.pool_memory.argtypes = [ctypes.POINTER(ctypes.c_uint64)] * 2
    a, b = ctypes.c_uint64(7), ctypes.c_uint64(7)
    assert lib.pool_memory(ctypes.byref(a), ctypes.byref(b)) == 0
    assert (a.value, b.value) == (0, 0)  # pool not created before first use
    assert lib.set_pool_mode(1) == 0
    assert lib.pool_reset_peak() == 0


def test_invalid_arguments_rejected_without_gpu():
    lib = _library.load("gsa_bvh")
    P = ctypes.c_void_p
    lib.build_bvh.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(P), P]
    h = P()
    assert lib.build_bvh(None, 10, 1, 16, ctypes.byref(h), None) == -1
    assert lib.build_bvh(P(16), 0, 1, 16, ctypes.byref(h), None) == -1
    assert lib.build_bvh(P(16), 10, 1, 0, ctypes.byref(h), None) == -1
    lib.query_ball_bvh.argtypes = [P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, P, P, P]
    assert lib.query_ball_bvh(None, None, 1, 1, 0, 1.0, 8, None, None, None) == -2
    lib.free_bvh.argtypes = [P, ctypes.c_int, P]
    assert lib.free_bvh(None, 1, None) == -3
    ref = _library.load("reference_queries")
    ref.ball.argtypes = [ctypes.c_int] * 3 + [ctypes.c_float, ctypes.c_int, P, P, P, P]
    assert ref.ball(0, 5, 0, 1.0, 4, None, None, None, None) == 0  # empty batch is a no-op
    assert ref.ball(1, 5, 3, 1.0, 0, None, None, None, None) == -2
