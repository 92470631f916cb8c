"""CPU checks of the C ABI: the library loads, exports every declared symbol, and its host-only
planning entry points validate shapes (no kernel is launched: there is no GPU here)."""

import ctypes
import os
import re

import pytest

from conftest import REPO
from packref import part_begin, part_owner

HEADER = os.path.join(REPO, "include", "qd_decode.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qd_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from decode_b200 import build, lib as L

    build.build()
    return L.load()


def test_header_declares_and_library_exports_every_symbol(lib):
    from decode_b200 import lib as L

    syms = declared_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/qd_decode.h but not exported"
        assert s in L.PROTOTYPES, f"{s} has no ctypes prototype"
    assert set(L.PROTOTYPES) <= set(syms)


def test_version_and_errors(lib):
    assert b"sm_100a" in lib.qd_version()
    g, nb = ctypes.c_int(0), ctypes.c_int64(0)
    rc = lib.qd_gemv_plan(100, 2560, 1, 0, ctypes.byref(g), ctypes.byref(nb))
    assert rc == 4 and b"n%128" in lib.qd_last_error()
    rc = lib.qd_gemv_plan(6144, 2560, 9, 0, ctypes.byref(g), ctypes.byref(nb))
    assert rc == 4


@pytest.mark.parametrize("n,k,m", [(6144, 2560, 1), (2560, 4096, 4), (19456, 2560, 8), (2560, 9728, 2),
                                   (151936, 2560, 1), (256, 128, 3)])
def test_gemv_plan_sizes(lib, n, k, m):
    g, nb = ctypes.c_int(0), ctypes.c_int64(0)
    assert lib.qd_gemv_plan(n, k, m, 148, ctypes.byref(g), ctypes.byref(nb)) == 0
    T = (n // 128) * (k // 64)
    assert g.value == min(148, T)
    assert nb.value >= (n // 128) * 4 + m * 128 * 4


def test_attn_plan(lib):
    s, ch, nb = ctypes.c_int(0), ctypes.c_int64(0), ctypes.c_int64(0)
    assert lib.qd_attn_plan(1, 8, 384, 296, ctypes.byref(s), ctypes.byref(ch), ctypes.byref(nb)) == 0
    assert s.value * ch.value >= 384 and ch.value % 32 == 0
    assert lib.qd_attn_plan(32, 8, 32768, 296, ctypes.byref(s), ctypes.byref(ch), ctypes.byref(nb)) == 0
    assert s.value * ch.value >= 32768


def test_packed_bytes(lib):
    lib.qd_packed_bytes.restype = ctypes.c_int64
    assert lib.qd_packed_bytes(151936, 2560) == 151936 * 2560 * 2
    assert lib.qd_packed_bytes(100, 64) == 128 * 64 * 2


@pytest.mark.parametrize("T,G", [(1920, 148), (1280, 148), (47480, 148), (3040, 148), (10, 3), (148, 148),
                                 (7, 7), (1000, 999)])
def test_stream_k_partition_covers_every_block_once(T, G):
    owners = [part_owner(T, G, b) for b in range(T)]
    for c in range(G):
        for b in range(part_begin(T, G, c), part_begin(T, G, c + 1)):
            assert owners[b] == c
    assert part_begin(T, G, 0) == 0 and part_begin(T, G, G) == T
    assert all(part_begin(T, G, c + 1) - part_begin(T, G, c) in (T // G, T // G + 1) for c in range(G))
