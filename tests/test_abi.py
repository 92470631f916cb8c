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


def header_prototypes():
    """{name: (return type, [parameter types])} of every qd_* prototype in the header."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    out = {}
    for m in re.finditer(r"([A-Za-z_][\w\s*]*?)\b(qd_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text):
        params = [p.strip() for p in m.group(3).split(",")]
        if params in ([""], ["void"]):
            params = []
        types = [p if p.endswith("*") else re.sub(r"\s*\b\w+$", "", p) for p in params]  # drop the name
        out[m.group(2)] = (" ".join(m.group(1).split()), [" ".join(t.split()) for t in types])
    return out


def _ctype_matches(c_type: str, ct) -> bool:
    if "*" in c_type or c_type == "cudaStream_t":  # any pointer, the stream handle included
        return ct in (ctypes.c_void_p, ctypes.c_char_p) or (isinstance(ct, type) and issubclass(ct, ctypes._Pointer))
    return ct is {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "float": ctypes.c_float,
                  "double": ctypes.c_double}[c_type]


def test_ctypes_table_matches_every_header_prototype():
    """decode_b200/lib.py's PROTOTYPES (the table every Python call goes through) against the header:
    the same entry points, the same number of parameters and a matching C type for each, and the
    same return type, so a changed signature cannot leave a stale ctypes binding behind."""
    from decode_b200 import lib as L

    protos = header_prototypes()
    assert sorted(protos) == sorted(L.PROTOTYPES)
    for name, (ret, params) in protos.items():
        restype, argtypes = L.PROTOTYPES[name]
        assert len(argtypes) == len(params), (name, params, argtypes)
        for i, (c_type, ct) in enumerate(zip(params, argtypes)):
            assert _ctype_matches(c_type, ct), (name, i, c_type, ct)
        assert _ctype_matches(ret, restype), (name, ret, restype)


def test_step_desc_mirrors_the_header_struct():
    """decode_b200/lib.py's StepDesc against qd_step_desc in the header: the same field names in the same
    order, pointers as pointers, int64_t / double as themselves (so the same offsets and size)."""
    from decode_b200 import lib as L

    text = open(HEADER).read()
    body = re.search(r"typedef struct qd_step_desc \{(.*?)\} qd_step_desc;", text, flags=re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for decl in body.split(";"):
        decl = " ".join(decl.split())
        if not decl:
            continue
        m = re.match(r"((?:const )?[A-Za-z_0-9]+\s*\**)\s*(.*)", decl)
        ctype, names = m.group(1).replace(" ", ""), [n.strip() for n in m.group(2).split(",")]
        for n in names:
            kind = "ptr" if ctype.endswith("*") else {"int64_t": "i64", "double": "f64"}[ctype]
            fields.append((n, kind))
    ours = [(n, "ptr" if t is ctypes.c_void_p else {ctypes.c_int64: "i64", ctypes.c_double: "f64"}[t])
            for n, t in L.StepDesc._fields_]
    assert ours == fields
    assert ctypes.sizeof(L.StepDesc) == 8 * len(fields)


def test_integration_stubs_bind_the_header_signatures():
    """The reference-side ctypes stubs in INTEGRATION.md, executed against a stand-in library object:
    every argtypes list they set has the header prototype's parameter count and kinds."""
    import types

    class StandIn:
        def __init__(self):
            self.fns = {}

        def __getattr__(self, name):
            return self.fns.setdefault(name, types.SimpleNamespace())

    text = open(os.path.join(REPO, "INTEGRATION.md")).read()
    blocks = re.findall(r"```python\n(.*?)```", text, flags=re.S)
    stand_in = StandIn()
    ns = {}
    ran = 0
    for b in blocks:
        if "_lib." not in b:
            continue  # the engine usage example (needs a checkpoint)
        b = re.sub(r"_lib = ctypes\.CDLL\([^)]*\)", "_lib = __stand_in__", b)
        ns["__stand_in__"] = stand_in
        exec(compile(b, "INTEGRATION.md", "exec"), ns)
        ran += 1
    assert ran >= 3
    protos = header_prototypes()
    bound = {n: f.argtypes for n, f in stand_in.fns.items() if hasattr(f, "argtypes")}
    assert len(bound) >= 6
    for name, argtypes in bound.items():
        params = protos[name][1]
        assert len(argtypes) == len(params), (name, params, argtypes)
        for i, (c_type, ct) in enumerate(zip(params, argtypes)):
            assert _ctype_matches(c_type, ct), (name, i, c_type, ct)


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


def test_prompt_entry_points_validate_arguments(lib):
    """The prompt kernels' entry points reject bad shapes, strides and pointers on the host, before any
    launch (every call here is invalid, so nothing reaches the GPU)."""
    P = ctypes.c_void_p
    a, b, c = P(0x10000), P(0x20000), P(0x30000)  # 16-byte aligned stand-ins, never dereferenced
    ERR_ARG = 1
    # qd_tc_gemm(x, ldx, m, w, n, k, out, ldo, res, ldr, epilogue, scratch, scratch_bytes, err, stream)
    assert lib.qd_tc_gemm(None, 2560, 8, b, 2560, 2560, c, 2560, None, 0, 0, None, 0, None, None) == ERR_ARG
    assert lib.qd_tc_gemm(a, 2560, 0, b, 2560, 2560, c, 2560, None, 0, 0, None, 0, None, None) == ERR_ARG
    assert lib.qd_tc_gemm(a, 2560, 8, b, 2500, 2560, c, 2560, None, 0, 0, None, 0, None, None) == ERR_ARG   # n % 128
    assert lib.qd_tc_gemm(a, 2560, 8, b, 2560, 2500, c, 2560, None, 0, 0, None, 0, None, None) == ERR_ARG   # k % 64
    assert lib.qd_tc_gemm(a, 2560, 8, b, 2560, 2560, c, 2560, None, 0, 7, None, 0, None, None) == ERR_ARG   # epilogue
    assert lib.qd_tc_gemm(a, 2560, 8, b, 2560, 2560, c, 2560, None, 0, 1, None, 0, None, None) == ERR_ARG   # RES, no res
    assert lib.qd_tc_gemm(P(0x10008), 2560, 8, b, 2560, 2560, c, 2560, None, 0, 0, None, 0, None, None) == ERR_ARG
    assert lib.qd_tc_gemm(a, 2560, 8, b, 19456, 2560, c, 9000, None, 0, 2, None, 0, None, None) == ERR_ARG  # ldo < n/2
    # qd_rmsnorm_rows(x, ldx, m, k, w, eps, out, ldo, stream)
    assert lib.qd_rmsnorm_rows(a, 2560, 4, 2561, b, 1e-6, c, 2560, None) == ERR_ARG
    assert lib.qd_rmsnorm_rows(a, 2560, 4, 2560, None, 1e-6, c, 2560, None) == ERR_ARG
    # qd_prefill_qk_rope(qkv, ldqkv, batch, S, nq, nkv, qn, kn, eps, cos, sin, q_out, ldq, kc, vc, cap, cs_b, cs_h, s)
    assert lib.qd_prefill_qk_rope(a, 6144, 1, 200, 32, 8, b, b, 1e-6, c, c, a, 4096, b, c, 128, 8 * 128 * 128,
                                  128 * 128, None) == ERR_ARG                                   # S > cap
    # qd_prefill_attn(q, ldq, batch, S, q_begin, nq, nkv, kc, vc, cap, cs_b, cs_h, scale, out, ldo, err, stream)
    cs_h, cs_b = 256 * 128, 8 * 256 * 128
    assert lib.qd_prefill_attn(a, 4096, 1, 200, 200, 32, 8, b, c, 256, cs_b, cs_h, 0.088, a, 4096, None,
                               None) == ERR_ARG                                                 # q_begin >= S
    assert lib.qd_prefill_attn(a, 4096, 1, 200, 0, 30, 8, b, c, 256, cs_b, cs_h, 0.088, a, 4096, None,
                               None) == ERR_ARG                                                 # nq % nkv
    assert lib.qd_prefill_attn(a, 4096, 1, 200, 0, 32, 8, b, c, 256, cs_b, 100, 0.088, a, 4096, None,
                               None) == ERR_ARG                                                 # cs_h < cap*128
    assert lib.qd_prefill_attn(a, 4000, 1, 200, 0, 32, 8, b, c, 256, cs_b, cs_h, 0.088, a, 4096, None,
                               None) == ERR_ARG                                                 # ldq < nq*128


def test_tc_gemm_plan_tile_choice(lib):
    """Prompt GEMM plan: 256-wide weight tiles once they alone give every SM a tile, else 128; K split
    across CTAs for the tiles of the last, partial wave (as many splits as fit one wave, >= 8 K-blocks a
    split), their fp32 partials in scratch; 148 SMs here (no device: the default count)."""
    g, bn, ks, nb = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int64(0)
    args = (ctypes.byref(g), ctypes.byref(bn), ctypes.byref(ks), ctypes.byref(nb))
    assert lib.qd_tc_gemm_plan(16384, 19456, 2560, *args) == 0
    assert (bn.value, g.value, ks.value, nb.value) == (256, 148, 1, 0)
    assert lib.qd_tc_gemm_plan(128, 2560, 4096, *args) == 0          # O of a 128-token prompt: 20 tiles
    assert (bn.value, ks.value, g.value, nb.value) == (128, 7, 140, 20 * 7 * 128 * 128 * 4)
    assert lib.qd_tc_gemm_plan(128, 6144, 2560, *args) == 0          # QKV: 48 tiles, 40 K-blocks
    assert (ks.value, g.value) == (3, 144)
    assert lib.qd_tc_gemm_plan(1, 2560, 640, *args) == 0             # 10 K-blocks: no split
    assert (ks.value, nb.value) == (1, 0)
    assert lib.qd_tc_gemm_plan(1024, 2560, 9728, *args) == 0         # 160 tiles: 148 whole, the last 12 split
    assert (bn.value, ks.value, g.value, nb.value) == (128, 12, 148, 12 * 12 * 128 * 128 * 4)
    assert lib.qd_tc_gemm_plan(1, 100, 64, *args) == 1


def test_recorded_calls_replay_in_order_and_raise_on_error():
    """lib.recording / bind / replay (the speculative verify's launch list): calls are collected with
    their argument lists, replayed with edited arguments, and a non-zero status raises QDError."""
    from decode_b200 import lib as qdlib

    g, bn, ks, nb = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int64(0)
    out = (ctypes.byref(g), ctypes.byref(bn), ctypes.byref(ks), ctypes.byref(nb))
    with qdlib.recording() as rec:
        qdlib.call("qd_tc_gemm_plan", 128, 2560, 4096, *out)
    assert [name for name, _ in rec] == ["qd_tc_gemm_plan"] and g.value == 0  # nothing ran yet
    bound = qdlib.bind(rec)
    qdlib.replay(bound)
    assert (bn.value, ks.value) == (128, 7)
    bound[0][2][0] = 16384  # edit the recorded arguments in place, as the verify does per round
    bound[0][2][1] = 19456
    bound[0][2][2] = 2560
    qdlib.replay(bound)
    assert (bn.value, ks.value, nb.value) == (256, 1, 0)
    bound[0][2][1] = 100  # n % 128 != 0
    with pytest.raises(qdlib.QDError):
        qdlib.replay(bound)
