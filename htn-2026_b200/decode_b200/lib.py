"""ctypes binding of libqd_decode.so (the C ABI declared in include/qd_decode.h).

The library is the only compute path of the decode step: there is no CPU or PyTorch fallback.
If it is missing or fails to load, `load()` raises; build it with `python -m decode_b200.build`.
"""

from __future__ import annotations

import ctypes
import os

from . import build as _build

_LIB = None

c_void_p, c_int, c_int64, c_float = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
P_I64 = ctypes.POINTER(ctypes.c_int64)
P_INT = ctypes.POINTER(ctypes.c_int)

class StepDesc(ctypes.Structure):
    """qd_step_desc of include/qd_decode.h (every field 8 bytes wide, same order)."""

    _fields_ = [
        ("w_qkv", c_void_p), ("w_qkv_layer_bytes", c_int64), ("w_o", c_void_p), ("w_o_layer_bytes", c_int64),
        ("w_gu", c_void_p), ("w_gu_layer_bytes", c_int64), ("w_down", c_void_p), ("w_down_layer_bytes", c_int64),
        ("e_packed", c_void_p), ("ln1", c_void_p), ("ln2", c_void_p), ("q_norm", c_void_p), ("k_norm", c_void_p),
        ("final_norm", c_void_p), ("layers", c_int64), ("hidden", c_int64), ("inter", c_int64),
        ("nq_heads", c_int64), ("nkv_heads", c_int64), ("vocab", c_int64), ("batch", c_int64),
        ("eps", ctypes.c_double), ("scale", ctypes.c_double), ("tok", c_void_p), ("pos", c_void_p),
        ("x", c_void_p), ("q", c_void_p), ("attn", c_void_p), ("act", c_void_p), ("k_cache", c_void_p),
        ("v_cache", c_void_p), ("cache_layer_stride", c_int64), ("cs_b", c_int64), ("cs_h", c_int64),
        ("cap", c_int64), ("cos", c_void_p), ("sin", c_void_p), ("logits", c_void_p), ("ld_logits", c_int64),
        ("err", c_void_p), ("trace", c_void_p),
    ]


P_DESC = ctypes.POINTER(StepDesc)

# name -> (restype, argtypes); every function declared in include/qd_decode.h
PROTOTYPES = {
    "qd_version": (ctypes.c_char_p, []),
    "qd_last_error": (ctypes.c_char_p, []),
    "qd_sm_count": (c_int, [P_INT]),
    "qd_packed_bytes": (c_int64, [c_int64, c_int64]),
    "qd_pack_rows": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64,
                             c_void_p]),
    "qd_embed": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int, c_void_p, c_int64, c_void_p, c_int, c_void_p]),
    "qd_gemv_plan": (c_int, [c_int64, c_int64, c_int, c_int, P_INT, P_I64]),
    "qd_gemv": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_void_p, c_int64, c_void_p, c_int64,
                        c_void_p, c_float, c_int, c_int, c_void_p, c_int64, c_void_p, c_int, c_void_p]),
    "qd_gemv_noalloc": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_void_p, c_int64, c_void_p,
                                c_int64, c_void_p, c_float, c_int, c_void_p, c_int, c_void_p]),
    "qd_qkv_rope_append": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p, c_float, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p,
                                   c_void_p, c_int64, c_int64, c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int,
                                   c_void_p]),
    "qd_lm_head_plan": (c_int, [c_int64, c_int64, c_int, c_int, P_INT, P_I64]),
    "qd_lm_head_argmax": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_void_p, c_float, c_void_p,
                                  c_void_p, c_int, c_void_p, c_int64, c_int, c_void_p, c_int64, c_void_p, c_int,
                                  c_void_p]),
    "qd_pack_act": (c_int, [c_void_p, c_int64, c_int, c_int, c_int64, c_void_p, c_float, c_void_p, c_int, c_void_p]),
    "qd_qkv_rope_sums": (c_int, [c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p, c_float, c_void_p,
                                 c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                 c_int, c_void_p]),
    "qd_pack_act_res": (c_int, [c_void_p, c_int64, c_int, c_int, c_int64, c_void_p, c_void_p, c_float, c_void_p,
                                c_int, c_void_p]),
    "qd_tc_gemv_plan": (c_int, [c_int64, c_int64, c_int, c_int, P_INT, P_I64]),
    "qd_tc_gemv": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                           c_int, c_int, c_void_p, c_int64, c_void_p, c_int, c_void_p]),
    "qd_tc_qkv_rope_append": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                      c_int64, c_int64, c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int,
                                      c_void_p]),
    "qd_tc_lm_head_argmax": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int,
                                     c_void_p, c_int64, c_int, c_void_p, c_int64, c_void_p, c_int, c_void_p]),
    "qd_attn_stream_plan": (c_int, [c_int, c_int, c_int64, c_int, P_INT, P_INT, P_I64]),
    "qd_attn_decode_stream": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                      c_int64, c_int64, c_int64, c_int, c_int, c_float, c_void_p, c_int64,
                                      c_void_p, c_int, c_void_p]),
    "qd_attn_tc_plan": (c_int, [c_int, c_int, c_int64, c_int, P_INT, P_INT, P_I64]),
    "qd_attn_decode_tc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                  c_int64, c_int64, c_int64, c_int, c_int, c_float, c_void_p, c_int64,
                                  c_void_p, c_int, c_void_p]),
    "qd_attn_plan": (c_int, [c_int, c_int, c_int64, c_int, P_INT, P_I64, P_I64]),
    "qd_decode_step_plan": (c_int, [P_DESC, P_I64, P_INT]),
    "qd_decode_step": (c_int, [P_DESC, c_void_p, c_int64, c_void_p]),
    "qd_tc_decode_step_plan": (c_int, [P_DESC, P_I64, P_INT]),
    "qd_tc_decode_step": (c_int, [P_DESC, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "qd_attn_decode": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int64,
                               c_int64, c_int64, c_int, c_int64, c_float, c_void_p, c_int64, c_void_p, c_int,
                               c_void_p]),
    "qd_tc_gemm_plan": (c_int, [c_int64, c_int64, c_int64, P_INT, P_INT, P_INT, P_I64]),
    "qd_tc_gemm": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p,
                           c_int64, c_int, c_void_p, c_int64, c_void_p, c_void_p]),
    "qd_rmsnorm_rows": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_float, c_void_p, c_int64, c_void_p]),
    "qd_argmax_rows": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "qd_tree_qk_rope": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p,
                                c_float, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64,
                                c_int64, c_void_p, c_void_p]),
    "qd_tree_attn": (c_int, [c_void_p, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int64, c_int64,
                             c_int64, c_void_p, c_void_p, c_float, c_void_p, c_int64, c_void_p, c_void_p]),
    "qd_tree_attn_rows": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int, c_int, c_void_p, c_void_p,
                                  c_int64, c_int64, c_float, c_void_p, c_int64, c_void_p, c_void_p]),
    "qd_tree_compact": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int, c_int64, c_int, c_int64, c_int64, c_void_p,
                                c_int, c_void_p]),
    "qd_prefill_qk_rope": (c_int, [c_void_p, c_int64, c_int, c_int64, c_int, c_int, c_void_p, c_void_p, c_float,
                                   c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64,
                                   c_int64, c_void_p]),
    "qd_prefill_attn": (c_int, [c_void_p, c_int64, c_int, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p, c_int64,
                                c_int64, c_int64, c_float, c_void_p, c_int64, c_void_p, c_void_p]),
    "qd_prefill_attn_rows": (c_int, [c_void_p, c_int64, c_int, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p,
                                     c_int64, c_int64, c_int64, c_float, c_void_p, c_int64, c_void_p, c_void_p]),
    "qd_prefill_qk_rope_at": (c_int, [c_void_p, c_int64, c_int, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p,
                                      c_float, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64,
                                      c_int64, c_int64, c_void_p]),
}

QD_OK, QD_ERR_ARG, QD_ERR_SCRATCH, QD_ERR_CUDA, QD_ERR_UNSUPPORTED = 0, 1, 2, 3, 4
QD_EPI_STORE, QD_EPI_RES, QD_EPI_SWIGLU, QD_EPI_SWIGLU_PACKED, QD_EPI_RES_SUMS, QD_EPI_STORE_SUMS = 0, 1, 2, 3, 4, 5
DEVERR = {1: "wait for a weight block timed out", 2: "wait for a free ring slot timed out",
          4: "drain of in-flight copies timed out", 8: "token id out of range",
          16: "decode position outside the cache", 32: "a wait for another CTA's results timed out",
          64: "dynamic shared memory misaligned (kernel did nothing)"}


class QDError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with code {code}: {msg}")
        self.code = code


def lib_path() -> str:
    return os.environ.get("QD_DECODE_LIB", _build.LIB)


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = path or lib_path()
    if not os.path.exists(path):
        raise RuntimeError(f"libqd_decode.so not found at {path}; build it with `python -m decode_b200.build` "
                           "(there is no fallback path)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


_RECORDING: list | None = None


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise QDError on a non-zero status (inside `recording`,
    collect (name, args) instead)."""
    if _RECORDING is not None:
        _RECORDING.append((name, list(args)))
        return
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != QD_OK:
        raise QDError(name, rc, lib.qd_last_error().decode(errors="replace"))


class recording:
    """Collect the entry-point calls made inside the block as (name, argument list) instead of running
    them, for a caller that replays a fixed launch sequence with `replay` (the Python-side argument
    checks of the wrappers run once, when recorded)."""

    def __enter__(self) -> list:
        global _RECORDING
        if _RECORDING is not None:
            raise RuntimeError("recordings do not nest")
        _RECORDING = []
        return _RECORDING

    def __exit__(self, *exc) -> None:
        global _RECORDING
        _RECORDING = None


def bind(recorded: list) -> list:
    """(entry point, argument list) pairs of a recording, ready for `replay`."""
    lib = load()
    return [(getattr(lib, name), name, args) for name, args in recorded]


def replay(bound: list) -> None:
    """Run a bound recording in order; raise QDError at the first non-zero status."""
    for fn, name, args in bound:
        rc = fn(*args)
        if rc != QD_OK:
            raise QDError(name, rc, load().qd_last_error().decode(errors="replace"))


def describe_device_error(code: int) -> str:
    return ", ".join(msg for bit, msg in DEVERR.items() if code & bit) or f"unknown ({code})"
