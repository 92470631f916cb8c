"""Python wrappers over the C ABI, shaped like the reference's kernel wrapper classes.

  pack_matrix / PackedMatrix   engine/engine.py:255-282 (weight packing)
  embed                        engine/kernels/fast.py:73-76 (embed_ss)
  Gemv                         engine/kernels/fast.py:173-213 (FastGemm) / gemv.py:157-248 (Gemv)
  QkvRopeAppend                FastGemm "qkv" + the q/k-norm/RoPE/KV-append of FastAttention (fast.py:240-293)
  LmHeadArgmax                 engine/kernels/fast.py:439-465 (FastLmHead) / gemv.py:251-287
  DecodeAttention              engine/kernels/decode_attn.py:89-119 / FastAttention (fast.py:353-376)
  DecodeAttentionStream        the same, streamed stream-K over all (sequence, KV head) chunks (large batch)
  DecodeAttentionTc            the same with q.k and P.V on tcgen05 tensor cores
  DecodeStep                   the persistent whole-step kernel (engine/kernels/mega.py MegaStep, tier T6)
  PackedActivations, TcGemv, TcQkvRopeAppend, TcLmHeadArgmax
                               FastGemm / FastLmHead at 9..64 rows (fast.py:173-213, :439-465) on tcgen05

Each object owns its scratch buffer (split-K partials and tickets, zero-filled once) and launches
on the current torch CUDA stream, so calls are graph-capturable. Tensors must be CUDA tensors.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import lib as L

BF16 = torch.bfloat16


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _check_bf16(*ts):
    for t in ts:
        if t is not None:
            assert t.is_cuda and t.dtype == BF16, f"expected a CUDA BF16 tensor, got {t.dtype} on {t.device}"


def sm_count() -> int:
    n = ctypes.c_int(0)
    L.call("qd_sm_count", ctypes.byref(n))
    return n.value


# ------------------------------------------------------------------------------------ packing
def packed_rows(n: int) -> int:
    return (n + 127) // 128 * 128


def new_packed(n_rows: int, k: int, device, count: int | None = None) -> torch.Tensor:
    """Uninitialised packed storage for one matrix [n_rows, k] (or `count` stacked matrices)."""
    elems = packed_rows(n_rows) * k
    shape = (elems,) if count is None else (count, elems)
    return torch.zeros(shape, dtype=BF16, device=device)


def pack_rows(src: torch.Tensor, dst: torch.Tensor, n_dst_rows: int, span: int | None = None,
              group_stride: int = 0, row_offset: int = 0) -> None:
    """Copy row-major src [n, k] into rows (j // span) * group_stride + row_offset + j % span of the
    packed destination (a flat BF16 tensor holding [n_dst_rows, k])."""
    _check_bf16(src, dst)
    n, k = src.shape
    assert src.stride(1) == 1
    L.call("qd_pack_rows", _ptr(src), src.stride(0), n, k, _ptr(dst), n_dst_rows, span or n, group_stride,
           row_offset, _stream())


def pack_matrix(w: torch.Tensor) -> torch.Tensor:
    """Packed copy of a row-major [n, k] weight (rows padded to a multiple of 128 with zeros)."""
    n, k = w.shape
    out = new_packed(n, k, w.device)
    pack_rows(w.contiguous(), out, packed_rows(n))
    return out


def pack_gate_up(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Gate/up matrix packed interleaved for the SwiGLU epilogue: each 128-row group holds 64 gate rows
    followed by the 64 up rows of the same outputs."""
    inter, k = gate.shape
    assert up.shape == gate.shape and inter % 64 == 0
    if out is None:
        out = new_packed(2 * inter, k, gate.device)
    pack_rows(gate.contiguous(), out, 2 * inter, 64, 128, 0)
    pack_rows(up.contiguous(), out, 2 * inter, 64, 128, 64)
    return out


# ------------------------------------------------------------------------------------ kernels
class _ErrWord:
    """Device int32 word the kernels OR their bounded-wait / token-range failures into."""

    def __init__(self, device):
        self.t = torch.zeros((1,), dtype=torch.int32, device=device)

    @property
    def ptr(self):
        return _ptr(self.t)


def embed(tok: torch.Tensor, e_packed: torch.Tensor, vocab: int, x: torch.Tensor, err: torch.Tensor | None = None,
          pdl: bool = True) -> torch.Tensor:
    """x[i] = E[tok[i]] (tok int64 [m], x [m, k] BF16)."""
    assert tok.dtype == torch.int64 and tok.is_cuda
    m, k = x.shape
    L.call("qd_embed", _ptr(tok), _ptr(e_packed), vocab, k, m, _ptr(x), x.stride(0), _ptr(err), int(pdl), _stream())
    return x


class Gemv:
    """out[m, :] (+epilogue) = norm?(x)[m, k] @ W^T for a packed W [n, k]; see qd_gemv."""

    STORE, RES, SWIGLU = L.QD_EPI_STORE, L.QD_EPI_RES, L.QD_EPI_SWIGLU

    def __init__(self, m: int, n: int, k: int, epilogue: int, device, grid: int = 0, eps: float = 1e-6):
        self.m, self.n, self.k, self.epilogue, self.eps = m, n, k, epilogue, eps
        g, nbytes = ctypes.c_int(0), ctypes.c_int64(0)
        L.call("qd_gemv_plan", n, k, m, grid, ctypes.byref(g), ctypes.byref(nbytes))
        self.grid = g.value
        self.scratch = torch.zeros((max(1, nbytes.value),), dtype=torch.uint8, device=device)

    def __call__(self, x, w, out, res=None, norm_w=None, err=None, pdl=True):
        _check_bf16(x, w, out, res, norm_w)
        assert x.shape[0] == self.m and x.stride(1) == 1 and out.stride(1) == 1
        L.call("qd_gemv", _ptr(x), x.stride(0), _ptr(w), self.n, self.k, self.m, _ptr(out), out.stride(0),
               _ptr(res), res.stride(0) if res is not None else 0, _ptr(norm_w), self.eps, self.epilogue, self.grid,
               _ptr(self.scratch), self.scratch.numel(), _ptr(err), int(pdl), _stream())
        return out


class QkvRopeAppend:
    """Packed QKV projection of RMSNorm(x) with per-head q/k RMSNorm, RoPE at *pos and the K/V append."""

    def __init__(self, m: int, k: int, nq: int, nkv: int, device, grid: int = 0, eps: float = 1e-6):
        self.m, self.k, self.nq, self.nkv, self.eps = m, k, nq, nkv, eps
        self.n = (nq + 2 * nkv) * 128
        g, nbytes = ctypes.c_int(0), ctypes.c_int64(0)
        L.call("qd_gemv_plan", self.n, k, m, grid, ctypes.byref(g), ctypes.byref(nbytes))
        self.grid = g.value
        self.scratch = torch.zeros((max(1, nbytes.value),), dtype=torch.uint8, device=device)

    def __call__(self, x, w, norm_w, q_norm, k_norm, cos, sin, pos, q_out, k_cache, v_cache, raw_out=None,
                 err=None, pdl=True):
        _check_bf16(x, w, norm_w, q_norm, k_norm, cos, sin, q_out, k_cache, v_cache, raw_out)
        assert pos.dtype == torch.int64 and k_cache.stride(2) == 128 and k_cache.stride() == v_cache.stride()
        L.call("qd_qkv_rope_append", _ptr(x), x.stride(0), _ptr(w), self.k, self.m, _ptr(norm_w), self.eps,
               _ptr(q_norm), _ptr(k_norm), _ptr(cos), _ptr(sin), _ptr(pos), k_cache.shape[2], self.nq, self.nkv,
               _ptr(q_out),
               _ptr(k_cache), _ptr(v_cache), k_cache.stride(0), k_cache.stride(1), _ptr(raw_out), self.grid,
               _ptr(self.scratch), self.scratch.numel(), _ptr(err), int(pdl), _stream())
        return q_out


class LmHeadArgmax:
    """tok[m] = argmax(bf16(RMSNorm(x) @ E^T)) (lowest index on ties); optionally *pos += 1 and logits."""

    def __init__(self, m: int, vocab: int, k: int, device, grid: int = 0, eps: float = 1e-6):
        self.m, self.vocab, self.k, self.eps = m, vocab, k, eps
        g, nbytes = ctypes.c_int(0), ctypes.c_int64(0)
        L.call("qd_lm_head_plan", vocab, k, m, grid, ctypes.byref(g), ctypes.byref(nbytes))
        self.grid = g.value
        self.scratch = torch.zeros((max(1, nbytes.value),), dtype=torch.uint8, device=device)

    def __call__(self, x, e_packed, norm_w, tok, pos=None, inc_pos=False, logits=None, err=None, pdl=True):
        _check_bf16(x, e_packed, norm_w, logits)
        assert tok.dtype == torch.int64
        L.call("qd_lm_head_argmax", _ptr(x), x.stride(0), _ptr(e_packed), self.vocab, self.k, self.m, _ptr(norm_w),
               self.eps, _ptr(tok), _ptr(pos), int(inc_pos), _ptr(logits),
               logits.stride(0) if logits is not None else 0, self.grid, _ptr(self.scratch), self.scratch.numel(),
               _ptr(err), int(pdl), _stream())
        return tok


# ------------------------------------------------------------------ tensor-core batch path (16..64 rows)
TC_MIN_BATCH, TC_MAX_BATCH = 9, 64


def tc_n_pad(m: int) -> int:
    """Batch padded to the MMA N dimension (a multiple of 16, at most 64)."""
    assert 1 <= m <= TC_MAX_BATCH
    return (m + 15) // 16 * 16


class PackedActivations:
    """The activation operand of the tensor-core kernels: [k/64][n_pad][64] swizzled BF16 tiles, with the
    RMSNorm prologue applied while packing (qd_pack_act). Padding rows stay zero."""

    def __init__(self, m: int, k: int, device):
        self.m, self.k, self.n_pad = m, k, tc_n_pad(m)
        self.t = torch.zeros((k * self.n_pad,), dtype=BF16, device=device)

    def pack(self, x, norm_w=None, eps: float = 1e-6, pdl=True):
        _check_bf16(x, norm_w)
        assert x.shape == (self.m, self.k) and x.stride(1) == 1
        L.call("qd_pack_act", _ptr(x), x.stride(0), self.m, self.n_pad, self.k, _ptr(norm_w), eps, _ptr(self.t),
               int(pdl), _stream())
        return self

    def pack_res(self, x, sums, norm_w=None, eps: float = 1e-6, pdl=True):
        """x += the deferred residual sums of a RES_SUMS projection (qd_pack_act_res: x written back, the
        sums cleared), then pack as `pack` does."""
        _check_bf16(x, norm_w)
        assert x.shape == (self.m, self.k) and x.stride(1) == 1
        assert sums.dtype == torch.int64 and sums.is_contiguous() and sums.numel() >= self.m * self.k
        L.call("qd_pack_act_res", _ptr(x), x.stride(0), self.m, self.n_pad, self.k, _ptr(sums), _ptr(norm_w), eps,
               _ptr(self.t), int(pdl), _stream())
        return self


class _TcOp:
    def __init__(self, n_pad: int, n: int, k: int, device, grid: int = 0):
        g, nbytes = ctypes.c_int(0), ctypes.c_int64(0)
        L.call("qd_tc_gemv_plan", n, k, n_pad, grid, ctypes.byref(g), ctypes.byref(nbytes))
        self.grid = g.value
        self.scratch = torch.zeros((max(1, nbytes.value),), dtype=torch.uint8, device=device)


class TcGemv(_TcOp):
    """Gemv for 9..64 rows on the tensor cores; x comes packed (PackedActivations). With SWIGLU_PACKED
    `out` is the next projection's PackedActivations, written directly by the epilogue."""

    STORE, RES, SWIGLU, SWIGLU_PACKED = L.QD_EPI_STORE, L.QD_EPI_RES, L.QD_EPI_SWIGLU, L.QD_EPI_SWIGLU_PACKED
    RES_SUMS = L.QD_EPI_RES_SUMS  # `out` = int64 fixed-point sums [m, n], applied by PackedActivations.pack_res
    STORE_SUMS = L.QD_EPI_STORE_SUMS  # `out` = int64 fixed-point sums [m, n], applied by qkv_rope_sums

    def __init__(self, m: int, n: int, k: int, epilogue: int, device, grid: int = 0):
        self.m, self.n, self.k, self.epilogue, self.n_pad = m, n, k, epilogue, tc_n_pad(m)
        super().__init__(self.n_pad, n, k, device, grid)

    def __call__(self, xp: PackedActivations, w, out, res=None, err=None, pdl=True):
        if self.epilogue == self.SWIGLU_PACKED:
            assert isinstance(out, PackedActivations) and out.m == self.m and out.k == self.n // 2
            out = out.t
        if self.epilogue in (self.RES_SUMS, self.STORE_SUMS):
            assert out.dtype == torch.int64 and out.is_contiguous() and out.numel() >= self.m * self.n
            _check_bf16(w)
            L.call("qd_tc_gemv", _ptr(xp.t), self.n_pad, self.m, _ptr(w), self.n, self.k, _ptr(out), 0, None, 0,
                   self.epilogue, self.grid, _ptr(self.scratch), self.scratch.numel(), _ptr(err), int(pdl), _stream())
            return out
        _check_bf16(w, out, res)
        assert xp.m == self.m and xp.k == self.k and out.stride(-1) == 1
        ldo = out.stride(0) if out.dim() > 1 else 0
        L.call("qd_tc_gemv", _ptr(xp.t), self.n_pad, self.m, _ptr(w), self.n, self.k, _ptr(out), ldo,
               _ptr(res), res.stride(0) if res is not None else 0, self.epilogue, self.grid, _ptr(self.scratch),
               self.scratch.numel(), _ptr(err), int(pdl), _stream())
        return out


class TcQkvRopeAppend(_TcOp):
    """QkvRopeAppend for 9..64 rows on the tensor cores (the ln1 RMSNorm is applied when packing)."""

    def __init__(self, m: int, k: int, nq: int, nkv: int, device, grid: int = 0):
        self.m, self.k, self.nq, self.nkv, self.n_pad = m, k, nq, nkv, tc_n_pad(m)
        self.n = (nq + 2 * nkv) * 128
        super().__init__(self.n_pad, self.n, k, device, grid)

    def __call__(self, xp: PackedActivations, w, q_norm, k_norm, cos, sin, pos, q_out, k_cache, v_cache,
                 raw_out=None, err=None, pdl=True):
        _check_bf16(w, q_norm, k_norm, cos, sin, q_out, k_cache, v_cache, raw_out)
        assert xp.m == self.m and pos.dtype == torch.int64
        assert k_cache.stride(2) == 128 and k_cache.stride() == v_cache.stride()
        L.call("qd_tc_qkv_rope_append", _ptr(xp.t), self.n_pad, self.m, _ptr(w), self.k, _ptr(q_norm),
               _ptr(k_norm), _ptr(cos), _ptr(sin), _ptr(pos), k_cache.shape[2], self.nq, self.nkv, _ptr(q_out),
               _ptr(k_cache), _ptr(v_cache), k_cache.stride(0), k_cache.stride(1), _ptr(raw_out), self.grid,
               _ptr(self.scratch), self.scratch.numel(), _ptr(err), int(pdl), _stream())
        return q_out


class TcLmHeadArgmax(_TcOp):
    """LmHeadArgmax for 9..64 rows on the tensor cores (the final RMSNorm is applied when packing)."""

    def __init__(self, m: int, vocab: int, k: int, device, grid: int = 0):
        self.m, self.vocab, self.k, self.n_pad = m, vocab, k, tc_n_pad(m)
        super().__init__(self.n_pad, packed_rows(vocab), k, device, grid)

    def __call__(self, xp: PackedActivations, e_packed, tok, pos=None, inc_pos=False, logits=None, err=None,
                 pdl=True):
        _check_bf16(e_packed, logits)
        assert xp.m == self.m and tok.dtype == torch.int64
        L.call("qd_tc_lm_head_argmax", _ptr(xp.t), self.n_pad, self.m, _ptr(e_packed), self.vocab, self.k,
               _ptr(tok), _ptr(pos), int(inc_pos), _ptr(logits), logits.stride(0) if logits is not None else 0,
               self.grid, _ptr(self.scratch), self.scratch.numel(), _ptr(err), int(pdl), _stream())
        return tok


# ------------------------------------------------------------------------------------ prompt (prefill)
def tc_gemm(x, w, n: int, out, res=None, epilogue: int = L.QD_EPI_STORE, err=None, scratch=None):
    """out = epilogue(x @ W^T) on the tensor cores for any number of token rows (qd_tc_gemm): x [m, k]
    BF16 (unit column stride), W packed [n, k]; SWIGLU writes n / 2 columns. `scratch` (uint8, at least
    tc_gemm_plan's bytes, any contents) is needed when the plan splits K; without one a buffer is allocated."""
    _check_bf16(x, w, out, res)
    m, k = x.shape
    assert x.stride(1) == 1 and out.stride(1) == 1 and out.shape[0] == m
    need = tc_gemm_plan(m, n, k)[3]
    if need and (scratch is None or scratch.numel() < need):
        scratch = torch.empty((need,), dtype=torch.uint8, device=x.device)
    L.call("qd_tc_gemm", _ptr(x), x.stride(0), m, _ptr(w), n, k, _ptr(out), out.stride(0), _ptr(res),
           res.stride(0) if res is not None else 0, epilogue, _ptr(scratch) if need else None,
           scratch.numel() if need else 0, _ptr(err), _stream())
    return out


def tc_gemm_plan(m: int, n: int, k: int) -> tuple[int, int, int, int]:
    """(grid, tile width, K split, scratch bytes) of qd_tc_gemm for this shape."""
    g, bn, ks, nb = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int64(0)
    L.call("qd_tc_gemm_plan", m, n, k, ctypes.byref(g), ctypes.byref(bn), ctypes.byref(ks), ctypes.byref(nb))
    return g.value, bn.value, ks.value, nb.value


def rmsnorm_rows(x, w, eps: float, out):
    """out = Qwen3RMSNorm(x) row by row (qd_rmsnorm_rows)."""
    _check_bf16(x, w, out)
    m, k = x.shape
    assert x.stride(1) == 1 and out.stride(1) == 1
    L.call("qd_rmsnorm_rows", _ptr(x), x.stride(0), m, k, _ptr(w), eps, _ptr(out), out.stride(0), _stream())
    return out


def tree_qk_rope(qkv, B: int, T: int, slot0, rope_pos, nq: int, nkv: int, q_norm, k_norm, eps: float, cos, sin,
                 q_out, k_cache, v_cache, err=None):
    """q/k RMSNorm + RoPE of the T token-tree nodes of each of B sequences (qd_tree_qk_rope): row b * T + t
    rotated at rope_pos[row] (device int32 [B * T]), its K/V at slot slot0[b] + t (device int32 [B]) of
    sequence b. qkv [B * T, (nq + 2 nkv) * 128]; q_out [B * T, nq * 128]; caches [B, nkv, cap, 128]."""
    _check_bf16(qkv, q_norm, k_norm, cos, sin, q_out, k_cache, v_cache)
    assert rope_pos.dtype == torch.int32 and rope_pos.numel() >= B * T
    assert slot0.dtype == torch.int32 and slot0.numel() >= B
    assert k_cache.dim() == 4 and k_cache.shape[0] >= B and k_cache.stride() == v_cache.stride()
    L.call("qd_tree_qk_rope", _ptr(qkv), qkv.stride(0), B, T, _ptr(slot0), _ptr(rope_pos), nq, nkv, _ptr(q_norm),
           _ptr(k_norm), eps, _ptr(cos), _ptr(sin), _ptr(q_out), q_out.stride(0), _ptr(k_cache), _ptr(v_cache),
           k_cache.shape[-2], k_cache.stride(0), k_cache.stride(1), _ptr(err), _stream())


def tree_attn(q, B: int, T: int, nq: int, nkv: int, k_cache, v_cache, prefix, anc, out, err=None):
    """Ancestor-masked attention of the T token-tree nodes of each of B sequences (qd_tree_attn): q / out
    [B * T, nq * 128]; caches [B, nkv, cap, 128]; prefix device int32 [B] (each tree's root slot); anc
    device uint32 [B * T] (passed as int32)."""
    _check_bf16(q, k_cache, v_cache, out)
    assert anc.dtype == torch.int32 and anc.numel() >= B * T and prefix.dtype == torch.int32 and prefix.numel() >= B
    assert k_cache.dim() == 4 and k_cache.shape[0] >= B and k_cache.stride() == v_cache.stride()
    L.call("qd_tree_attn", _ptr(q), q.stride(0), B, T, nq, nkv, _ptr(k_cache), _ptr(v_cache), k_cache.shape[-2],
           k_cache.stride(0), k_cache.stride(1), _ptr(prefix), _ptr(anc), 1.0 / math.sqrt(128), _ptr(out),
           out.stride(0), _ptr(err), _stream())
    return out


def tree_attn_rows(q, T: int, pos0: int, anc, nq: int, nkv: int, k_cache, v_cache, out, err=None):
    """Ancestor-masked attention of one sequence's T tree rows on the tensor cores (qd_tree_attn_rows):
    node t at slot pos0 + t; q / out [T, nq * 128]; caches [nkv, cap, 128]; anc device uint32 [T] (int32)."""
    _check_bf16(q, k_cache, v_cache, out)
    assert anc.dtype == torch.int32 and anc.numel() >= T and k_cache.stride() == v_cache.stride()
    L.call("qd_tree_attn_rows", _ptr(q), q.stride(0), pos0 + T, pos0, _ptr(anc), nq, nkv, _ptr(k_cache), _ptr(v_cache),
           k_cache.shape[-2], k_cache.stride(-3), 1.0 / math.sqrt(128), _ptr(out), out.stride(0), _ptr(err), _stream())
    return out


def tree_compact(k_all, v_all, moves, n: int):
    """Move the accepted paths' K/V rows of every layer (qd_tree_compact): caches [layers, B, nkv, cap, 128];
    moves device int32 [n, 3] (sequence, source slot, destination slot), applied in order."""
    _check_bf16(k_all, v_all)
    assert k_all.dim() == 5 and k_all.stride() == v_all.stride() and moves.dtype == torch.int32
    L.call("qd_tree_compact", _ptr(k_all), _ptr(v_all), k_all.shape[0], k_all.stride(0), k_all.shape[1],
           k_all.stride(1), k_all.shape[2], k_all.stride(2), k_all.shape[3], _ptr(moves), n, _stream())


def qkv_rope_sums(sums, m: int, nq: int, nkv: int, q_norm, k_norm, eps: float, cos, sin, pos, q_out, k_cache,
                  v_cache, err=None, pdl=True):
    """The QKV epilogue applied to a STORE_SUMS projection's fixed-point sums (qd_qkv_rope_sums), which
    it clears: q_out [m, nq, 128]; K/V appended at *pos into caches [B, nkv, cap, 128]."""
    _check_bf16(q_norm, k_norm, cos, sin, q_out, k_cache, v_cache)
    assert sums.dtype == torch.int64 and sums.stride(-1) == 1 and pos.dtype == torch.int64
    assert k_cache.stride(2) == 128 and k_cache.stride() == v_cache.stride()
    L.call("qd_qkv_rope_sums", _ptr(sums), sums.stride(0), m, nq, nkv, _ptr(q_norm), _ptr(k_norm), eps, _ptr(cos),
           _ptr(sin), _ptr(pos), k_cache.shape[2], _ptr(q_out), _ptr(k_cache), _ptr(v_cache), k_cache.stride(0),
           k_cache.stride(1), _ptr(err), int(pdl), _stream())
    return q_out


def argmax_rows(logits, n: int, out):
    """out[i] = index of the largest of logits[i, :n], lowest index on exact ties (qd_argmax_rows).
    logits [rows, ld] BF16 with unit column stride; out int64 [rows]."""
    _check_bf16(logits)
    assert logits.stride(1) == 1 and out.dtype == torch.int64 and out.is_contiguous()
    rows = logits.shape[0]
    assert out.numel() >= rows and n <= logits.shape[1]
    L.call("qd_argmax_rows", _ptr(logits), logits.stride(0), n, rows, _ptr(out), _stream())
    return out


def prefill_qk_rope(qkv, batch: int, S: int, nq: int, nkv: int, q_norm, k_norm, eps: float, cos, sin, q_out,
                    k_cache, v_cache, pos0: int = 0):
    """q/k RMSNorm + RoPE of the positions pos0..pos0+S-1, K/V into the caches (qd_prefill_qk_rope, or
    qd_prefill_qk_rope_at when pos0 > 0). qkv [batch * S, (nq + 2 nkv) * 128]; q_out [batch * S, nq * 128];
    caches [batch, nkv, cap, 128]."""
    _check_bf16(qkv, q_norm, k_norm, cos, sin, q_out, k_cache, v_cache)
    assert k_cache.stride() == v_cache.stride() and qkv.stride(1) == 1 and q_out.stride(1) == 1
    L.call("qd_prefill_qk_rope_at", _ptr(qkv), qkv.stride(0), batch, S, pos0, nq, nkv, _ptr(q_norm), _ptr(k_norm),
           eps, _ptr(cos), _ptr(sin), _ptr(q_out), q_out.stride(0), _ptr(k_cache), _ptr(v_cache), k_cache.shape[2],
           k_cache.stride(0), k_cache.stride(1), _stream())
    return q_out


def prefill_attn(q, batch: int, S: int, nq: int, nkv: int, k_cache, v_cache, out, q_begin: int = 0, err=None,
                 q_rows: bool = False):
    """Causal GQA attention of the positions q_begin..S-1 over the cached keys 0..s (qd_prefill_attn):
    q [batch * S, nq * 128] token-major, or with q_rows only the computed rows [batch * (S - q_begin), nq * 128]
    (qd_prefill_attn_rows); out [batch * (S - q_begin), nq * 128]."""
    _check_bf16(q, k_cache, v_cache, out)
    assert k_cache.stride() == v_cache.stride() and q.stride(1) == 1 and out.stride(1) == 1
    L.call("qd_prefill_attn_rows" if q_rows else "qd_prefill_attn", _ptr(q), q.stride(0), batch, S, q_begin, nq, nkv,
           _ptr(k_cache), _ptr(v_cache),
           k_cache.shape[2], k_cache.stride(0), k_cache.stride(1), 1.0 / math.sqrt(128), _ptr(out), out.stride(0),
           _ptr(err), _stream())
    return out


class DecodeAttention:
    """Split-K GQA flash-decode + LSE merge for a fixed (batch, capacity); see qd_attn_decode."""

    def __init__(self, batch: int, nq: int, nkv: int, capacity: int, device, grid: int = 0):
        self.batch, self.nq, self.nkv, self.capacity = batch, nq, nkv, capacity
        s, ch, nbytes = ctypes.c_int(0), ctypes.c_int64(0), ctypes.c_int64(0)
        L.call("qd_attn_plan", batch, nkv, capacity, grid, ctypes.byref(s), ctypes.byref(ch), ctypes.byref(nbytes))
        self.splits, self.chunk = s.value, ch.value
        self.scratch = torch.zeros((max(1, nbytes.value),), dtype=torch.uint8, device=device)
        self.scale = 1.0 / math.sqrt(128)

    def __call__(self, q, k_cache, v_cache, pos, out, err=None, pdl=True):
        _check_bf16(q, k_cache, v_cache, out)
        assert k_cache.shape[2] == self.capacity and k_cache.stride() == v_cache.stride()
        L.call("qd_attn_decode", _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(pos), _ptr(out), self.batch, self.nq,
               self.nkv, self.capacity, k_cache.stride(0), k_cache.stride(1), self.splits, self.chunk, self.scale,
               _ptr(self.scratch), self.scratch.numel(), _ptr(err), int(pdl), _stream())
        return out


class TcDecodeStep:
    """Persistent tcgen05 decode step (qd_tc_decode_step) for batches of 4..64: one launch per step over
    the engine's packed weights, with the state's packed activation operands (xp_h, xp_a, xp_i)."""

    def __init__(self, eng, st, logits=None, trace=None):
        self.desc = _step_desc(eng, st, logits, trace)
        self._keep = (eng, st, logits, trace)
        nbytes, npad = ctypes.c_int64(0), ctypes.c_int(0)
        L.call("qd_tc_decode_step_plan", ctypes.byref(self.desc), ctypes.byref(nbytes), ctypes.byref(npad))
        assert npad.value == st.xp_h.n_pad
        self.ptrs = (_ptr(st.xp_h.t), _ptr(st.xp_a.t), _ptr(st.xp_i.t))
        self.scratch = torch.zeros((max(1, nbytes.value),), dtype=torch.uint8, device=st.x.device)

    def __call__(self):
        L.call("qd_tc_decode_step", ctypes.byref(self.desc), *self.ptrs, _ptr(self.scratch), self.scratch.numel(),
               _stream())

    def reset(self):
        self.scratch.zero_()


class DecodeAttentionStream:
    """Streaming split-K GQA flash-decode (qd_attn_decode_stream): chunks of every (sequence, KV head)
    dealt out evenly over the CTAs; the large-batch / long-cache counterpart of DecodeAttention."""

    PLAN, RUN = "qd_attn_stream_plan", "qd_attn_decode_stream"

    def __init__(self, batch: int, nq: int, nkv: int, capacity: int, device, grid: int = 0):
        self.batch, self.nq, self.nkv, self.capacity = batch, nq, nkv, capacity
        g, sm, nbytes = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int64(0)
        L.call(self.PLAN, batch, nkv, capacity, grid, ctypes.byref(g), ctypes.byref(sm), ctypes.byref(nbytes))
        self.grid, self.smax = g.value, sm.value
        self.scratch = torch.zeros((max(1, nbytes.value),), dtype=torch.uint8, device=device)
        self.scale = 1.0 / math.sqrt(128)

    def __call__(self, q, k_cache, v_cache, pos, out, err=None, pdl=True):
        _check_bf16(q, k_cache, v_cache, out)
        assert k_cache.shape[2] == self.capacity and k_cache.stride() == v_cache.stride()
        L.call(self.RUN, _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(pos), _ptr(out), self.batch,
               self.nq, self.nkv, self.capacity, k_cache.stride(0), k_cache.stride(1), self.grid, self.smax,
               self.scale, _ptr(self.scratch), self.scratch.numel(), _ptr(err), int(pdl), _stream())
        return out


class DecodeAttentionTc(DecodeAttentionStream):
    """The same on the tensor cores (qd_attn_decode_tc): q.k and P.V as tcgen05 MMAs per 128-key chunk.
    `out` is a [B, nq, 128] tensor or a PackedActivations (the O projection's operand, written directly)."""

    PLAN, RUN = "qd_attn_tc_plan", "qd_attn_decode_tc"

    def __call__(self, q, k_cache, v_cache, pos, out, err=None, pdl=True):
        packed = isinstance(out, PackedActivations)
        _check_bf16(q, k_cache, v_cache, out.t if packed else out)
        assert k_cache.shape[2] == self.capacity and k_cache.stride() == v_cache.stride()
        if packed:
            assert out.m == self.batch and out.k == self.nq * 128
        L.call(self.RUN, _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(pos), _ptr(out.t if packed else out),
               out.n_pad if packed else 0, self.batch, self.nq, self.nkv, self.capacity, k_cache.stride(0),
               k_cache.stride(1), self.grid, self.smax, self.scale, _ptr(self.scratch), self.scratch.numel(),
               _ptr(err), int(pdl), _stream())
        return out


def _step_desc(eng, st, logits=None, trace=None):
    """qd_step_desc over the engine's packed weights and one shape state."""
    d = L.StepDesc()
    Lyr = eng.n_layers
    d.w_qkv, d.w_qkv_layer_bytes = eng.w_qkv.data_ptr(), eng.w_qkv.stride(0) * 2
    d.w_o, d.w_o_layer_bytes = eng.w_o.data_ptr(), eng.w_o.stride(0) * 2
    d.w_gu, d.w_gu_layer_bytes = eng.w_gu.data_ptr(), eng.w_gu.stride(0) * 2
    d.w_down, d.w_down_layer_bytes = eng.w_down.data_ptr(), eng.w_down.stride(0) * 2
    d.e_packed = eng.e_packed.data_ptr()
    d.ln1, d.ln2 = eng.ln1.data_ptr(), eng.ln2.data_ptr()
    d.q_norm, d.k_norm, d.final_norm = eng.qn.data_ptr(), eng.kn.data_ptr(), eng.final_norm.data_ptr()
    d.layers, d.hidden, d.inter = Lyr, eng.hidden, eng.inter
    d.nq_heads, d.nkv_heads, d.vocab, d.batch = eng.nq, eng.nkv, eng.vocab, st.B
    d.eps, d.scale = eng.eps, 1.0 / math.sqrt(eng.head_dim)
    d.tok, d.pos = st.tok.data_ptr(), st.pos.data_ptr()
    d.x, d.q, d.attn, d.act = st.x.data_ptr(), st.q.data_ptr(), st.attn_out.data_ptr(), st.act.data_ptr()
    d.k_cache, d.v_cache = st.k_all.data_ptr(), st.v_all.data_ptr()
    d.cache_layer_stride, d.cs_b, d.cs_h = st.k_all.stride(0), st.k_all.stride(1), st.k_all.stride(2)
    d.cap = st.k_all.shape[3]
    d.cos, d.sin = st.cos.data_ptr(), st.sin.data_ptr()
    d.logits = logits.data_ptr() if logits is not None else None
    d.ld_logits = logits.stride(0) if logits is not None else 0
    d.err = st.err.data_ptr()
    d.trace = trace.data_ptr() if trace is not None else None
    return d


class DecodeStep:
    """One persistent launch per decode step (qd_decode_step): embedding, every layer and the LM head.
    Holds the descriptor (pointers into the engine's weights and per-shape state) and the scratch."""

    def __init__(self, eng, st, logits=None, trace=None):
        d = self.desc = _step_desc(eng, st, logits, trace)
        self._keep = (eng, st, logits, trace)
        nbytes, splits = ctypes.c_int64(0), ctypes.c_int(0)
        L.call("qd_decode_step_plan", ctypes.byref(d), ctypes.byref(nbytes), ctypes.byref(splits))
        self.splits = splits.value
        self.scratch = torch.zeros((max(1, nbytes.value),), dtype=torch.uint8, device=st.x.device)

    def __call__(self):
        L.call("qd_decode_step", ctypes.byref(self.desc), _ptr(self.scratch), self.scratch.numel(), _stream())

    def reset(self):
        """Clear counters / tickets after a device error (they are left mid-step)."""
        self.scratch.zero_()
