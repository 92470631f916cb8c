"""Qwen3 greedy decode engine for NVIDIA B200 (sm_100a).

Drop-in for the reference's `engine/engine.py`: the same `Engine(model_path)` constructor and
`generate(input_ids, max_new_tokens)` generator (engine/engine.py:232-293, :1105-1132; contract in
QWEN_ENGINE_CONTRACT.md): it yields exactly `max_new_tokens` lists, one token id per sequence in
input order, ignores end-of-sequence ids, and yields nothing for max_new_tokens <= 0.

Decode runs entirely in the hand-written CUDA library (decode_b200/libqd_decode.so, C ABI in
include/qd_decode.h); there is no Triton, no tier fallback and no CPU path. By default a decode step
is one persistent launch (qd_decode_step: one CTA per SM streams every weight block in op order while
its consumers wait on completion counters); ENGINE_STEP=kernels runs the same arithmetic as
1 + 5 x layers + 1 launches. Either way the step is captured once per shape in a CUDA graph:

  embed          x = E[tok]
  per layer      qkv   RMSNorm(x) @ Wqkv^T, per-head q/k RMSNorm + RoPE(pos), K/V appended at pos
                 attn  split-K GQA flash-decode over [0, pos] + log-sum-exp merge
                 o     x = bf16(x + bf16(attn @ Wo^T))
                 gu    act = bf16(silu(bf16 g)) * bf16 u with g, u = RMSNorm(x) @ [Wg; Wu]^T
                 down  x = bf16(x + bf16(act @ Wd^T))
  lm head        tok = argmax(bf16(RMSNorm(x) @ E^T)), pos += 1

Weights are packed once at load into the kernels' blocked layout (decode_b200/ops.py), the only copy
kept. The prompt forward (prefill, engine/engine.py:550-592) runs on the same packed weights through
the library's tcgen05 GEMM (qd_tc_gemm, fused residual / SwiGLU epilogues), row RMSNorm, prompt
q/k-norm + RoPE + KV-cache kernel and tcgen05 causal flash attention (qd_prefill_attn). It is
captured in a CUDA graph too. Tokens reach the host through a ring of pinned slots (`_TokenRing`): the
GPU runs up to ENGINE_AHEAD decode steps ahead of the caller, who gets each step's token list as soon as
its copy has landed (the reference's stream loop, engine/engine.py:719-757, keeps one step ahead).
"""

from __future__ import annotations

import contextlib
import gc
import os
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from decode_b200 import lib as qdlib  # noqa: E402
from decode_b200 import ops  # noqa: E402
from decode_b200 import spec  # noqa: E402
from decode_b200 import tree as tree_spec  # noqa: E402
from decode_b200.loader import load_checkpoint  # noqa: E402

DEVICE = os.environ.get("ENGINE_DEVICE", "cuda:0")
BF16 = torch.bfloat16
MAX_BATCH = 8             # the streaming GEMV keeps up to 8 activation rows in registers
TC_MAX_BATCH = ops.TC_MAX_BATCH  # larger batches run the tcgen05 kernels (batch padded to 16/32/48/64)
# From this batch up the tcgen05 kernel chain beats the CUDA-core persistent step on B200 (measured:
# tie at batch 4 with a 128-token prompt, tc ahead at 4 with 1024 and at 8 by 1.5-1.7x).
TC_MIN_BATCH = int(os.environ.get("ENGINE_TC_MIN_BATCH", "4"))
# tensor-core path: "persistent" = one qd_tc_decode_step launch per step; "chain" = the per-op kernels;
# "auto" = persistent up to TC_PERSISTENT_MAX_BATCH (measured: 9 % faster at batch 8, 2 % slower at 16 and
# 17 % slower at 64, where its attention has two K/V stages to the chain kernel's three)
TC_STEP = os.environ.get("ENGINE_TC_STEP", "auto")
TC_PERSISTENT_MAX_BATCH = int(os.environ.get("ENGINE_TC_PERSISTENT_MAX_BATCH", "12"))
PREFILL_TOKENS = 16384    # prefill processes at most this many tokens per row chunk (engine/engine.py:79)
USE_GRAPHS = os.environ.get("ENGINE_GRAPHS", "1") != "0"
USE_PDL = os.environ.get("ENGINE_PDL", "1") != "0"
# exact prompt-lookup speculative decoding at batch 1: verify width T = k + 1 (0 = off; the reference's
# default at batch 1 is 7, engine/engine.py:162)
SPEC_T = int(os.environ.get("ENGINE_SPEC_T", "0"))
# while drafts are not accepted often enough to pay for a verify, fall back to plain decode steps
SPEC_GATE = os.environ.get("ENGINE_SPEC_GATE", "1") != "0"
# exact token-tree speculative decoding: tree nodes per sequence and verify (0 = off), at most
# TREE_MAX_ROWS // batch of them (the reference's rule: 32 nodes up to batch 2, fewer per sequence above,
# no trees past batch 32, engine/engine.py:166-172), and their deepest level (engine/engine.py:833)
TREE_T = int(os.environ.get("ENGINE_TREE_T", "0"))
TREE_DEPTH = int(os.environ.get("ENGINE_TREE_DEPTH", "12"))
TREE_MAX_ROWS = 64
# the tree attention of a single sequence: "tc" = the tensor-core prompt attention with the ancestor mask
# (qd_tree_attn_rows), "cuda" = the CUDA-core kernel that batches of trees use (qd_tree_attn)
TREE_ATTN = os.environ.get("ENGINE_TREE_ATTN", "tc")
# "persistent": one launch per decode step (qd_decode_step); "kernels": 1 + 5 x layers + 1 launches;
# "tc": the tensor-core kernels (used from TC_MIN_BATCH up): one persistent launch per step, or the
# chain of 1 + 7 x layers + 2 launches (TC_STEP)
STEP_MODE = os.environ.get("ENGINE_STEP", "persistent")
# decode steps the GPU may have queued beyond the one whose tokens the caller is waiting for
AHEAD = max(1, int(os.environ.get("ENGINE_AHEAD", "2")))


def log(msg):
    print(f"[engine] {msg}", file=sys.stderr, flush=True)


def rope_tables(cap: int, head_dim: int, theta: float):
    """cos, sin [cap, head_dim] BF16, computed on the CPU exactly as transformers'
    Qwen3RotaryEmbedding does (fp32 inv_freq, fp32 matmul, cat(freqs, freqs), cos/sin, cast)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim))
    pos = torch.arange(cap)[None]
    freqs = (inv_freq[None, :, None].float() @ pos[:, None, :].float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos()[0].to(BF16).contiguous(), emb.sin()[0].to(BF16).contiguous()


class _TokenRing:
    """Delivers each decode step's token vector from the device to the host.

    `post` enqueues, on the current stream, a copy of the device token vector into the next pinned
    slot and records an event behind it; `take` waits for the oldest posted copy and returns it as a
    list. A ring of `slots` slots lets the device run up to slots - 1 steps ahead of the host; a slot is
    reused only after `take` has read it."""

    def __init__(self, batch: int, slots: int, pin: bool):
        self.buf = torch.empty((slots, batch), dtype=torch.int64, pin_memory=pin)
        self.landed = [torch.cuda.Event() for _ in range(slots)]
        self.posted = self.taken = 0

    def reset(self) -> None:
        self.posted = self.taken = 0

    def in_flight(self) -> int:
        return self.posted - self.taken

    def post(self, tok: torch.Tensor) -> None:
        if self.in_flight() == len(self.landed):
            raise RuntimeError("token ring overrun: take() before posting more steps")
        i = self.posted % len(self.landed)
        self.buf[i].copy_(tok, non_blocking=True)
        self.landed[i].record()
        self.posted += 1

    def take(self) -> list[int]:
        i = self.taken % len(self.landed)
        self.landed[i].synchronize()
        self.taken += 1
        return self.buf[i].tolist()


class _StepTimer:
    """Optional CUDA-event brackets around each enqueued step (prefill first), read after the run."""

    def __init__(self):
        self.pairs = []

    @contextlib.contextmanager
    def span(self):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        yield
        b.record()
        self.pairs.append((a, b))

    def ms(self) -> list[float]:
        return [a.elapsed_time(b) for a, b in self.pairs]


def prefill_chunks(batch: int, prompt_len: int, max_tokens: int) -> list[tuple[int, int]]:
    """Row ranges [r0, r1) of whole sequences for the prompt forward, each holding at most max_tokens
    tokens (or one sequence when a single prompt is longer), so a long batch runs as several forwards
    of bounded activation size (the reference bounds its prefill the same way, engine/engine.py:79)."""
    per = max(1, max_tokens // prompt_len)
    return [(r0, min(batch, r0 + per)) for r0 in range(0, batch, per)]


def _timed(timer: _StepTimer, fn, st) -> None:
    with timer.span():
        fn(st)


@contextlib.contextmanager
def _collector_paused():
    """Python's cyclic garbage collector paused while tokens stream: a collection pass on the caller's
    thread would delay the next launch. Restored to its previous state afterwards."""
    was_on = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if was_on:
            gc.enable()


class _State:
    """Everything shape-dependent for one (batch, prompt length, new tokens)."""

    def __init__(self, eng: "Engine", B: int, S: int, N: int, spec_T: int = 0, tree_T: int = 0):
        dev = eng.device
        self.B, self.S, self.N = B, S, N
        # a verify writes up to T - 1 slots past the last emitted token
        cap = self.capacity = S + N + max(spec_T, tree_T)
        Lyr, H, I = eng.n_layers, eng.hidden, eng.inter
        nq, nkv, D = eng.nq, eng.nkv, eng.head_dim
        self.k_all = torch.zeros((Lyr, B, nkv, cap, D), dtype=BF16, device=dev)
        self.v_all = torch.zeros((Lyr, B, nkv, cap, D), dtype=BF16, device=dev)
        cos, sin = rope_tables(cap, D, eng.theta)
        self.cos, self.sin = cos.to(dev), sin.to(dev)
        self.ids = torch.zeros((B, S), dtype=torch.int64, device=dev)
        self.tok = torch.zeros((B,), dtype=torch.int64, device=dev)
        self.pos = torch.zeros((1,), dtype=torch.int64, device=dev)
        self.err = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.x = torch.zeros((B, H), dtype=BF16, device=dev)
        self.q = torch.zeros((B, nq, D), dtype=BF16, device=dev)
        self.attn_out = torch.zeros((B, nq, D), dtype=BF16, device=dev)
        self.act = torch.zeros((B, I), dtype=BF16, device=dev)
        self.logits = None
        self.mode = "tc" if (B > MAX_BATCH or B >= TC_MIN_BATCH) else STEP_MODE
        if self.mode == "tc":
            self.attn = ops.DecodeAttentionTc(B, nq, nkv, cap, dev)
            # activation operands in the swizzled tile layout (RMSNorm applied while packing)
            self.xp_h = ops.PackedActivations(B, H, dev)
            self.xp_a = ops.PackedActivations(B, nq * D, dev)
            self.xp_i = ops.PackedActivations(B, I, dev)
            self.qkv = ops.TcQkvRopeAppend(B, H, nq, nkv, dev)
            # the residual projections leave fixed-point sums that the next packing applies
            self.o = ops.TcGemv(B, H, nq * D, ops.TcGemv.RES_SUMS, dev)
            self.gu = ops.TcGemv(B, 2 * I, H, ops.TcGemv.SWIGLU_PACKED, dev)
            self.down = ops.TcGemv(B, H, I, ops.TcGemv.RES_SUMS, dev)
            self.lm = ops.TcLmHeadArgmax(B, eng.vocab, H, dev)
            self.res_sums = torch.zeros((B, H), dtype=torch.int64, device=dev)
            # the chain's QKV: the projection into fixed-point sums, then the epilogue kernel
            self.qkv_mm = ops.TcGemv(B, (nq + 2 * nkv) * D, H, ops.TcGemv.STORE_SUMS, dev)
            self.qkv_sums = torch.zeros((B, (nq + 2 * nkv) * D), dtype=torch.int64, device=dev)
        else:
            self.attn = ops.DecodeAttention(B, nq, nkv, cap, dev)
            self.qkv = ops.QkvRopeAppend(B, H, nq, nkv, dev, eps=eng.eps)
            self.o = ops.Gemv(B, H, nq * D, ops.Gemv.RES, dev, eps=eng.eps)
            self.gu = ops.Gemv(B, 2 * I, H, ops.Gemv.SWIGLU, dev, eps=eng.eps)
            self.down = ops.Gemv(B, H, I, ops.Gemv.RES, dev, eps=eng.eps)
            self.lm = ops.LmHeadArgmax(B, eng.vocab, H, dev, eps=eng.eps)
        self.step = ops.DecodeStep(eng, self) if self.mode == "persistent" else None
        persistent_tc = TC_STEP == "persistent" or (TC_STEP == "auto" and B <= TC_PERSISTENT_MAX_BATCH)
        self.tstep = ops.TcDecodeStep(eng, self) if (self.mode == "tc" and persistent_tc) else None
        self.tstep_logits = None
        self.step_logits = None
        self.chunks = prefill_chunks(B, S, PREFILL_TOKENS)
        pin = torch.cuda.is_available()
        self.prompt_host = torch.empty((B, S), dtype=torch.int64, pin_memory=pin)  # staging of the prompt upload
        self.ring = _TokenRing(B, AHEAD + 1, pin)
        self.step_host = torch.empty((2,), dtype=torch.int64, pin_memory=pin)  # plain-step fallback: tok, pos
        self.prefill_graph = self.decode_graph = None
        self.prefill_logits = None
        self.verify = _Verify(eng, self, spec_T) if spec_T else None
        self.tree = _TreeVerify(eng, self, tree_T) if tree_T else None


class _Verify:
    """Speculative verify forward of one sequence (the reference's `_verify`, engine/engine.py:479-498):
    T tokens at positions pos0 .. pos0 + T - 1 after a cached prefix of pos0 tokens. The projections run
    on the decode GEMVs with the T tokens as activation rows (RMSNorm fused where the decode step fuses
    it); q/k RMSNorm + RoPE + the K/V of the T positions by qd_prefill_qk_rope_at; the T rows attend
    causally over the cache by qd_prefill_attn_rows; the LM head's argmax gives, for every row t, the
    greedy token after the prefix ending at row t."""

    def __init__(self, eng: "Engine", st: "_State", T: int):
        if not 2 <= T <= MAX_BATCH:
            raise ValueError(f"speculative verify width must be in [2, {MAX_BATCH}], got {T}")
        dev = eng.device
        H, I, nq, nkv, D, eps = eng.hidden, eng.inter, eng.nq, eng.nkv, eng.head_dim, eng.eps
        self.T = T
        n_qkv = (nq + 2 * nkv) * D
        self.tok = torch.zeros((T,), dtype=torch.int64, device=dev)
        self.out = torch.zeros((T,), dtype=torch.int64, device=dev)
        self.x = torch.zeros((T, H), dtype=BF16, device=dev)
        self.qkv = torch.zeros((T, n_qkv), dtype=BF16, device=dev)
        self.q = torch.zeros((T, nq * D), dtype=BF16, device=dev)
        self.att = torch.zeros((T, nq * D), dtype=BF16, device=dev)
        self.act = torch.zeros((T, I), dtype=BF16, device=dev)
        # projections as in decode at batch T: CUDA-core GEMVs below TC_MIN_BATCH rows, else the tcgen05
        # GEMVs on packed activations (RMSNorm applied while packing)
        self.tc = T >= TC_MIN_BATCH
        if self.tc:
            self.xp_h = ops.PackedActivations(T, H, dev)
            self.xp_a = ops.PackedActivations(T, nq * D, dev)
            self.xp_i = ops.PackedActivations(T, I, dev)
            self.qkv_op = ops.TcGemv(T, n_qkv, H, ops.TcGemv.STORE, dev)
            self.o = ops.TcGemv(T, H, nq * D, ops.TcGemv.RES, dev)
            self.gu = ops.TcGemv(T, 2 * I, H, ops.TcGemv.SWIGLU_PACKED, dev)
            self.down = ops.TcGemv(T, H, I, ops.TcGemv.RES, dev)
            self.lm = ops.TcLmHeadArgmax(T, eng.vocab, H, dev)
        else:
            self.qkv_op = ops.Gemv(T, n_qkv, H, ops.Gemv.STORE, dev, eps=eps)
            self.o = ops.Gemv(T, H, nq * D, ops.Gemv.RES, dev, eps=eps)
            self.gu = ops.Gemv(T, 2 * I, H, ops.Gemv.SWIGLU, dev, eps=eps)
            self.down = ops.Gemv(T, H, I, ops.Gemv.RES, dev, eps=eps)
            self.lm = ops.LmHeadArgmax(T, eng.vocab, H, dev, eps=eps)
        pin = torch.cuda.is_available()
        self.tok_host = torch.empty((T,), dtype=torch.int64, pin_memory=pin)
        self.out_host = torch.empty((T,), dtype=torch.int64, pin_memory=pin)
        self.event = torch.cuda.Event()
        self.calls = None  # the recorded launch sequence (its positions and stream are set per verify)

    def launch(self, eng: "Engine", st: "_State", pos0: int) -> None:
        """Enqueue the verify of self.tok at positions pos0 .. pos0 + T - 1 (the result lands in self.out).
        The ~6 x layers + 2 launches are recorded once through the wrappers and replayed from bound
        argument lists: only the positions (q/k RoPE, attention) and the stream change between verifies,
        and the replay costs a few microseconds of host time per launch instead of the wrappers' tens."""
        if self.calls is None:
            with qdlib.recording() as rec:
                self._enqueue(eng, st, 0)
            self.calls = qdlib.bind(rec)
            self.rope = [c[2] for c in self.calls if c[1] == "qd_prefill_qk_rope_at"]
            self.attn = [c[2] for c in self.calls if c[1] == "qd_prefill_attn_rows"]
            assert len(self.rope) == len(self.attn) == eng.n_layers
        stream = torch.cuda.current_stream().cuda_stream
        for args in self.rope:
            args[4] = pos0                 # pos0
        for args in self.attn:
            args[3], args[4] = pos0 + self.T, pos0  # S, q_begin
        for _, _, args in self.calls:
            args[-1] = stream
        qdlib.replay(self.calls)

    def _enqueue(self, eng: "Engine", st: "_State", pos0: int) -> None:
        T, nq, nkv, eps, err, pdl = self.T, eng.nq, eng.nkv, eng.eps, st.err, USE_PDL
        ops.embed(self.tok, eng.e_packed, eng.vocab, self.x, err, pdl)
        for i in range(eng.n_layers):
            kc, vc = st.k_all[i], st.v_all[i]
            if self.tc:
                self.xp_h.pack(self.x, eng.ln1[i], eps, pdl)
                self.qkv_op(self.xp_h, eng.w_qkv[i], self.qkv, err=err, pdl=pdl)
            else:
                self.qkv_op(self.x, eng.w_qkv[i], self.qkv, norm_w=eng.ln1[i], err=err, pdl=pdl)
            ops.prefill_qk_rope(self.qkv, 1, T, nq, nkv, eng.qn[i], eng.kn[i], eps, st.cos, st.sin, self.q, kc, vc,
                                pos0=pos0)
            ops.prefill_attn(self.q, 1, pos0 + T, nq, nkv, kc, vc, self.att, q_begin=pos0, err=err, q_rows=True)
            if self.tc:
                self.o(self.xp_a.pack(self.att, None, eps, pdl), eng.w_o[i], self.x, res=self.x, err=err, pdl=pdl)
                self.xp_h.pack(self.x, eng.ln2[i], eps, pdl)
                self.gu(self.xp_h, eng.w_gu[i], self.xp_i, err=err, pdl=pdl)
                self.down(self.xp_i, eng.w_down[i], self.x, res=self.x, err=err, pdl=pdl)
            else:
                self.o(self.att, eng.w_o[i], self.x, res=self.x, err=err, pdl=pdl)
                self.gu(self.x, eng.w_gu[i], self.act, norm_w=eng.ln2[i], err=err, pdl=pdl)
                self.down(self.act, eng.w_down[i], self.x, res=self.x, err=err, pdl=pdl)
        if self.tc:
            self.lm(self.xp_h.pack(self.x, eng.final_norm, eps, pdl), eng.e_packed, self.out, err=err, pdl=pdl)
        else:
            self.lm(self.x, eng.e_packed, eng.final_norm, self.out, err=err, pdl=pdl)

    def __call__(self, eng: "Engine", st: "_State", row: list[int], pos0: int) -> list[int]:
        """Greedy token after every prefix of `row` (T tokens at positions pos0 ..), on the host."""
        with torch.inference_mode():
            self.tok_host.copy_(torch.tensor(row, dtype=torch.int64))
            self.tok.copy_(self.tok_host, non_blocking=True)
            self.launch(eng, st, pos0)
            self.out_host.copy_(self.out, non_blocking=True)
            self.event.record()
        self.event.synchronize()
        return self.out_host.tolist()


class _TreeVerify:
    """Verify forward of one token tree per sequence (the reference's tree verify, engine/engine.py:418-462,
    830-936): the B x T nodes run as activation rows (row b * T + i = node i of sequence b) through the
    tcgen05 projections; node i's q/k are rotated at prefix[b] + depth(i) and its K/V written to slot
    prefix[b] + i of its sequence (qd_tree_qk_rope); every node attends to its sequence's cached prefix and
    to its ancestors (qd_tree_attn; for one sequence the tensor-core qd_tree_attn_rows); the LM head's
    argmax gives the greedy token at every node. After the walks, the accepted nodes' K/V move to
    consecutive slots (qd_tree_compact). The per-round inputs (tokens, positions, masks, prefixes) live in
    device buffers, so the ~8 x layers + 3 launches are recorded once and replayed, only the tensor-core
    tree attention's root slot (a host argument) patched per round."""

    def __init__(self, eng: "Engine", st: "_State", T: int):
        if not 2 <= T <= 32:
            raise ValueError(f"token-tree verify width must be in [2, 32], got {T}")
        B = st.B
        if B * T > TREE_MAX_ROWS:
            raise ValueError(f"token-tree verify of {B} x {T} rows > {TREE_MAX_ROWS}")
        dev = eng.device
        H, I, nq, nkv, D = eng.hidden, eng.inter, eng.nq, eng.nkv, eng.head_dim
        self.B, self.T, self.depth = B, T, max(1, min(TREE_DEPTH, T - 1))
        M = self.M = B * T
        n_qkv = (nq + 2 * nkv) * D
        self.tok = torch.zeros((M,), dtype=torch.int64, device=dev)
        # int32 inputs in one buffer (one upload): RoPE positions [M], ancestor masks [M], root slots [B]
        self.ints = torch.zeros((2 * M + B,), dtype=torch.int32, device=dev)
        self.rope_pos, self.anc, self.prefix = self.ints[:M], self.ints[M:2 * M], self.ints[2 * M:]
        self.moves = torch.zeros((M, 3), dtype=torch.int32, device=dev)
        self.out = torch.zeros((M,), dtype=torch.int64, device=dev)
        self.x = torch.zeros((M, H), dtype=BF16, device=dev)
        self.qkv = torch.zeros((M, n_qkv), dtype=BF16, device=dev)
        self.q = torch.zeros((M, nq * D), dtype=BF16, device=dev)
        self.att = torch.zeros((M, nq * D), dtype=BF16, device=dev)
        self.xp_h = ops.PackedActivations(M, H, dev)
        self.xp_a = ops.PackedActivations(M, nq * D, dev)
        self.xp_i = ops.PackedActivations(M, I, dev)
        self.qkv_op = ops.TcGemv(M, n_qkv, H, ops.TcGemv.STORE, dev)
        self.o = ops.TcGemv(M, H, nq * D, ops.TcGemv.RES, dev)
        self.gu = ops.TcGemv(M, 2 * I, H, ops.TcGemv.SWIGLU_PACKED, dev)
        self.down = ops.TcGemv(M, H, I, ops.TcGemv.RES, dev)
        self.lm = ops.TcLmHeadArgmax(M, eng.vocab, H, dev)
        pin = torch.cuda.is_available()
        self.tok_host = torch.zeros((M,), dtype=torch.int64, pin_memory=pin)
        self.ints_host = torch.zeros((2 * M + B,), dtype=torch.int32, pin_memory=pin)
        self.moves_host = torch.zeros((M, 3), dtype=torch.int32, pin_memory=pin)
        self.out_host = torch.zeros((M,), dtype=torch.int64, pin_memory=pin)
        self.event = torch.cuda.Event()
        self.calls = None
        self.rows_attn = B == 1 and TREE_ATTN == "tc"
        self.root1 = 0

    def _enqueue(self, eng: "Engine", st: "_State") -> None:
        B, T, nq, nkv, eps, err, pdl = self.B, self.T, eng.nq, eng.nkv, eng.eps, st.err, USE_PDL
        ops.embed(self.tok, eng.e_packed, eng.vocab, self.x, err, pdl)
        for i in range(eng.n_layers):
            kc, vc = st.k_all[i], st.v_all[i]
            self.xp_h.pack(self.x, eng.ln1[i], eps, pdl)
            self.qkv_op(self.xp_h, eng.w_qkv[i], self.qkv, err=err, pdl=pdl)
            ops.tree_qk_rope(self.qkv, B, T, self.prefix, self.rope_pos, nq, nkv, eng.qn[i], eng.kn[i], eps, st.cos,
                             st.sin, self.q, kc, vc, err=err)
            if self.rows_attn:  # root slot patched per round at launch (recorded at 0)
                ops.tree_attn_rows(self.q, T, 0, self.anc, nq, nkv, kc[0], vc[0], self.att, err=err)
            else:
                ops.tree_attn(self.q, B, T, nq, nkv, kc, vc, self.prefix, self.anc, self.att, err=err)
            self.o(self.xp_a.pack(self.att, None, eps, pdl), eng.w_o[i], self.x, res=self.x, err=err, pdl=pdl)
            self.xp_h.pack(self.x, eng.ln2[i], eps, pdl)
            self.gu(self.xp_h, eng.w_gu[i], self.xp_i, err=err, pdl=pdl)
            self.down(self.xp_i, eng.w_down[i], self.x, res=self.x, err=err, pdl=pdl)
        self.lm(self.xp_h.pack(self.x, eng.final_norm, eps, pdl), eng.e_packed, self.out, err=err, pdl=pdl)

    def prime(self, root_slot: int) -> None:
        """Fill the device inputs with root-only trees at `root_slot` (every row attends to the prefix
        and itself), for warm-up launches."""
        B, T, M = self.B, self.T, self.M
        ints = [root_slot + (i % T > 0) for i in range(M)] + [1 << (i % T) if i % T < 31 else -(1 << 31)
                                                                for i in range(M)] + [root_slot] * B
        self.tok.zero_()
        self.ints.copy_(torch.tensor(ints, dtype=torch.int32))
        self.root1 = root_slot

    def launch(self, eng: "Engine", st: "_State") -> None:
        """Run the verify forward on the current stream over the device buffers' current contents (and, for
        the tensor-core tree attention of one sequence, the host's root slot self.root1)."""
        if self.calls is None:
            with qdlib.recording() as rec:
                self._enqueue(eng, st)
            self.calls = qdlib.bind(rec)
            self.rows_calls = [c[2] for c in self.calls if c[1] == "qd_tree_attn_rows"]
        stream = torch.cuda.current_stream().cuda_stream
        for args in self.rows_calls:
            args[2] = self.root1 + self.T  # keys end
            args[3] = self.root1           # first tree row's position
        for _, _, args in self.calls:
            args[-1] = stream
        qdlib.replay(self.calls)

    def __call__(self, eng: "Engine", st: "_State", trees: list, pos0s: list[int]):
        """Greedy token at every node of each sequence's tree (its root at position pos0s[b]; a None tree
        runs inert rows), and the commit callback that, given the accepted path of each sequence (None
        for none), moves the paths' keys / values into place."""
        B, T = self.B, self.T
        tok, pos, anc = [], [], []
        for b in range(B):
            if pos0s[b] < 0 or pos0s[b] + T > st.capacity:
                raise RuntimeError("token tree past the cache capacity")
            tree = trees[b]
            if tree is None:
                tree = tree_spec.TokenTree(0, T)
            t, d, m = tree.padded(T)
            tok += t
            pos += [pos0s[b] + x for x in d]
            anc += [x - (1 << 32) if x >= 1 << 31 else x for x in m]  # 32-bit masks as int32 (two's complement)
        self.root1 = pos0s[0]
        with torch.inference_mode():
            self.tok_host.copy_(torch.tensor(tok, dtype=torch.int64))
            self.ints_host.copy_(torch.tensor(pos + anc + list(pos0s), dtype=torch.int32))
            self.tok.copy_(self.tok_host, non_blocking=True)
            self.ints.copy_(self.ints_host, non_blocking=True)
            self.launch(eng, st)
            self.out_host.copy_(self.out, non_blocking=True)
            self.event.record()
        self.event.synchronize()
        g = self.out_host.tolist()
        greedy = [g[b * T:(b + 1) * T] for b in range(B)]

        def commit(paths, p0s):
            moves = [(b, src, dst) for b, path in enumerate(paths) if path
                     for src, dst in tree_spec.compaction_moves(path, p0s[b])]
            if moves:
                with torch.inference_mode():
                    self.moves_host[:len(moves)].copy_(torch.tensor(moves, dtype=torch.int32))
                    self.moves.copy_(self.moves_host, non_blocking=True)
                    ops.tree_compact(st.k_all, st.v_all, self.moves, len(moves))
        return greedy, commit


class Engine:
    def __init__(self, model_path: str, device: str | None = None) -> None:
        t0 = time.perf_counter()
        state, cfg = load_checkpoint(model_path, "cpu")
        self._setup(state, cfg, device or DEVICE)
        self.load_s = time.perf_counter() - t0
        log(f"loaded {model_path} in {self.load_s:.1f}s: {self.n_layers} layers, {qdlib.load().qd_version().decode()}")

    @classmethod
    def from_state_dict(cls, state: dict, cfg: dict, device: str | None = None) -> "Engine":
        """Build from Hugging Face-named BF16 tensors (CPU or CUDA) and a config dict."""
        eng = cls.__new__(cls)
        t0 = time.perf_counter()
        eng._setup(state, cfg, device or DEVICE)
        eng.load_s = time.perf_counter() - t0
        return eng

    # ------------------------------------------------------------------ weights
    def _setup(self, state: dict, cfg: dict, device: str) -> None:
        qdlib.load()  # fail loudly before anything else if the CUDA library is missing
        if not torch.cuda.is_available():
            raise RuntimeError("the decode engine needs a CUDA device (sm_100a); there is no CPU path")
        torch.backends.cuda.matmul.allow_tf32 = False
        torch.backends.cudnn.allow_tf32 = False
        self.device = torch.device(device)
        torch.cuda.set_device(self.device)
        self.cfg = dict(cfg)
        self.n_layers = cfg["num_hidden_layers"]
        self.hidden = H = cfg["hidden_size"]
        self.inter = I = cfg["intermediate_size"]
        self.nq, self.nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
        self.head_dim = D = cfg.get("head_dim") or H // self.nq
        self.vocab = cfg["vocab_size"]
        self.eps = float(cfg["rms_norm_eps"])
        self.theta = float(cfg.get("rope_theta", 5e6))
        if D != 128 or self.nq != 4 * self.nkv or H % 64 or I % 64 or self.nq * D % 64:
            raise NotImplementedError("kernels are built for head_dim 128, 4 query heads per KV head, "
                                      "hidden/intermediate multiples of 64")
        dev = self.device
        get = lambda name: state[name].to(dev, BF16)  # noqa: E731
        Lyr = self.n_layers
        nq_rows, nkv_rows = self.nq * D, self.nkv * D
        n_qkv = nq_rows + 2 * nkv_rows
        # one packed copy of every matrix serves prefill and decode; row-major checkpoint tensors are
        # staged one at a time and dropped after packing
        if "lm_head.weight" in state and not cfg.get("tie_word_embeddings", True):
            raise NotImplementedError("untied LM head: the embedding gather reads the packed LM matrix")
        self.final_norm = get("model.norm.weight")
        self.ln1 = torch.empty((Lyr, H), dtype=BF16, device=dev)
        self.ln2 = torch.empty((Lyr, H), dtype=BF16, device=dev)
        self.qn = torch.empty((Lyr, D), dtype=BF16, device=dev)
        self.kn = torch.empty((Lyr, D), dtype=BF16, device=dev)
        self.w_qkv = ops.new_packed(n_qkv, H, dev, Lyr)
        self.w_o = ops.new_packed(H, nq_rows, dev, Lyr)
        self.w_gu = ops.new_packed(2 * I, H, dev, Lyr)
        self.w_down = ops.new_packed(H, I, dev, Lyr)
        with torch.no_grad():
            qkv_rm = torch.empty((n_qkv, H), dtype=BF16, device=dev)
            for i in range(Lyr):
                p = f"model.layers.{i}."
                self.ln1[i].copy_(state[p + "input_layernorm.weight"])
                self.ln2[i].copy_(state[p + "post_attention_layernorm.weight"])
                self.qn[i].copy_(state[p + "self_attn.q_norm.weight"])
                self.kn[i].copy_(state[p + "self_attn.k_norm.weight"])
                qkv_rm[:nq_rows].copy_(state[p + "self_attn.q_proj.weight"])
                qkv_rm[nq_rows:nq_rows + nkv_rows].copy_(state[p + "self_attn.k_proj.weight"])
                qkv_rm[nq_rows + nkv_rows:].copy_(state[p + "self_attn.v_proj.weight"])
                ops.pack_rows(qkv_rm, self.w_qkv[i], n_qkv)
                ops.pack_rows(get(p + "self_attn.o_proj.weight"), self.w_o[i], H)
                ops.pack_gate_up(get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight"), self.w_gu[i])
                ops.pack_rows(get(p + "mlp.down_proj.weight"), self.w_down[i], H)
            self.e_packed = ops.pack_matrix(get("model.embed_tokens.weight"))
            del qkv_rm
        torch.cuda.synchronize()
        self.state = None
        self.sm_count = ops.sm_count()
        self.speculate = SPEC_T  # verify width of exact speculative decoding at batch 1 (0 = plain greedy)
        self.tree = TREE_T  # nodes per token tree of exact tree speculation (0 = off; wins over speculate)

    # ------------------------------------------------------------------ model step
    def _prefill(self, st: _State) -> torch.Tensor:
        """Prompt forward in row chunks (engine/engine.py:550-592) on the library's prompt kernels:
        qd_tc_gemm over the packed weights, qd_rmsnorm_rows, qd_prefill_qk_rope (K/V [0, S) into the
        cache) and qd_prefill_attn (causal GQA flash attention on the tensor cores). The first token goes
        into st.tok; returns the last position's logits [B, V]."""
        B, S = st.B, st.S
        H, D, nq, nkv, I, eps = self.hidden, self.head_dim, self.nq, self.nkv, self.inter, self.eps
        n_qkv = (nq + 2 * nkv) * D
        vrows = ops.packed_rows(self.vocab)
        dev, err = self.device, st.err
        RES, SWIGLU = ops.Gemv.RES, ops.Gemv.SWIGLU
        last_layer = self.n_layers - 1
        logits = torch.empty((B, vrows), dtype=BF16, device=dev)
        for r0, r1 in st.chunks:
            b, M = r1 - r0, (r1 - r0) * S
            x = torch.empty((M, H), dtype=BF16, device=dev)
            h = torch.empty((M, H), dtype=BF16, device=dev)
            qkv = torch.empty((M, n_qkv), dtype=BF16, device=dev)
            q = torch.empty((M, nq * D), dtype=BF16, device=dev)
            att = torch.empty((M, nq * D), dtype=BF16, device=dev)
            act = torch.empty((M, I), dtype=BF16, device=dev)
            # one split-K partials scratch for every GEMM of the chunk (they run in stream order)
            shapes = [(M, n_qkv, H), (M, H, nq * D), (M, 2 * I, H), (M, H, I), (b, H, nq * D), (b, 2 * I, H),
                      (b, H, I), (b, vrows, H)]
            nb = max(ops.tc_gemm_plan(*s)[3] for s in shapes)
            sc = torch.empty((max(nb, 16),), dtype=torch.uint8, device=dev)
            ops.embed(st.ids[r0:r1].reshape(M), self.e_packed, self.vocab, x, err, pdl=False)
            xl, hl = x.view(b, S, H)[:, -1], h[:b]  # the last position of every sequence
            for i in range(self.n_layers):
                kc, vc = st.k_all[i, r0:r1], st.v_all[i, r0:r1]
                ops.rmsnorm_rows(x, self.ln1[i], eps, h)
                ops.tc_gemm(h, self.w_qkv[i], n_qkv, qkv, err=err, scratch=sc)
                ops.prefill_qk_rope(qkv, b, S, nq, nkv, self.qn[i], self.kn[i], eps, st.cos, st.sin, q, kc, vc)
                if i == last_layer:  # only the last position continues (engine/engine.py:577-583)
                    ops.prefill_attn(q, b, S, nq, nkv, kc, vc, att[:b], q_begin=S - 1, err=err)
                    ops.tc_gemm(att[:b], self.w_o[i], H, xl, res=xl, epilogue=RES, err=err, scratch=sc)
                    ops.rmsnorm_rows(xl, self.ln2[i], eps, hl)
                    ops.tc_gemm(hl, self.w_gu[i], 2 * I, act[:b], epilogue=SWIGLU, err=err, scratch=sc)
                    ops.tc_gemm(act[:b], self.w_down[i], H, xl, res=xl, epilogue=RES, err=err, scratch=sc)
                    break
                ops.prefill_attn(q, b, S, nq, nkv, kc, vc, att, err=err)
                ops.tc_gemm(att, self.w_o[i], H, x, res=x, epilogue=RES, err=err, scratch=sc)
                ops.rmsnorm_rows(x, self.ln2[i], eps, h)
                ops.tc_gemm(h, self.w_gu[i], 2 * I, act, epilogue=SWIGLU, err=err, scratch=sc)
                ops.tc_gemm(act, self.w_down[i], H, x, res=x, epilogue=RES, err=err, scratch=sc)
            ops.rmsnorm_rows(xl, self.final_norm, eps, hl)
            ops.tc_gemm(hl, self.e_packed, vrows, logits[r0:r1], err=err, scratch=sc)
        ops.argmax_rows(logits, self.vocab, st.tok)  # the first generated token of every sequence
        return logits[:, :self.vocab]

    def _decode_step(self, st: _State, logits: torch.Tensor | None = None) -> None:
        """One token per sequence at st.pos, all in libqd_decode: one persistent launch, or
        1 + 5 * layers + 1 per-op launches."""
        if st.mode == "persistent":
            if logits is None:
                st.step()
            else:
                if st.step_logits is None or st.step_logits._keep[2] is not logits:
                    st.step_logits = ops.DecodeStep(self, st, logits)
                st.step_logits()
            return
        if st.tstep is not None:
            if logits is None:
                st.tstep()
            else:
                if st.tstep_logits is None or st.tstep_logits._keep[2] is not logits:
                    st.tstep_logits = ops.TcDecodeStep(self, st, logits)
                st.tstep_logits()
            return
        pdl, err = USE_PDL, st.err
        ops.embed(st.tok, self.e_packed, self.vocab, st.x, err, pdl)
        if st.mode == "tc":
            self._decode_layers_tc(st, logits, pdl, err)
            return
        for i in range(self.n_layers):
            kc, vc = st.k_all[i], st.v_all[i]
            st.qkv(st.x, self.w_qkv[i], self.ln1[i], self.qn[i], self.kn[i], st.cos, st.sin, st.pos, st.q, kc, vc,
                   err=err, pdl=pdl)
            st.attn(st.q, kc, vc, st.pos, st.attn_out, err=err, pdl=pdl)
            st.o(st.attn_out.view(st.B, -1), self.w_o[i], st.x, res=st.x, err=err, pdl=pdl)
            st.gu(st.x, self.w_gu[i], st.act, norm_w=self.ln2[i], err=err, pdl=pdl)
            st.down(st.act, self.w_down[i], st.x, res=st.x, err=err, pdl=pdl)
        st.lm(st.x, self.e_packed, self.final_norm, st.tok, st.pos, inc_pos=True, logits=logits, err=err, pdl=pdl)

    def _decode_layers_tc(self, st: _State, logits, pdl, err) -> None:
        """Layers and LM head on the tensor-core kernels: each projection reads its activations packed
        into the MMA operand layout - RMSNorm-ed by a packing kernel before QKV, gate/up and the LM head,
        written packed directly by the attention and SwiGLU epilogues before O and down."""
        B, eps, sums = st.B, self.eps, st.res_sums
        # O and down leave their outputs as fixed-point sums; the packing for the next projection adds them
        # to the residual stream x (and clears them), so no split-K last arriver sits between the two
        for i in range(self.n_layers):
            kc, vc = st.k_all[i], st.v_all[i]
            if i == 0:
                st.xp_h.pack(st.x, self.ln1[i], eps, pdl)
            else:
                st.xp_h.pack_res(st.x, sums, self.ln1[i], eps, pdl)
            st.qkv_mm(st.xp_h, self.w_qkv[i], st.qkv_sums, err=err, pdl=pdl)
            ops.qkv_rope_sums(st.qkv_sums, B, self.nq, self.nkv, self.qn[i], self.kn[i], eps, st.cos, st.sin, st.pos,
                              st.q, kc, vc, err=err, pdl=pdl)
            st.attn(st.q, kc, vc, st.pos, st.xp_a, err=err, pdl=pdl)       # written packed for O
            st.o(st.xp_a, self.w_o[i], sums, err=err, pdl=pdl)
            st.xp_h.pack_res(st.x, sums, self.ln2[i], eps, pdl)
            st.gu(st.xp_h, self.w_gu[i], st.xp_i, err=err, pdl=pdl)        # SwiGLU written packed for down
            st.down(st.xp_i, self.w_down[i], sums, err=err, pdl=pdl)
        st.xp_h.pack_res(st.x, sums, self.final_norm, eps, pdl)
        st.lm(st.xp_h, self.e_packed, st.tok, st.pos, inc_pos=True, logits=logits, err=err, pdl=pdl)

    def check_device_errors(self, st: _State) -> None:
        code = int(st.err.item())
        if code:
            # counters and tickets may be left mid-step: clear every scratch buffer before raising
            extra = [v for side in (st.verify, st.tree) if side is not None
                     for v in (side.qkv_op, side.o, side.gu, side.down, side.lm)]
            for plan in (st.qkv, getattr(st, "qkv_mm", None), st.attn, st.o, st.gu, st.down, st.lm, st.step,
                         st.step_logits, st.tstep,
                         st.tstep_logits, *extra):
                if plan is not None:
                    plan.scratch.zero_()
            for sums in (getattr(st, "res_sums", None), getattr(st, "qkv_sums", None)):
                if sums is not None:  # deferred fixed-point sums may be half added
                    sums.zero_()
            st.err.zero_()
            raise RuntimeError(f"decode kernels reported a device error: {qdlib.describe_device_error(code)}")

    # ------------------------------------------------------------------ shapes, graphs
    def _side_widths(self, B: int, N: int) -> tuple[int, int]:
        """(token-tree nodes per sequence, prompt-lookup verify width) for a request of B sequences and N
        new tokens; 0 = off. Trees are cut to TREE_MAX_ROWS // B nodes and need at least 2; prompt-lookup
        speculation runs at batch 1 only and yields to trees."""
        tree_T = min(self.tree, TREE_MAX_ROWS // B) if (self.tree and N > 1) else 0
        tree_T = tree_T if tree_T >= 2 else 0
        spec_T = self.speculate if (self.speculate and B == 1 and N > 1 and not tree_T) else 0
        return tree_T, spec_T

    def _build(self, B: int, S: int, N: int) -> _State:
        if B > TC_MAX_BATCH:
            raise NotImplementedError(f"batch {B} > {TC_MAX_BATCH} per GPU: shard the batch across GPUs")
        self.state = None
        gc.collect()
        torch.cuda.empty_cache()
        tree_T, spec_T = self._side_widths(B, N)
        st = _State(self, B, S, N, spec_T, tree_T)
        t0 = time.perf_counter()
        with torch.inference_mode():
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(2):
                    self._prefill(st)
                    if N > 1:
                        st.pos.fill_(S)
                        self._decode_step(st)
                    if st.verify is not None:
                        st.verify.launch(self, st, S - 1)
                    if st.tree is not None:
                        st.tree.prime(S - 1)
                        st.tree.launch(self, st)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            self.check_device_errors(st)
            if USE_GRAPHS:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    st.prefill_logits = self._prefill(st)
                st.prefill_graph = g
                if N > 1:
                    st.pos.fill_(S)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        self._decode_step(st)
                    st.decode_graph = g
            torch.cuda.synchronize()
        st.build_s = time.perf_counter() - t0
        self.state = st
        return st

    def _upload_prompt(self, st: _State, input_ids) -> None:
        """Prompt ids into the device buffer the prefill graph reads (through pinned staging), and the
        decode position reset to the prompt length: everything a replay of a new request needs."""
        st.prompt_host.copy_(torch.as_tensor(input_ids, dtype=torch.int64))
        st.ids.copy_(st.prompt_host, non_blocking=True)
        st.pos.fill_(st.S)

    def _enqueue_prefill(self, st: _State) -> None:
        if st.prefill_graph is None:
            st.prefill_logits = self._prefill(st)
        else:
            st.prefill_graph.replay()

    def _enqueue_decode(self, st: _State) -> None:
        if st.decode_graph is None:
            self._decode_step(st)
        else:
            st.decode_graph.replay()

    def _stream(self, st: _State, input_ids, N: int, timing: list | None = None):
        """Greedy token lists of N steps. The prefill and then the decode steps are enqueued while the
        caller consumes earlier steps; at most AHEAD steps sit queued beyond the one being delivered.
        With `timing` (a list), the device milliseconds of every step are appended to it at the end."""
        ring, timer = st.ring, (_StepTimer() if timing is not None else None)
        run = (lambda fn: fn(st)) if timer is None else (lambda fn: _timed(timer, fn, st))
        ring.reset()
        with torch.inference_mode():
            self._upload_prompt(st, input_ids)
            run(self._enqueue_prefill)
            ring.post(st.tok)
        enqueued = 1
        for delivered in range(N):
            while enqueued < N and ring.in_flight() <= AHEAD:
                with torch.inference_mode():
                    run(self._enqueue_decode)
                    ring.post(st.tok)
                enqueued += 1
            row = ring.take()
            if delivered == N - 1:  # everything has run: surface a device-side error before the last list
                self.check_device_errors(st)
                if timer is not None:
                    timing.extend(timer.ms())
            yield row

    def _stream_spec(self, st: _State, input_ids, N: int):
        """Exact prompt-lookup speculative decoding of one sequence (the reference's _stream_spec,
        engine/engine.py:759-828): after the prompt forward, every verify runs T = k + 1 tokens (the last
        emitted token and a k-token draft from the sequence's own history) and emits the accepted drafts
        plus the greedy token after them; exactly N steps are yielded. The emitted tokens are the verify
        forward's greedy tokens whatever the draft was."""
        S, vf = st.S, st.verify
        ring = st.ring
        ring.reset()
        with torch.inference_mode():
            self._upload_prompt(st, input_ids)
            self._enqueue_prefill(st)
            ring.post(st.tok)
        first = ring.take()
        yield first
        st.spec_stats = {}
        plain = (lambda tok, pos, n: self._plain_steps(st, tok, pos, n)) if SPEC_GATE else None
        for tok in spec.stream(list(input_ids[0]) + first, S, N, vf.T - 1, lambda row, pos0: vf(self, st, row, pos0),
                               st.spec_stats, step=plain, gate=spec.Gate() if SPEC_GATE else None):
            yield [tok]
        self.check_device_errors(st)

    def _stream_tree(self, st: _State, input_ids, N: int):
        """Exact token-tree speculative decoding (the reference's tree stream, engine/engine.py:830-936):
        after the prompt forward, every round verifies one drafted tree of st.tree.T nodes per sequence
        in one forward and emits the model's greedy tokens along each accepted path plus the one after
        it; exactly N steps are yielded. At batch 1 runs of plain decode steps stand in while trees do not
        pay (spec.Gate); at batch > 1 the sequences' positions drift apart, and the decode step takes one
        position, so every round is a tree verify."""
        S, tv, ring = st.S, st.tree, st.ring
        ring.reset()
        with torch.inference_mode():
            self._upload_prompt(st, input_ids)
            self._enqueue_prefill(st)
            ring.post(st.tok)
        first = ring.take()
        yield first
        st.spec_stats = {}
        seqs = [list(row) + [t] for row, t in zip(input_ids, first)]
        if st.B > 1:
            yield from tree_spec.stream_batch(seqs, S, N, tv.T, tv.depth,
                                              lambda trees, pos0s: tv(self, st, trees, pos0s), st.spec_stats)
            self.check_device_errors(st)
            return

        def verify(tree, pos0):
            greedy, commit = tv(self, st, [tree], [pos0])
            return greedy[0], lambda path, p0: commit([path], [p0])

        plain = (lambda tok, pos, n: self._plain_steps(st, tok, pos, n)) if SPEC_GATE else None
        for tok in tree_spec.stream(seqs[0], S, N, tv.T, tv.depth, verify, st.spec_stats, step=plain,
                                    gate=spec.Gate() if SPEC_GATE else None):
            yield [tok]
        self.check_device_errors(st)

    def _plain_steps(self, st: _State, tok: int, pos: int, n: int):
        """n plain decode steps of a batch-1 state continuing from the host's token at position `pos` (the
        speculative loop's fallback), yielding the n greedy tokens one at a time. The first replay takes
        its token and position from the host; each later one from the replay before it, so the device
        runs ahead of the caller through the token ring as in `_stream`."""
        ring = st.ring
        ring.reset()
        with torch.inference_mode():
            st.step_host[0], st.step_host[1] = tok, pos
            st.tok.copy_(st.step_host[0:1], non_blocking=True)
            st.pos.copy_(st.step_host[1:2], non_blocking=True)
        enqueued = 0
        for _ in range(n):
            while enqueued < n and ring.in_flight() <= AHEAD:
                with torch.inference_mode():
                    self._enqueue_decode(st)
                    ring.post(st.tok)
                enqueued += 1
            yield ring.take()[0]

    # ------------------------------------------------------------------ API
    def generate(self, input_ids: list[list[int]], max_new_tokens: int):
        N = int(max_new_tokens)
        if N <= 0:
            return
        B, S = len(input_ids), len(input_ids[0])
        if B < 1 or S < 1 or any(len(r) != S for r in input_ids):
            raise ValueError("input_ids must be a non-empty batch of equal-length rows")
        tree_T, spec_T = self._side_widths(B, N)
        st = self.state
        fits = st is not None and (st.B, st.S, st.N) == (B, S, N) and (st.verify.T if st.verify else 0) == spec_T \
            and (st.tree.T if st.tree else 0) == tree_T
        if not fits:
            st = self._build(B, S, N)
        stream = self._stream_tree if st.tree is not None else (self._stream_spec if st.verify is not None else
                                                                 self._stream)
        with _collector_paused():
            yield from stream(st, input_ids, N)

    def generate_with_logits(self, input_ids: list[list[int]], max_new_tokens: int,
                             forced: list[list[int]] | None = None):
        """Test hook: eager (un-graphed) greedy run returning (tokens [B][N], list of N host logits [B, V]).
        With `forced` (tokens [B][N]), step t decodes from forced[:, t - 1] instead of the engine's own
        token: teacher forcing, so step t's logits are the engine's logits after the forced prefix (the
        reference checks its tiers this way, engine/engine.py:974-996). The returned tokens are still
        the engine's own argmax at every step."""
        N = int(max_new_tokens)
        B, S = len(input_ids), len(input_ids[0])
        st = self.state
        if st is None or (st.B, st.S, st.N) != (B, S, N):
            st = self._build(B, S, N)
        if st.logits is None:
            st.logits = torch.empty((B, self.vocab), dtype=BF16, device=self.device)
        buf = st.logits
        toks, logits = [], []
        with torch.inference_mode():
            st.ids.copy_(torch.tensor(input_ids, dtype=torch.int64))
            st.pos.fill_(S)
            lg = self._prefill(st)
            toks.append(st.tok.tolist())
            logits.append(lg.cpu())
            for t in range(1, N):
                if forced is not None:
                    st.tok.copy_(torch.tensor([row[t - 1] for row in forced], dtype=torch.int64))
                self._decode_step(st, logits=buf)
                toks.append(st.tok.tolist())
                logits.append(buf.cpu())
        self.check_device_errors(st)
        return [list(r) for r in zip(*toks)], logits
