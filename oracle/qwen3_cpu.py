"""Torch-CPU restatement of the reference's eager Qwen3 decode path (TEST INFRASTRUCTURE ONLY).

Follows the reference engine's tier-1 arithmetic operation by operation (engine/engine.py):

  _norm            :501-509  Qwen3RMSNorm: fp32 mean of squares, x*rsqrt(var+eps) in fp32,
                             cast to BF16, *then* multiply by the BF16 weight
  _act             :511-514  silu(gate) * up on BF16 tensors
  _prefill         :550-592  prompt forward (causal SDPA, repeat_kv), K/V into the static cache
  _decode          :594-643  one token per sequence: norm -> packed QKV linear -> q/k norm ->
                             RoPE with BF16 products (:622-623) -> cache write at pos ->
                             SDPA over cache[:pos+1] -> O + residual -> norm -> gate_up ->
                             SwiGLU -> down + residual; final norm -> tied LM head -> argmax
  rotary tables    :182-185  cos/sin [cap, 128] BF16 from the model's rotary module; restated
                             here as transformers' Qwen3RotaryEmbedding.forward computes them

Per-op functions double as the checkers for the CUDA kernels (tests/test_*_gpu.py). Everything runs
on CPU in BF16 with torch's own kernels, exactly as the reference's tier 1 does when
ENGINE_DEVICE=cpu; tests/test_oracle.py pins the whole path against tests/golden/*.json (tokens
and logits of the reference engine's tiers 0 and 1).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

BF16 = torch.bfloat16
N_HEADS, N_KV, HEAD_DIM = 32, 8, 128


# ------------------------------------------------------------------------------------ ops
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, heads: int = 1) -> torch.Tensor:
    """Qwen3RMSNorm over rows of width w.numel() (engine/engine.py:505-509).
    x [M, >= heads*n] BF16 -> [M, heads, n] BF16."""
    n = w.numel()
    xf = x[:, : heads * n].reshape(x.shape[0], heads, n).to(torch.float32)
    var = xf.pow(2).mean(-1, keepdim=True)
    xf = xf * torch.rsqrt(var + eps)
    return w * xf.to(BF16)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """engine/engine.py:104-106 (transformers rotate_half)."""
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def rope_tables(cap: int, head_dim: int = HEAD_DIM, theta: float = 5e6) -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin [cap, head_dim] BF16 for positions 0..cap-1, computed as transformers'
    Qwen3RotaryEmbedding (default rope type, attention_scaling 1) does on CPU:
    inv_freq = 1/theta^(arange(0,d,2)/d) in fp32, freqs = inv_freq @ pos (fp32 matmul),
    emb = cat(freqs, freqs), cos/sin in fp32, cast to BF16 (engine/engine.py:182-185)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim))
    pos = torch.arange(cap)[None]
    inv_freq_expanded = inv_freq[None, :, None].float().expand(pos.shape[0], -1, 1)
    position_ids_expanded = pos[:, None, :].float()
    freqs = (inv_freq_expanded.float() @ position_ids_expanded.float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos()[0].to(BF16).contiguous(), emb.sin()[0].to(BF16).contiguous()


def repeat_kv(x: torch.Tensor, groups: int = N_HEADS // N_KV) -> torch.Tensor:
    """engine/engine.py:109-111."""
    b, h, s, d = x.shape
    return x[:, :, None].expand(b, h, groups, s, d).reshape(b, h * groups, s, d)


def qk_norm_rope(qkv: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor, cos_row: torch.Tensor,
                 sin_row: torch.Tensor, eps: float, n_heads: int = N_HEADS, n_kv: int = N_KV):
    """Per-head q/k RMSNorm then RoPE at one position (engine/engine.py:619-623).
    qkv [B, (nq+2nkv)*128] BF16; cos_row/sin_row [128] BF16. Returns q [B,nq,128], k, v [B,nkv,128]."""
    D = q_norm.numel()
    B = qkv.shape[0]
    q = rms_norm(qkv, q_norm, eps, n_heads)
    k = rms_norm(qkv[:, n_heads * D:], k_norm, eps, n_kv)
    v = qkv[:, (n_heads + n_kv) * D:].reshape(B, n_kv, D)
    c, s = cos_row[None, None], sin_row[None, None]
    q = (q * c) + (rotate_half(q) * s)
    k = (k * c) + (rotate_half(k) * s)
    return q, k, v


def attention_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, n: int) -> torch.Tensor:
    """SDPA of one query per sequence over cache[:, :, :n] with repeat_kv (engine/engine.py:633-636).
    q [B, 32, 128]; caches [B, 8, cap, 128]. Returns [B, 32, 128] BF16."""
    B, H, D = q.shape
    a = F.scaled_dot_product_attention(q.view(B, H, 1, D).contiguous(), repeat_kv(k_cache[:, :, :n]),
                                       repeat_kv(v_cache[:, :, :n]), scale=D ** -0.5)
    return a.view(B, H, D)


def swiglu(gu: torch.Tensor, inter: int) -> torch.Tensor:
    """silu(gate) * up on a packed [M, 2*inter] gate|up row (engine/engine.py:511-514)."""
    return F.silu(gu[:, :inter]) * gu[:, inter:]


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    return F.linear(x, w)


def lm_logits(x: torch.Tensor, final_norm: torch.Tensor, lm_head: torch.Tensor, eps: float) -> torch.Tensor:
    """Final RMSNorm + tied LM head: BF16 logits [M, V] (engine/engine.py:640)."""
    return F.linear(rms_norm(x, final_norm, eps).view(x.shape[0], -1), lm_head)


def argmax_lowest(logits: torch.Tensor) -> torch.Tensor:
    """Greedy token with the lowest index on exact ties (torch.argmax's rule on CPU and CUDA)."""
    lf = logits.float()
    best = lf.max(dim=-1, keepdim=True).values
    idx = torch.arange(lf.shape[-1]).expand_as(lf)
    return torch.where(lf == best, idx, lf.shape[-1]).min(dim=-1).values


# ------------------------------------------------------------------------------------ model
class Qwen3Oracle:
    """Whole-model CPU restatement (engine/engine.py tier 1) over a Hugging Face state dict."""

    def __init__(self, state: dict, cfg: dict):
        self.cfg = cfg
        self.eps = float(cfg["rms_norm_eps"])
        self.theta = float(cfg.get("rope_theta", 5e6))
        self.inter = int(cfg["intermediate_size"])
        self.nq, self.nkv, self.D = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
        self.embed = state["model.embed_tokens.weight"]
        self.lm_head = state.get("lm_head.weight", self.embed)
        self.final_norm = state["model.norm.weight"]
        self.layers = []
        for i in range(cfg["num_hidden_layers"]):
            p = f"model.layers.{i}."
            self.layers.append({
                "ln1": state[p + "input_layernorm.weight"],
                "ln2": state[p + "post_attention_layernorm.weight"],
                "q_norm": state[p + "self_attn.q_norm.weight"],
                "k_norm": state[p + "self_attn.k_norm.weight"],
                # packed like the reference (engine/engine.py:267-273)
                "w_qkv": torch.cat([state[p + "self_attn.q_proj.weight"], state[p + "self_attn.k_proj.weight"],
                                    state[p + "self_attn.v_proj.weight"]], 0),
                "w_o": state[p + "self_attn.o_proj.weight"],
                "w_gu": torch.cat([state[p + "mlp.gate_proj.weight"], state[p + "mlp.up_proj.weight"]], 0),
                "w_down": state[p + "mlp.down_proj.weight"],
            })

    # -- state
    def reset(self, B: int, cap: int):
        L = len(self.layers)
        self.k = torch.zeros((L, B, self.nkv, cap, self.D), dtype=BF16)
        self.v = torch.zeros((L, B, self.nkv, cap, self.D), dtype=BF16)
        self.cos, self.sin = rope_tables(cap, self.D, self.theta)

    def prefill(self, ids: torch.Tensor) -> torch.Tensor:
        """Prompt forward (engine/engine.py:550-592); fills K/V [0,S); returns logits [B, V]."""
        B, S = ids.shape
        M = B * S
        cos = self.cos[:S][None, None]
        sin = self.sin[:S][None, None]
        D, nq, nkv = self.D, self.nq, self.nkv
        x = F.embedding(ids, self.embed).view(M, -1)
        last = len(self.layers) - 1
        for i, L in enumerate(self.layers):
            h = rms_norm(x, L["ln1"], self.eps).view(M, -1)
            qkv = F.linear(h, L["w_qkv"])
            q = rms_norm(qkv, L["q_norm"], self.eps, nq).view(B, S, nq, D).transpose(1, 2)
            k = rms_norm(qkv[:, nq * D:], L["k_norm"], self.eps, nkv).view(B, S, nkv, D).transpose(1, 2)
            v = qkv[:, (nq + nkv) * D:].view(B, S, nkv, D).transpose(1, 2)
            q = (q * cos) + (rotate_half(q) * sin)
            k = (k * cos) + (rotate_half(k) * sin)
            self.k[i, :, :, :S].copy_(k)
            self.v[i, :, :, :S].copy_(v)
            kc, vc = self.k[i, :, :, :S], self.v[i, :, :, :S]
            if i == last:
                a = F.scaled_dot_product_attention(q[:, :, -1:].contiguous(), repeat_kv(kc), repeat_kv(vc),
                                                   scale=D ** -0.5)
                x = x.view(B, S, -1)[:, -1] + F.linear(a.reshape(B, nq * D), L["w_o"])
                h = rms_norm(x, L["ln2"], self.eps).view(B, -1)
                x = x + F.linear(swiglu(F.linear(h, L["w_gu"]), self.inter), L["w_down"])
                break
            a = F.scaled_dot_product_attention(q.contiguous(), repeat_kv(kc), repeat_kv(vc), is_causal=True,
                                               scale=D ** -0.5)
            x = x + F.linear(a.transpose(1, 2).reshape(M, nq * D), L["w_o"])
            h = rms_norm(x, L["ln2"], self.eps).view(M, -1)
            x = x + F.linear(swiglu(F.linear(h, L["w_gu"]), self.inter), L["w_down"])
        return lm_logits(x, self.final_norm, self.lm_head, self.eps)

    def decode(self, tok: torch.Tensor, pos: int) -> torch.Tensor:
        """One token per sequence at position pos (engine/engine.py:594-643, host_pos path)."""
        B = tok.shape[0]
        D, nq, nkv = self.D, self.nq, self.nkv
        x = F.embedding(tok, self.embed)
        for i, L in enumerate(self.layers):
            h = rms_norm(x, L["ln1"], self.eps).view(B, -1)
            qkv = F.linear(h, L["w_qkv"])
            q, k, v = qk_norm_rope(qkv, L["q_norm"], L["k_norm"], self.cos[pos], self.sin[pos], self.eps, nq, nkv)
            self.k[i, :, :, pos].copy_(k)
            self.v[i, :, :, pos].copy_(v)
            a = attention_decode(q, self.k[i], self.v[i], pos + 1).reshape(B, nq * D)
            x = x + F.linear(a, L["w_o"])
            h = rms_norm(x, L["ln2"], self.eps).view(B, -1)
            x = x + F.linear(swiglu(F.linear(h, L["w_gu"]), self.inter), L["w_down"])
        return lm_logits(x, self.final_norm, self.lm_head, self.eps)

    @torch.inference_mode()
    def generate(self, input_ids, N: int, forced: list[list[int]] | None = None):
        """Greedy decode of N tokens; returns (tokens [B][N], logits list of N [B, V] BF16).
        With `forced` (tokens [B][N]) the model is teacher-forced on those tokens instead of its own
        argmax, so step t's logits are the oracle's logits given the forced prefix."""
        ids = torch.tensor(input_ids, dtype=torch.int64)
        B, S = ids.shape
        self.reset(B, S + N)
        logits = self.prefill(ids)
        out_logits = [logits]
        toks = [argmax_lowest(logits)]
        for t in range(1, N):
            prev = torch.tensor([r[t - 1] for r in forced]) if forced is not None else toks[-1]
            logits = self.decode(prev, S + t - 1)
            out_logits.append(logits)
            toks.append(argmax_lowest(logits))
        return [list(r) for r in zip(*[t.tolist() for t in toks])], out_logits


def log_softmax_maxdiff(a: torch.Tensor, b: torch.Tensor) -> float:
    """max |log_softmax(a) - log_softmax(b)| over all entries (the parity metric for logits)."""
    return (torch.log_softmax(a.float(), -1) - torch.log_softmax(b.float(), -1)).abs().max().item()


def softmax_maxdiff(a: torch.Tensor, b: torch.Tensor) -> float:
    """max |softmax(a) - softmax(b)| (the north star's "after softmax-normalising" metric)."""
    return (torch.softmax(a.float(), -1) - torch.softmax(b.float(), -1)).abs().max().item()


def token_ok(tok: int, ref_logits: torch.Tensor, tol: float) -> bool:
    """Tie rule: tok must be a reference argmax, or, where the reference's own top-2 gap is below
    tol, any token within tol of the reference maximum."""
    lf = ref_logits.float()
    best = lf.max()
    if lf[tok] == best:
        return True
    top2 = lf.topk(2).values
    return bool((top2[0] - top2[1]) < tol and lf[tok] >= best - tol)
