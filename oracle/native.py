"""The reference's tier 0 on CPU: the plain Transformers greedy loop (TEST INFRASTRUCTURE ONLY).

Restates engine/engine.py:963-972 (`_native`): Qwen3ForCausalLM in BF16 with
attn_implementation="sdpa", a KV cache carried between calls, `logits_to_keep=1`, argmax of the
last position; and engine/engine.py:974-996 (`_teacher_force`): the margin
`max logit - logit[token]` when the emitted tokens are replayed through one full forward.

The arithmetic lives in the third-party `transformers` package (the reference pins 4.51.3,
requirements.txt:10; this image has 5.5.0, modeling_qwen3.py). It is used here, on CPU, as the
reference's CPU implementation of the decode path: bench.py's `--impl reference` arm and
`cpu_baseline` time it on the GPU box's host cores.
"""

from __future__ import annotations

import time

import torch

BF16 = torch.bfloat16


def build_model(state: dict, cfg: dict, threads: int | None = None):
    """Qwen3ForCausalLM on CPU holding `state` (HF-named BF16 tensors), as from_pretrained would."""
    from transformers import Qwen3Config, Qwen3ForCausalLM

    if threads:
        torch.set_num_threads(threads)
    conf = Qwen3Config(
        vocab_size=cfg["vocab_size"], hidden_size=cfg["hidden_size"], intermediate_size=cfg["intermediate_size"],
        num_hidden_layers=cfg["num_hidden_layers"], num_attention_heads=cfg["num_attention_heads"],
        num_key_value_heads=cfg["num_key_value_heads"], head_dim=cfg["head_dim"],
        rms_norm_eps=cfg["rms_norm_eps"], rope_theta=cfg["rope_theta"],
        tie_word_embeddings=cfg.get("tie_word_embeddings", True),
        max_position_embeddings=cfg.get("max_position_embeddings", 262144),
    )
    conf._attn_implementation = "sdpa"
    with torch.device("meta"):
        model = Qwen3ForCausalLM(conf)
    model = model.to_empty(device="cpu").to(BF16)
    sd = dict(state)
    if conf.tie_word_embeddings:
        sd.pop("lm_head.weight", None)
    missing, unexpected = model.load_state_dict(sd, strict=False, assign=True)
    missing = [m for m in missing if m != "lm_head.weight"]
    if missing or unexpected:
        raise RuntimeError(f"state dict mismatch: missing={missing} unexpected={unexpected}")
    if conf.tie_word_embeddings:
        model.tie_weights()
    # rotary buffers were created on meta; recompute them on CPU
    rot = model.model.rotary_emb
    inv, scale = rot.compute_default_rope_parameters(conf, "cpu")
    rot.inv_freq = inv
    rot.original_inv_freq = inv.clone()
    rot.attention_scaling = scale
    return model.eval()


@torch.inference_mode()
def greedy(model, input_ids, N: int, keep_logits: bool = True):
    """engine/engine.py:963-972: returns (tokens [B][N], list of N logits [B, V] or None, per-step seconds)."""
    current = torch.tensor(input_ids, dtype=torch.int64)
    cache = None
    toks, logits_out, times = [], [], []
    for _ in range(N):
        t0 = time.perf_counter()
        out = model(input_ids=current, past_key_values=cache, use_cache=True, logits_to_keep=1, return_dict=True)
        current = out.logits[:, -1, :].argmax(dim=-1, keepdim=True)
        cache = out.past_key_values
        times.append(time.perf_counter() - t0)
        toks.append(current[:, 0].tolist())
        if keep_logits:
            logits_out.append(out.logits[:, -1, :].clone())
    return [list(r) for r in zip(*toks)], (logits_out if keep_logits else None), times


@torch.inference_mode()
def teacher_forced_logits(model, input_ids, toks):
    """Logits at every emitted position when prompt + toks[:-1] is replayed in one forward
    (engine/engine.py:983-985). Returns [B, K, V] float."""
    K = len(toks[0])
    seqs = [list(p) + list(t[:-1]) for p, t in zip(input_ids, toks)]
    ids = torch.tensor(seqs, dtype=torch.int64)
    return model(input_ids=ids, logits_to_keep=K, use_cache=False).logits.float()


def teacher_forced_margin(model, input_ids, toks) -> float:
    """engine/engine.py:974-996: max over positions of (max logit - logit[emitted token])."""
    logits = teacher_forced_logits(model, input_ids, toks)
    tgt = torch.tensor(toks, dtype=torch.int64)
    margin = logits.max(-1).values - logits.gather(-1, tgt[..., None])[..., 0]
    if not torch.isfinite(margin).all():
        return float("inf")
    return float(margin.max().item())
