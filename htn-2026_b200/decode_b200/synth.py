"""Seeded random-init Qwen3 checkpoints in the Hugging Face layout.

The reference engine loads a Hugging Face directory (config.json + safetensors) with
`AutoModelForCausalLM.from_pretrained` (engine/engine.py:237-241). The pinned checkpoint is not
available offline, so every test and benchmark here uses a synthetic one with the Qwen3-4B
architecture: all projection and embedding matrices N(0, 0.02), all RMSNorm weights 1, BF16.

Generation is deterministic and independent of the thread count: every tensor is cut into chunks
of CHUNK elements and chunk j of tensor i is drawn from its own torch CPU generator seeded with
(seed, i, j). Chunks run on a thread pool (torch releases the GIL), so the 4-layer checkpoint takes
a few seconds and the 36-layer one about ten on an 8-core host.
"""

from __future__ import annotations

import json
import os
from concurrent.futures import ThreadPoolExecutor

import torch

CHUNK = 1 << 22

# Qwen/Qwen3-4B-Instruct-2507 architecture (the reference's OPTIMIZATION_GUIDE.md architecture table).
QWEN3_4B = {
    "hidden_size": 2560,
    "intermediate_size": 9728,
    "num_hidden_layers": 36,
    "num_attention_heads": 32,
    "num_key_value_heads": 8,
    "head_dim": 128,
    "vocab_size": 151936,
    "rms_norm_eps": 1e-6,
    "rope_theta": 5000000.0,
    "tie_word_embeddings": True,
    "max_position_embeddings": 262144,
}


def qwen3_config(n_layers: int = 36, **overrides) -> dict:
    cfg = dict(QWEN3_4B)
    cfg["num_hidden_layers"] = int(n_layers)
    cfg.update(overrides)
    return cfg


def hf_config_json(cfg: dict) -> dict:
    """config.json contents that both transformers 4.51 and 5.x read as a Qwen3ForCausalLM."""
    out = {
        "architectures": ["Qwen3ForCausalLM"],
        "model_type": "qwen3",
        "hidden_act": "silu",
        "attention_bias": False,
        "attention_dropout": 0.0,
        "initializer_range": 0.02,
        "rope_scaling": None,
        "use_cache": True,
        "use_sliding_window": False,
        "sliding_window": None,
        "max_window_layers": cfg["num_hidden_layers"],
        "torch_dtype": "bfloat16",
        "bos_token_id": 151643,
        "eos_token_id": 151645,
    }
    out.update(cfg)
    return out


def tensor_specs(cfg: dict) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, init) in a fixed order; init is 'normal' or 'ones'."""
    H, I = cfg["hidden_size"], cfg["intermediate_size"]
    nq = cfg["num_attention_heads"] * cfg["head_dim"]
    nkv = cfg["num_key_value_heads"] * cfg["head_dim"]
    D = cfg["head_dim"]
    specs = [("model.embed_tokens.weight", (cfg["vocab_size"], H), "normal")]
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        specs += [
            (p + "input_layernorm.weight", (H,), "ones"),
            (p + "self_attn.q_proj.weight", (nq, H), "normal"),
            (p + "self_attn.k_proj.weight", (nkv, H), "normal"),
            (p + "self_attn.v_proj.weight", (nkv, H), "normal"),
            (p + "self_attn.q_norm.weight", (D,), "ones"),
            (p + "self_attn.k_norm.weight", (D,), "ones"),
            (p + "self_attn.o_proj.weight", (H, nq), "normal"),
            (p + "post_attention_layernorm.weight", (H,), "ones"),
            (p + "mlp.gate_proj.weight", (I, H), "normal"),
            (p + "mlp.up_proj.weight", (I, H), "normal"),
            (p + "mlp.down_proj.weight", (H, I), "normal"),
        ]
    specs.append(("model.norm.weight", (H,), "ones"))
    if not cfg.get("tie_word_embeddings", True):
        specs.append(("lm_head.weight", (cfg["vocab_size"], H), "normal"))
    return specs


def _chunk_seed(seed: int, tensor_idx: int, chunk_idx: int) -> int:
    return (seed * 1_000_003 + tensor_idx) * 65_537 + chunk_idx


def make_state_dict(cfg: dict, seed: int = 0, std: float = 0.02, threads: int | None = None) -> dict:
    """Host (CPU) BF16 tensors keyed by Hugging Face parameter names."""
    specs = tensor_specs(cfg)
    out = {}
    jobs = []
    for ti, (name, shape, init) in enumerate(specs):
        t = torch.empty(shape, dtype=torch.bfloat16)
        out[name] = t
        if init == "ones":
            t.fill_(1.0)
            continue
        flat = t.view(-1)
        n = flat.numel()
        for j in range((n + CHUNK - 1) // CHUNK):
            jobs.append((flat, ti, j, n))

    def work(job):
        flat, ti, j, n = job
        lo, hi = j * CHUNK, min(n, (j + 1) * CHUNK)
        g = torch.Generator().manual_seed(_chunk_seed(seed, ti, j))
        buf = torch.empty(hi - lo, dtype=torch.float32)
        buf.normal_(0.0, std, generator=g)
        flat[lo:hi].copy_(buf)

    with ThreadPoolExecutor(threads or min(16, os.cpu_count() or 1)) as ex:
        list(ex.map(work, jobs))
    return out


def write_checkpoint(path: str, cfg: dict, seed: int = 0, state: dict | None = None, shards: int = 1) -> str:
    """Write config.json and the weights under `path` (created if missing); returns path. shards == 1:
    one model.safetensors; shards > 1: model-0000i-of-0000n.safetensors files (tensors dealt out in
    order, by size) plus the model.safetensors.index.json weight map, as Hugging Face saves large
    checkpoints."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    if state is None:
        state = make_state_dict(cfg, seed)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf_config_json(cfg), f, indent=1)
    if shards <= 1:
        save_file({k: v.contiguous() for k, v in state.items()}, os.path.join(path, "model.safetensors"),
                  metadata={"format": "pt"})
    else:
        names = list(state)
        total = sum(state[n].numel() for n in names)
        groups, acc = [[] for _ in range(shards)], 0
        for n in names:  # contiguous runs of roughly total / shards elements each
            groups[min(shards - 1, acc * shards // max(total, 1))].append(n)
            acc += state[n].numel()
        weight_map = {}
        for i, group in enumerate(groups):
            fn = f"model-{i + 1:05d}-of-{shards:05d}.safetensors"
            save_file({n: state[n].contiguous() for n in group}, os.path.join(path, fn), metadata={"format": "pt"})
            weight_map.update({n: fn for n in group})
        with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {"total_size": 2 * total}, "weight_map": weight_map}, f, indent=1)
    with open(os.path.join(path, "synth.json"), "w") as f:
        json.dump({"seed": seed, "std": 0.02, "generator": "torch CPU normal_ per 4Mi-element chunk"}, f)
    return path


def random_prompt(batch: int, length: int, vocab: int = 151936, seed: int = 0) -> list[list[int]]:
    """Uniform token ids in [0, vocab) (the BASELINE workloads use uniform-random prompts)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (batch, length), generator=g).tolist()
