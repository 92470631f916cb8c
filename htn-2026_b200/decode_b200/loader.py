"""Checkpoint loading: Hugging Face Qwen3 directory -> config dict + BF16 state dict.

Replaces the reference's `AutoModelForCausalLM.from_pretrained(model_path, torch_dtype=BF16, ...)`
(engine/engine.py:237-241) with a direct safetensors read: the engine never builds a Transformers
model, it only needs the named tensors. Single-file (model.safetensors) and sharded
(model.safetensors.index.json) checkpoints are both read; tied embeddings (no lm_head.weight)
are handled by the engine.
"""

from __future__ import annotations

import json
import os

import torch

REQUIRED = ("hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
            "vocab_size", "rms_norm_eps")


def read_config(path: str) -> dict:
    with open(os.path.join(path, "config.json")) as f:
        raw = json.load(f)
    missing = [k for k in REQUIRED if k not in raw]
    if missing:
        raise ValueError(f"config.json lacks {missing}")
    cfg = {k: raw[k] for k in REQUIRED}
    cfg["head_dim"] = raw.get("head_dim") or raw["hidden_size"] // raw["num_attention_heads"]
    theta = raw.get("rope_theta")
    if theta is None and isinstance(raw.get("rope_parameters"), dict):
        theta = raw["rope_parameters"].get("rope_theta")
    cfg["rope_theta"] = float(theta if theta is not None else 10000.0)
    scaling = raw.get("rope_scaling")
    if isinstance(scaling, dict) and scaling.get("rope_type", scaling.get("type", "default")) not in ("default", None):
        raise NotImplementedError(f"rope scaling {scaling} is not supported")
    cfg["tie_word_embeddings"] = bool(raw.get("tie_word_embeddings", False))
    return cfg


def read_state(path: str, device: str = "cpu") -> dict:
    from safetensors import safe_open

    index = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(index):
        with open(index) as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
    else:
        files = [f for f in sorted(os.listdir(path)) if f.endswith(".safetensors")]
    if not files:
        raise FileNotFoundError(f"no safetensors files under {path}")
    state = {}
    for fn in files:
        with safe_open(os.path.join(path, fn), framework="pt", device=device) as f:
            for name in f.keys():
                t = f.get_tensor(name)
                state[name] = t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)
    return state


def load_checkpoint(path: str, device: str = "cpu") -> tuple[dict, dict]:
    return read_state(path, device), read_config(path)
