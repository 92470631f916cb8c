"""The checkpoint reader behind `Engine(model_path)` (decode_b200/loader.py), on the CPU: a Hugging
Face directory with one model.safetensors and the same weights split over shards with a
model.safetensors.index.json read back to identical tensors and config (the reference loads the
directory with transformers' from_pretrained, engine/engine.py:237-241)."""

import json
import os

import torch

from decode_b200 import loader, synth


def _small_cfg():
    return synth.qwen3_config(2, hidden_size=256, intermediate_size=512, vocab_size=1000, num_attention_heads=2,
                              num_key_value_heads=1)


def test_single_file_and_sharded_checkpoints_read_back_identically(tmp_path):
    cfg = _small_cfg()
    state = synth.make_state_dict(cfg, seed=3)
    one = synth.write_checkpoint(str(tmp_path / "one"), cfg, state=state)
    three = synth.write_checkpoint(str(tmp_path / "three"), cfg, state=state, shards=3)
    shards = sorted(f for f in os.listdir(three) if f.endswith(".safetensors"))
    assert shards == [f"model-0000{i}-of-00003.safetensors" for i in (1, 2, 3)]
    with open(os.path.join(three, "model.safetensors.index.json")) as f:
        assert set(json.load(f)["weight_map"]) == set(state)
    for path in (one, three):
        st, c = loader.load_checkpoint(path)
        assert set(st) == set(state)
        assert all(st[k].dtype == torch.bfloat16 and torch.equal(st[k], state[k]) for k in state)
        assert c["num_hidden_layers"] == 2 and c["hidden_size"] == 256 and c["head_dim"] == 128
        assert c["rope_theta"] == 5e6 and c["tie_word_embeddings"] is True


def test_config_rope_theta_from_rope_parameters(tmp_path):
    cfg = _small_cfg()
    path = synth.write_checkpoint(str(tmp_path / "ck"), cfg, state=synth.make_state_dict(cfg, seed=1))
    p = os.path.join(path, "config.json")
    raw = json.load(open(p))
    raw.pop("rope_theta")
    raw["rope_parameters"] = {"rope_type": "default", "rope_theta": 1234.0}
    json.dump(raw, open(p, "w"))
    assert loader.read_config(path)["rope_theta"] == 1234.0
