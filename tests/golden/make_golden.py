"""Generate the golden decode fixtures by running the reference engine itself on CPU.

Run where the reference source tree exists, naming it (there is no default location):

    QD_REFERENCE=<path to the reference checkout> python tests/golden/make_golden.py [case ...]
    python tests/golden/make_golden.py --reference <path> [case ...]

With no case names every case below is written to tests/golden/<case>.json.

For each case it builds the seeded synthetic checkpoint (decode_b200.synth), imports the reference
`engine/engine.py` with ENGINE_DEVICE=cpu and records

  * tier 0 ("native", engine/engine.py:963-972): the plain Transformers greedy loop with a KV
    cache, per-step tokens and logits;
  * tier 1 (engine/engine.py:594-643, prefill :550-592): the reference's own eager torch
    restatement of the model (packed QKV / gate-up, static cache, SDPA over the cache);
  * the teacher-forced margin of the native tokens (engine/engine.py:974-996).

Logits are summarised per step as the top-8 (value, id) pairs, the log-sum-exp and the values at
fixed probe ids, which is enough to pin greedy tokens, near-ties and the normalisation without
storing 151,936 floats per step. The output files are small JSON documents.
"""

from __future__ import annotations

import json
import os
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "htn-2026_b200"))

REFERENCE = os.environ.get("QD_REFERENCE")  # the reference checkout; set by --reference too
N_PROBES = 16
TOPK = 8

CASES = {
    # 4 layers, batch 1, 64-token uniform prompt (seed 0), 32 new tokens
    "config0": dict(layers=4, batch=1, prompt=64, new=32, prompt_seed=0),
    # batch > 1 and a short prompt (exercises per-row state and the batch dimension)
    "b3_s17": dict(layers=2, batch=3, prompt=17, new=8, prompt_seed=5),
    # BASELINE config 1 at full size: 36 layers, batch 1, 128-token uniform prompt (seed 0), 256 new
    "config1": dict(layers=36, batch=1, prompt=128, new=256, prompt_seed=0),
    # config 4's per-GPU shape (8 of the 64 sequences, 1024-token prompts) on 4 layers, 16 new tokens
    "config4_b8": dict(layers=4, batch=8, prompt=1024, new=16, prompt_seed=4),
}


def probe_ids(vocab: int) -> list[int]:
    step = vocab // N_PROBES
    return [i * step + 7 for i in range(N_PROBES)]


def summarise(logits, probes):
    import torch

    lf = logits.float()
    vals, idx = torch.topk(lf, TOPK, dim=-1)
    return {
        "top_vals": vals.tolist(),
        "top_ids": idx.tolist(),
        "lse": torch.logsumexp(lf, dim=-1).tolist(),
        "probe_vals": lf[:, probes].tolist(),
    }


def run_case(name: str, spec: dict) -> dict:
    import torch
    from decode_b200 import synth

    torch.manual_seed(0)
    cfg = synth.qwen3_config(spec["layers"])
    ckpt = tempfile.mkdtemp(prefix=f"qd_golden_{name}_")
    synth.write_checkpoint(ckpt, cfg, seed=0)
    ids = synth.random_prompt(spec["batch"], spec["prompt"], cfg["vocab_size"], seed=spec["prompt_seed"])
    N = spec["new"]
    probes = probe_ids(cfg["vocab_size"])

    os.environ["ENGINE_DEVICE"] = "cpu"
    os.environ["ENGINE_TIER"] = "0"
    sys.path.insert(0, os.path.join(REFERENCE, "engine"))
    import engine as ref  # the reference engine module (engine/engine.py)

    t0 = time.time()
    eng = ref.Engine(ckpt)
    load_s = time.time() - t0

    # tier 0: native Transformers greedy loop
    native_toks, native_steps, native_logits = [], [], []
    t0 = time.time()
    for step, logits in eng._native(ids, N):
        native_toks.append(step)
        native_steps.append(summarise(logits, probes))
        native_logits.append(logits.clone())
    native_s = time.time() - t0
    toks = [list(r) for r in zip(*native_toks)]
    margin, nonarg, first = eng._teacher_force(ids, toks)
    # the reference's own noise floor: its cached decode vs one full forward of the same tokens
    # (the replay engine/engine.py:983-985 performs), compared after log-softmax / softmax
    with torch.inference_mode():
        seqs = torch.tensor([p + t[:-1] for p, t in zip(ids, toks)], dtype=torch.int64)
        tf = eng.hf(input_ids=seqs, logits_to_keep=N, use_cache=False).logits.float()
        drift_lsm, drift_p = [], []
        for t in range(N):
            a = torch.log_softmax(native_logits[t].float(), -1)
            b = torch.log_softmax(tf[:, t], -1)
            drift_lsm.append((a - b).abs().max().item())
            drift_p.append((a.exp() - b.exp()).abs().max().item())

    # tier 1: the reference's eager torch restatement (same process, state built directly)
    ref.FORCE_TIER = 1
    st = eng._build(len(ids), len(ids[0]), N, 1)
    t1_toks, t1_steps = [], []
    with torch.inference_mode():
        st.ids.copy_(torch.tensor(ids, dtype=torch.int64))
        st.pos.fill_(len(ids[0]))
        logits = eng._prefill(st)
        t1_toks.append(st.tok.tolist())
        t1_steps.append(summarise(logits, probes))
        for t in range(1, N):
            logits = eng._decode(st, host_pos=len(ids[0]) + t - 1)
            t1_toks.append(st.tok.tolist())
            t1_steps.append(summarise(logits, probes))
    t1 = [list(r) for r in zip(*t1_toks)]

    import transformers

    return {
        "case": name,
        "spec": spec,
        "config": cfg,
        "checkpoint_seed": 0,
        "prompt": ids,
        "probe_ids": probes,
        "native": {"tokens": toks, "steps": native_steps},
        "tier1": {"tokens": t1, "steps": t1_steps},
        "teacher_forced": {"margin": margin, "non_argmax": nonarg, "first_non_argmax": first},
        "self_drift": {"max_logsoftmax_diff": max(drift_lsm), "max_prob_diff": max(drift_p),
                       "per_step_logsoftmax_diff": drift_lsm,
                       "what": "reference native cached decode vs its own teacher-forced full forward"},
        "versions": {"torch": torch.__version__, "transformers": transformers.__version__},
        "reference_calls": {
            "native": "engine/engine.py:963-972 (_native)",
            "tier1_prefill": "engine/engine.py:550-592 (_prefill)",
            "tier1_decode": "engine/engine.py:594-643 (_decode, host_pos)",
            "teacher_force": "engine/engine.py:974-996 (_teacher_force)",
        },
        "timing_s": {"load": load_s, "native": native_s},
    }


def main(argv):
    global REFERENCE
    args = list(argv[1:])
    if "--reference" in args:
        i = args.index("--reference")
        REFERENCE = args[i + 1]
        del args[i:i + 2]
        os.environ["QD_REFERENCE"] = REFERENCE  # carried into the per-case re-exec below
    if not REFERENCE or not os.path.isfile(os.path.join(REFERENCE, "engine", "engine.py")):
        sys.exit("name the reference checkout: QD_REFERENCE=<path> or --reference <path> "
                 "(it must hold engine/engine.py)")
    names = args or list(CASES)
    for name in names:
        res = run_case(name, CASES[name])
        out = os.path.join(HERE, f"{name}.json")
        with open(out, "w") as f:
            json.dump(res, f)
        nt, t1 = res["native"]["tokens"], res["tier1"]["tokens"]
        print(f"{name}: native==tier1 tokens: {nt == t1}; margin={res['teacher_forced']['margin']:.3f} "
              f"self-drift={res['self_drift']['max_logsoftmax_diff']:.4f} -> {out}", flush=True)
        # one case per process: the reference module keeps global state
        if len(names) > 1:
            os.execv(sys.executable, [sys.executable, __file__] + names[names.index(name) + 1:])


if __name__ == "__main__":
    main(sys.argv)
