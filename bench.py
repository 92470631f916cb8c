"""Decode benchmark (BASELINE.json metric: decode tokens/s and % of the HBM roofline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--layers L] ...

Default workload: BASELINE config 1, the full 36-layer Qwen3-4B architecture (seeded random-init
BF16 weights, tied embeddings), batch 1, a 128-token uniform-random prompt, greedy decode. A "step"
is one decode step (one token per sequence) through the captured CUDA graph of the engine's
hand-written kernels. The timed region holds exactly K steps bracketed by barrier + synchronize,
measured with CUDA events on the launching stream; each step streams ~8 GB of weights, far more
than the 126 MB L2, so no flush is needed between steps.

With --gpus N > 1 (one process per GPU under torchrun) every rank runs its own replica of the
workload (batch-sharded, no collective on the hot path); value = tokens of all ranks / max-over-ranks
time.

--impl reference times the reference's own CPU implementation of the path on the host cores: the
plain Transformers greedy loop (the reference's tier 0, engine/engine.py:963-972, restated in
oracle/native.py over this image's transformers) on the same model and prompt.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "htn-2026_b200"))

METRIC = "decode tokens/s (bs1 latency ms/token; bs64 aggregate) and % of HBM roofline"


def rank_reduce(x: float, op: str, device) -> float:
    """x reduced over the ranks of the default process group ("max" or "min"; a float32 tensor on
    `device`, so every rank takes the same collective step); x itself without one, or with one rank."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return x
    t = torch.tensor([x], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.MIN)
    return float(t.item())


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--layers", type=int, default=36)
    p.add_argument("--batch", type=int, default=1, help="sequences per GPU")
    p.add_argument("--prompt", type=int, default=128)
    p.add_argument("--new", type=int, default=256)
    p.add_argument("--cpu-steps", type=int, default=96, help="decode steps in the CPU baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-config4", action="store_true",
                   help="skip the config-4 leg (global batch 64 split over the ranks, prompt 1024)")
    p.add_argument("--speculate", type=int, default=0,
                   help="also time the end-to-end run with exact prompt-lookup speculation of this verify width "
                        "(batch 1; reported as e2e_speculative, not the headline)")
    p.add_argument("--tree", type=int, default=0,
                   help="also time the end-to-end run with exact token-tree speculation of this many nodes per tree "
                        "(batch 1; reported as e2e_tree, not the headline)")
    p.add_argument("--kernel", default=None, choices=["qkv", "o", "gu", "down", "lm", "attn", "attn_stream", "attn_tc", "step",
                                                      "prefill_gu", "prefill_attn", "prefill_fwd", "tree_verify"],
                   help="time one decode kernel alone (small profiling case; random packed weights on the GPU)")
    p.add_argument("--launches", type=int, default=8)
    p.add_argument("--trace", action="store_true",
                   help="with --kernel step at batch 1-3: also run one step with the per-CTA timeline stamps on and "
                        "print the per-op timeline summary")
    p.add_argument("--tc", action="store_true", help="with --kernel: the tcgen05 kernel (activations pre-packed)")
    p.add_argument("--sweep", default=None, choices=["linear", "attn", "prefill"],
                   help="BASELINE config 2 (decode linear shapes x batch x kernel path) or config 3 (GQA decode "
                        "attention); one JSON line per case")
    return p.parse_args()


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def weight_bytes(cfg) -> int:
    H, I, V, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"], cfg["num_hidden_layers"]
    nq, nkv, D = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    layer = 2 * ((nq + 2 * nkv) * D * H + H * nq * D + 2 * I * H + H * I) + 2 * (2 * H + 2 * D)
    return L * layer + 2 * V * H + 2 * H


def kv_bytes_per_token(cfg) -> int:
    return cfg["num_hidden_layers"] * 2 * cfg["num_key_value_heads"] * cfg["head_dim"] * 2


class Clocks:
    """nvidia-smi sampler over the timed region (SM clock, throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"qd_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def make_model(layers: int):
    from decode_b200 import synth

    cfg = synth.qwen3_config(layers)
    return synth.make_state_dict(cfg, seed=0), cfg


def cpu_reference(state, cfg, prompt, steps: int, threads: int | None = None, warmup: int = 0):
    """Time the reference's Transformers greedy loop (oracle.native) on the host cores: `warmup` untimed
    decode steps after the prompt, then `steps` timed ones."""
    import torch

    from oracle import native

    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    model = native.build_model(state, cfg)
    t0 = time.perf_counter()
    _, _, times = native.greedy(model, prompt, warmup + steps + 1, keep_logits=False)
    total = time.perf_counter() - t0
    dec = times[1 + warmup:]
    return {"value": len(prompt) * len(dec) / sum(dec), "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port", "ttft_s": times[0], "decode_ms_per_step": 1e3 * sum(dec) / len(dec),
            "sample": f"Transformers CPU greedy decode (reference tier 0 restated), {cfg['num_hidden_layers']} layers, "
                      f"batch {len(prompt)}, prompt {len(prompt[0])}, {len(dec)} timed decode steps after prefill "
                      f"and {warmup} untimed ones ({total:.1f} s total)"}


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    state, cfg = make_model(a.layers)
    from decode_b200 import synth

    prompt = synth.random_prompt(a.batch, a.prompt, cfg["vocab_size"], seed=0)
    steps = max(1, min(a.steps, a.cpu_steps))
    W = max(0, a.warmup)
    r = cpu_reference(state, cfg, prompt, steps, warmup=W)
    out = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": a.gpus,
           "steps": steps, "warmup": W, "ms_per_step": r["decode_ms_per_step"], "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights, "
           "uniform-random prompt)",
           "config": {"workload": f"BASELINE config 1 (Qwen3-4B arch, {a.layers} layers, batch {a.batch}, prompt "
                                  f"{a.prompt}) on host CPU", "batch": a.batch, "prompt": a.prompt, "layers": a.layers},
           "cpu_baseline": {"value": r["value"], "unit": "tokens/s", "cores": r["cores"], "kind": "port",
                            "sample": r["sample"]},
           "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def gu_kernel_roofline(eng, st, launches_per_layer=3):
    """Average duration of the gate_up GEMV (the largest decode kernel, 99.6 MB of weights per launch)
    measured with CUDA events on its launching stream, cycling through all layers' weights."""
    import torch

    L = eng.n_layers
    stream = torch.cuda.current_stream()
    if st.mode == "tc":  # tensor-core kernel on the packed activations (packing is a separate launch)
        st.xp_h.pack(st.x, eng.ln2[0], eng.eps, False)
        gu = lambda i: st.gu(st.xp_h, eng.w_gu[i], st.xp_i, pdl=False)  # noqa: E731
    else:
        gu = lambda i: st.gu(st.x, eng.w_gu[i], st.act, norm_w=eng.ln2[i], pdl=False)  # noqa: E731
    for i in range(min(L, 4)):
        gu(i)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 0
    s.record(stream)
    for _ in range(launches_per_layer):
        for i in range(L):
            gu(i)
            n += 1
    e.record(stream)
    e.synchronize()
    ms = s.elapsed_time(e) / n
    nbytes = 2 * (2 * eng.inter) * eng.hidden + 2 * st.B * eng.hidden + 2 * st.B * eng.inter
    return ms, nbytes


def _traffic_from_profile(name):
    """`key: integer` lines (DRAM bytes per launch and the algorithmic bytes of the captured case) from a
    committed ncu summary under profiles/."""
    out = {}
    try:
        for line in open(os.path.join(REPO, "profiles", name)):
            for key in ("traffic_bytes_per_launch", "algorithmic_bytes_per_launch"):
                if line.startswith(key + ":"):
                    out[key] = int(line.split(":")[1])
    except Exception:
        pass
    return out or None


def run_ours(a):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device(f"cuda:{local}"))
    import engine as E
    from decode_b200 import synth

    state, cfg = make_model(a.layers)
    eng = E.Engine.from_state_dict(state, cfg, f"cuda:{local}")
    B, S = a.batch, a.prompt
    W, K = a.warmup, a.steps
    N = max(a.new, W + K + 1)
    prompt = synth.random_prompt(B, S, cfg["vocab_size"], seed=rank)
    st = eng._build(B, S, N)

    # ---------------- device-timed decode steps (graph replays)
    with torch.inference_mode():
        st.ids.copy_(torch.tensor(prompt, dtype=torch.int64))
        st.pos.fill_(S)
        st.prefill_graph.replay()
        for _ in range(W):
            st.decode_graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        t_s, t_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local) as clk:
            torch.cuda.nvtx.range_push("timed")
            t_s.record(stream)
            for _ in range(K):
                st.decode_graph.replay()
            t_e.record(stream)
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_pop()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        eng.check_device_errors(st)
    ms = t_s.elapsed_time(t_e)
    ms_max = rank_reduce(ms, "max", f"cuda:{local}")
    ms_step = ms_max / K
    value = world * B * K / (ms_max / 1e3)

    # ---------------- end to end through the public API (host lists in, host lists out)
    e2e = None
    if not a.no_e2e:
        n_e2e = a.new
        list(eng.generate(prompt, n_e2e))  # untimed: builds and captures the (B, S, n_e2e) shape
        stamps = []
        t0 = time.perf_counter()
        for _ in eng.generate(prompt, n_e2e):
            stamps.append(time.perf_counter())
        total = stamps[-1] - t0
        dec = stamps[-1] - stamps[0]
        e2e_val = B * (n_e2e - 1) / dec if n_e2e > 1 else 0.0
        if world > 1:
            e2e_val = rank_reduce(e2e_val, "min", f"cuda:{local}") * world
        e2e = {"value": e2e_val, "unit": "tokens/s", "h2d_bytes_per_step": round(B * S * 8 / n_e2e, 1),
               "d2h_bytes_per_step": B * 8, "ttft_ms": 1e3 * (stamps[0] - t0),
               "total_tokens_per_s_incl_prefill": world * B * n_e2e / total,
               "note": "decode tokens/s between the first and last yield of Engine.generate (host prompt list in, "
                       "host token lists out); the prompt upload is amortised over the steps in h2d_bytes_per_step"}

    e2e_spec = None
    if a.speculate and B == 1 and a.new > 1:
        # exact prompt-lookup speculation (engine/engine.py:759-828) through the same public call; the
        # emitted tokens must equal the plain run's up to a near-tie flip
        plain = [t[0] for t in eng.generate(prompt, a.new)]
        eng.speculate = a.speculate
        list(eng.generate(prompt, a.new))  # untimed: builds the state with the verify buffers
        stamps = []
        t0 = time.perf_counter()
        for _ in eng.generate(prompt, a.new):
            stamps.append(time.perf_counter())
        spec_toks = [t[0] for t in eng.generate(prompt, a.new)]
        verifies, plain_steps = eng.state.spec_stats["verifies"], eng.state.spec_stats["plain_steps"]
        eng.speculate = 0
        eng.state = None
        same = next((i for i, (x, y) in enumerate(zip(plain, spec_toks)) if x != y), len(plain))
        dec = stamps[-1] - stamps[0]
        e2e_spec = {"value": round((a.new - 1) / dec, 2), "unit": "tokens/s", "verify_width": a.speculate,
                    "verifies": verifies, "plain_steps": plain_steps,
                    "tokens_per_verify": round((a.new - 1 - plain_steps) / max(verifies, 1), 3),
                    "ttft_ms": round(1e3 * (stamps[0] - t0), 3), "tokens_equal_to_plain": same,
                    "note": "decode tokens/s between the first and last yield of Engine.generate with speculation; "
                            "the prompt and the random-init weights decide how many drafts are accepted"}

    e2e_tree = None
    if a.tree and B == 1 and a.new > 1:
        # exact token-tree speculation through the same public call; its tokens must equal the plain run's
        # up to a near-tie flip
        plain = [t[0] for t in eng.generate(prompt, a.new)]
        eng.tree = a.tree
        list(eng.generate(prompt, a.new))  # untimed: builds the state with the tree buffers
        stamps = []
        t0 = time.perf_counter()
        for _ in eng.generate(prompt, a.new):
            stamps.append(time.perf_counter())
        tree_toks = [t[0] for t in eng.generate(prompt, a.new)]
        stats = dict(eng.state.spec_stats)
        tv, st_t = eng.state.tree, eng.state
        # one verify of a full tree alone, device time (the prefix at the prompt's end)
        from decode_b200 import tree as tree_mod

        probe = tree_mod.TokenTree(prompt[0][-1], a.tree)
        while len(probe) < a.tree:
            probe.insert([len(probe) % 1000, (len(probe) * 7) % 1000], 4)
        with torch.inference_mode():
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            tv(eng, st_t, [probe], [S - 1])
            ev[0].record()
            for _ in range(5):
                tv(eng, st_t, [probe], [S - 1])
            ev[1].record()
            ev[1].synchronize()
        eng.tree = 0
        eng.state = None
        same = next((i for i, (x, y) in enumerate(zip(plain, tree_toks)) if x != y), len(plain))
        dec = stamps[-1] - stamps[0]
        e2e_tree = {"value": round((a.new - 1) / dec, 2), "unit": "tokens/s", "tree_nodes": a.tree,
                    "verifies": stats["verifies"], "plain_steps": stats["plain_steps"],
                    "accepted_drafts": stats["accepted"], "verify_ms": round(ev[0].elapsed_time(ev[1]) / 5, 3),
                    "tokens_equal_to_plain": same,
                    "note": "decode tokens/s between the first and last yield of Engine.generate with token trees; "
                            "verify_ms = one verify of a full tree including its host round trip; the prompt and "
                            "the random-init weights decide how many drafts are accepted"}

    # ---------------- roofline of the dominant kernel and of the whole step
    peak, peak_kind = _peaks()
    L_avg = S + W + K / 2
    step_bytes = weight_bytes(cfg) + B * kv_bytes_per_token(cfg) * (L_avg + 1)
    step_gbs = step_bytes / (ms_step / 1e3) / 1e9
    gu_ms, gu_bytes = gu_kernel_roofline(eng, st)
    gu_gbs = gu_bytes / (gu_ms / 1e3) / 1e9
    persistent = st.mode == "persistent"
    if persistent:
        # the timed region is one launch of the persistent step kernel per step: it is the kernel
        prof = _traffic_from_profile("decode_step_kernel_b1.md")
        traffic = None
        if prof:  # ncu capture of a smaller (fewer layers) step, scaled by algorithmic bytes
            traffic = round(prof["traffic_bytes_per_launch"] * step_bytes / prof["algorithmic_bytes_per_launch"])
        roofline = {"bound": "hbm", "kernel": "qd step_kernel<1> (persistent whole decode step, 1 launch/step)",
                    "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(step_gbs / peak, 4),
                    "peak_kind": peak_kind, "avg_launch_us": round(ms_step * 1e3, 2),
                    "algorithmic_bytes": int(step_bytes), "traffic": traffic}
    else:
        prof = _traffic_from_profile("gemv_gate_up_b1_full.md")
        roofline = {"bound": "hbm", "kernel": "qd gemv gate_up+SwiGLU (99.6 MB weights/launch)",
                    "achieved": round(gu_gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(gu_gbs / peak, 4),
                    "peak_kind": peak_kind, "avg_launch_us": round(gu_ms * 1e3, 2), "algorithmic_bytes": gu_bytes,
                    "traffic": (prof or {}).get("traffic_bytes_per_launch")}

    c4 = None
    if not a.no_config4 and a.layers == 36:
        c4 = config4_leg(eng, cfg, a, world, rank, local, peak)

    cpu = None
    if rank == 0 and not a.no_cpu_baseline:
        try:
            cpu = cpu_reference(state, cfg, prompt, a.cpu_steps)
        except Exception as exc:  # a baseline failure must not hide the GPU number
            cpu = {"value": None, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": f"failed: {repr(exc)[:200]}"}

    if rank == 0:
        out = {"metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": K,
               "warmup": W, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init BF16 weights, "
               "uniform-random prompt ids)",
               "config": {"workload": f"BASELINE config {'1' if (a.layers == 36 and B == 1) else 'custom'}: Qwen3-4B "
                                      f"arch {a.layers} layers, batch {B}/GPU, prompt {S}, greedy decode steps",
                          "batch_per_gpu": B, "global_batch": B * world, "prompt": S, "layers": a.layers,
                          "parallelism": f"batch-sharded replicas x{world} (no collective)",
                          "l2": "inputs larger than L2 (~8 GB of weights per step)"},
               "roofline": roofline,
               "step_roofline": {"bytes_per_step": step_bytes, "achieved": round(step_gbs, 1), "peak": peak,
                                 "unit": "GB/s", "frac": round(step_gbs / peak, 4),
                                 "roofline_tokens_per_s": round(world * B * peak * 1e9 / step_bytes, 1)},
               "kernel_rooflines": {"gate_up_gemv_per_op_kernel": {
                   "achieved": round(gu_gbs, 1), "avg_launch_us": round(gu_ms * 1e3, 2),
                   "frac": round(gu_gbs / peak, 4), "algorithmic_bytes": gu_bytes}},
               "step_mode": st.mode + ("+persistent" if st.tstep is not None else ""),
               "clocks": clk.summary(), "e2e": e2e, "cpu_baseline": cpu,
               "gpu_launches": K * (1 if st.tstep is not None else
                                    {"persistent": 1, "kernels": 2 + 5 * a.layers, "tc": 3 + 7 * a.layers}[st.mode])}
        if e2e_spec is not None:
            out["e2e_speculative"] = e2e_spec
        if c4 is not None:
            out["config4"] = c4
        if e2e_tree is not None:
            out["e2e_tree"] = e2e_tree
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def config4_leg(eng, cfg, a, world, rank, local, peak):
    """BASELINE config 4 under the same launch: a global batch of 64 sequences (prompt 1024, 512 new)
    split over the ranks (64 / N each, the shard launcher's contiguous split), no collective on the hot
    path. Each rank runs its own prompt forward and then decode steps; K steps (at most 64) are timed on
    the device, centred on the middle of the 512 new tokens (the steps before them run untimed), between
    barriers, and the max over ranks is taken. value = 64 * K / that time. The per-GPU roofline counts
    the weights plus the rank's KV cache read at the timed positions."""
    import torch
    import torch.distributed as dist

    from decode_b200 import shard, synth

    GB, S, NEW = 64, 1024, 512
    lo, hi = shard.split_rows(GB, world)[rank] if rank < min(world, GB) else (0, 0)
    b = hi - lo
    K = max(1, min(a.steps, 64))
    W = max(3, NEW // 2 - K // 2)
    prompt = synth.random_prompt(GB, S, cfg["vocab_size"], seed=4)[lo:hi]
    eng.state = None
    st = eng._build(b, S, NEW)
    with torch.inference_mode():
        st.ids.copy_(torch.tensor(prompt, dtype=torch.int64))
        st.pos.fill_(S)
        st.prefill_graph.replay()
        for _ in range(W):
            st.decode_graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        t_s, t_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t_s.record(stream)
        for _ in range(K):
            st.decode_graph.replay()
        t_e.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        eng.check_device_errors(st)
    ms = t_s.elapsed_time(t_e)
    ms_max = rank_reduce(ms, "max", f"cuda:{local}")
    L_avg = S + W + K / 2
    step_bytes = weight_bytes(cfg) + b * kv_bytes_per_token(cfg) * (L_avg + 1)
    per_gpu = step_bytes / (ms / K / 1e3) / 1e9
    mode = st.mode + ("+persistent" if st.tstep is not None else ("+chain" if st.mode == "tc" else ""))
    eng.state = None
    return {"workload": "BASELINE config 4: Qwen3-4B arch 36 layers, global batch 64 split over the GPUs, "
                        "prompt 1024, decode steps timed at new tokens "
                        f"{W + 1}..{W + K} of 512", "value": round(GB * K / (ms_max / 1e3), 1),
            "unit": "tokens/s", "global_batch": GB, "batch_per_gpu": b, "n_gpus": world, "steps": K,
            "ms_per_step": round(ms_max / K, 4), "step_mode": mode, "scaling": "strong",
            "roofline_per_gpu": {"bytes_per_step": int(step_bytes), "achieved": round(per_gpu, 1), "peak": peak,
                                 "unit": "GB/s", "frac": round(per_gpu / peak, 4)},
            "roofline_tokens_per_s": round(GB * peak * 1e9 / step_bytes, 1)}


def run_prefill_forward(a):
    """The engine's whole prompt forward (`--layers` layers, batch 1, `--prompt` tokens; random-init
    weights) as a CUDA graph replayed `--launches` times after the engine's own build: the profiling
    case for the launch list of the time to first token. Prints avg ms per forward and the number of
    library kernels one forward launches."""
    import torch

    import engine as E

    state, cfg = make_model(a.layers)
    eng = E.Engine.from_state_dict(state, cfg, "cuda:0")
    del state
    st = eng._build(1, a.prompt, 1)
    with torch.inference_mode():
        st.ids.copy_(torch.tensor(synth_prompt(1, a.prompt), dtype=torch.int64))
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(a.launches):
        st.prefill_graph.replay()
    e.record()
    e.synchronize()
    eng.check_device_errors(st)
    with qdlib_recording() as rec:
        eng._prefill(st)
    print(json.dumps({"kernel": "prefill_fwd", "layers": a.layers, "prompt": a.prompt, "launches": a.launches,
                      "avg_ms": round(s.elapsed_time(e) / a.launches, 3),
                      "library_launches_per_forward": sum(1 for name, _ in rec if not name.endswith("_plan"))}))


def run_tree_verify(a):
    """Token-tree verify forwards (`--layers` layers, `--batch` sequences of `--prompt` tokens, one tree of
    `--tree` nodes per sequence cut to 64 // batch; random-init weights): the prompt forward, then
    `--launches` verifies of full trees at the prompt's end, each with its host round trip (upload of
    the trees, launches, greedy tokens back). Prints avg ms per verify and the library launches of one
    verify; one further verify runs inside the NVTX range "tree_verify" for a launch-list capture."""
    import random

    import torch

    import engine as E
    from decode_b200 import tree as TT

    B, S = a.batch, a.prompt
    state, cfg = make_model(a.layers)
    eng = E.Engine.from_state_dict(state, cfg, "cuda:0")
    del state
    eng.tree = a.tree or 32
    st = eng._build(B, S, max(2, a.new))
    tv = st.tree
    prompt = synth_prompt(B, S)
    with torch.inference_mode():
        eng._upload_prompt(st, prompt)
        eng._enqueue_prefill(st)
    rnd = random.Random(0)
    trees = []
    for b in range(B):
        t = TT.TokenTree(prompt[b][-1], tv.T)
        while len(t) < tv.T:
            t.insert([rnd.randrange(cfg["vocab_size"]) for _ in range(rnd.randrange(1, tv.depth + 1))], tv.depth)
        trees.append(t)
    pos0s = [S - 1] * B
    for _ in range(3):
        tv(eng, st, trees, pos0s)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(a.launches):
        tv(eng, st, trees, pos0s)
    e.record()
    e.synchronize()
    torch.cuda.nvtx.range_push("tree_verify")  # one more verify, as an NVTX range for a launch-list capture
    tv(eng, st, trees, pos0s)
    torch.cuda.nvtx.range_pop()
    eng.check_device_errors(st)
    n_calls = len(tv.calls)
    print(json.dumps({"kernel": "tree_verify", "layers": a.layers, "batch": B, "prompt": S, "tree_nodes": tv.T,
                      "rows": tv.M, "launches": a.launches, "avg_ms": round(s.elapsed_time(e) / a.launches, 3),
                      "library_launches_per_verify": n_calls,
                      "note": "each verify includes its host round trip; the engine build runs 2 verifies and "
                              "this mode 3 more before the timed ones"}))


def qdlib_recording():
    from decode_b200 import lib as qdlib

    return qdlib.recording()


def run_prefill_kernel(a):
    """One prompt kernel alone on `--prompt` tokens of one sequence (profiling case): prefill_gu is
    qd_tc_gemm with the SwiGLU epilogue on the gate/up shape (x [S, 2560] N(0, 1), packed weights
    N(0, 0.02)); prefill_attn is qd_prefill_attn over the whole prompt (q, K, V N(0, 1), 32 q / 8 KV
    heads). Prints avg us and TFLOP/s over `--launches` launches after three warm-up launches."""
    import torch

    from decode_b200 import ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    S, H, I, nq, nkv, D = a.prompt, 2560, 9728, 32, 8, 128
    g = torch.Generator(device=dev).manual_seed(0)
    err = torch.zeros((1,), dtype=torch.int32, device=dev)
    if a.kernel == "prefill_gu":
        x = torch.randn((S, H), generator=g, device=dev).to(torch.bfloat16)
        w = ops.pack_matrix((torch.randn((2 * I, H), generator=g, device=dev) * 0.02).to(torch.bfloat16))
        out = torch.empty((S, I), dtype=torch.bfloat16, device=dev)
        fn = lambda i: ops.tc_gemm(x, w, 2 * I, out, epilogue=ops.Gemv.SWIGLU, err=err)  # noqa: E731
        flops = 2 * S * 2 * I * H
    else:
        q = torch.randn((S, nq * D), generator=g, device=dev).to(torch.bfloat16)
        kc = torch.randn((1, nkv, S, D), generator=g, device=dev).to(torch.bfloat16)
        vc = torch.randn((1, nkv, S, D), generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty((S, nq * D), dtype=torch.bfloat16, device=dev)
        fn = lambda i: ops.prefill_attn(q, 1, S, nq, nkv, kc, vc, out, err=err)  # noqa: E731
        flops = 4 * nq * (S * (S + 1) // 2) * D
    ms = _time_cycle(fn, 1, a.launches)
    assert int(err.item()) == 0
    tf = flops / (ms / 1e3) / 1e12
    print(json.dumps({"kernel": a.kernel, "prompt": S, "launches": a.launches, "avg_us": round(ms * 1e3, 2),
                      "TFLOPs": round(tf, 1), "frac_of_peak": round(tf / _tensor_peak(), 4),
                      "peak_tflops": _tensor_peak()}))


def run_kernel(a):
    """One decode kernel alone, cycling over `--layers` copies of its weights (random, packed on the
    GPU; > L2 from 2 copies for gate_up, down and the LM head), for profiling. Prints avg µs and GB/s."""
    import torch

    from decode_b200 import ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    if a.kernel == "step":
        return run_step_kernel(a)
    if a.kernel == "prefill_fwd":
        return run_prefill_forward(a)
    if a.kernel == "tree_verify":
        return run_tree_verify(a)
    if a.kernel in ("prefill_gu", "prefill_attn"):
        return run_prefill_kernel(a)
    H, I, V, nq, nkv, D, B, L = 2560, 9728, 151936, 32, 8, 128, a.batch, a.layers
    g = torch.Generator(device=dev).manual_seed(0)
    rnd = lambda *shape: (torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)  # noqa: E731
    x = torch.randn((B, I), generator=g, device=dev).to(torch.bfloat16)
    xh = x[:, :H].contiguous()
    nw = torch.ones(H, dtype=torch.bfloat16, device=dev)
    err = torch.zeros((1,), dtype=torch.int32, device=dev)
    cap = a.prompt + a.new
    pos = torch.tensor([cap - 1], dtype=torch.int64, device=dev)
    if a.kernel in ("attn", "attn_stream", "attn_tc"):
        kc = torch.randn((L, B, nkv, cap, D), generator=g, device=dev).to(torch.bfloat16)
        vc = torch.randn((L, B, nkv, cap, D), generator=g, device=dev).to(torch.bfloat16)
        q = torch.randn((B, nq, D), generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty((B, nq, D), dtype=torch.bfloat16, device=dev)
        attn = {"attn": ops.DecodeAttention, "attn_stream": ops.DecodeAttentionStream,
                "attn_tc": ops.DecodeAttentionTc}[a.kernel](B, nq, nkv, cap, dev)
        fn = lambda i: attn(q, kc[i], vc[i], pos, out, err=err, pdl=False)  # noqa: E731
        nbytes = 2 * B * nkv * cap * D * 2 + 2 * B * nq * D * 2
    else:
        shapes = {"qkv": ((nq + 2 * nkv) * D, H), "o": (H, nq * D), "gu": (2 * I, H), "down": (H, I), "lm": (V, H)}
        n, k = shapes[a.kernel]
        ws = [ops.pack_matrix(rnd(n, k)) for _ in range(L)]
        if a.tc:
            xp = ops.PackedActivations(B, k, dev).pack(x[:, :k].contiguous())
            outb = torch.zeros((B, n), dtype=torch.bfloat16, device=dev)
            if a.kernel == "lm":
                plan = ops.TcLmHeadArgmax(B, V, H, dev)
                tok = torch.zeros((B,), dtype=torch.int64, device=dev)
                fn = lambda i: plan(xp, ws[i], tok, err=err, pdl=False)  # noqa: E731
            else:
                epi = {"o": ops.TcGemv.RES, "gu": ops.TcGemv.SWIGLU, "down": ops.TcGemv.RES,
                       "qkv": ops.TcGemv.STORE}[a.kernel]
                plan = ops.TcGemv(B, n, k, epi, dev)
                if epi == ops.TcGemv.RES:
                    fn = lambda i: plan(xp, ws[i], outb, res=outb, err=err, pdl=False)  # noqa: E731
                else:
                    o = outb[:, : n // 2] if epi == ops.TcGemv.SWIGLU else outb
                    fn = lambda i: plan(xp, ws[i], o, err=err, pdl=False)  # noqa: E731
        elif a.kernel == "qkv":
            from engine import rope_tables

            cos, sin = (t.to(dev) for t in rope_tables(cap, D, 5e6))
            kc = torch.zeros((B, nkv, cap, D), dtype=torch.bfloat16, device=dev)
            vc = torch.zeros_like(kc)
            q = torch.empty((B, nq, D), dtype=torch.bfloat16, device=dev)
            plan = ops.QkvRopeAppend(B, H, nq, nkv, dev)
            qn = torch.ones(D, dtype=torch.bfloat16, device=dev)
            fn = lambda i: plan(xh, ws[i], nw, qn, qn, cos, sin, pos, q, kc, vc, err=err, pdl=False)  # noqa: E731
        elif a.kernel == "lm":
            plan = ops.LmHeadArgmax(B, V, H, dev)
            tok = torch.zeros((B,), dtype=torch.int64, device=dev)
            fn = lambda i: plan(xh, ws[i], nw, tok, err=err, pdl=False)  # noqa: E731
        else:
            epi = {"o": ops.Gemv.RES, "gu": ops.Gemv.SWIGLU, "down": ops.Gemv.RES}[a.kernel]
            plan = ops.Gemv(B, n, k, epi, dev)
            xin = x[:, :k].contiguous()
            outb = torch.zeros((B, n), dtype=torch.bfloat16, device=dev)
            if epi == ops.Gemv.RES:
                fn = lambda i: plan(xin, ws[i], outb, res=outb, err=err, pdl=False)  # noqa: E731
            else:
                fn = lambda i: plan(xin, ws[i], outb[:, : n // 2], norm_w=nw, err=err, pdl=False)  # noqa: E731
        nbytes = n * k * 2 + B * k * 2 + B * n * 2
    for i in range(min(3, a.launches)):
        fn(i % L)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(a.launches):
        fn(i % L)
    e.record()
    e.synchronize()
    us = s.elapsed_time(e) / a.launches * 1e3
    assert int(err.item()) == 0
    peak, kind = _peaks()
    print(json.dumps({"kernel": a.kernel + ("_tc" if a.tc else ""), "batch": B, "copies": L,
                      "launches": a.launches, "avg_us": round(us, 2),
                      "algorithmic_bytes": nbytes, "achieved_GBs": round(nbytes / us / 1e3, 1),
                      "frac_of_peak": round(nbytes / us / 1e3 / peak, 4), "peak": peak, "peak_kind": kind}))


def run_step_kernel(a):
    """One decode step alone on a `--layers`-layer synthetic model (profiling case): the persistent step
    kernel at batch 1-3, the persistent tcgen05 step at batch 4-12, the tcgen05 chain above (or with
    ENGINE_TC_STEP=chain)."""
    import torch

    import engine as E

    state, cfg = make_model(a.layers)
    eng = E.Engine.from_state_dict(state, cfg, "cuda:0")
    del state
    B, S = a.batch, a.prompt
    st = eng._build(B, S, a.launches + 8)
    with torch.inference_mode():
        st.ids.copy_(torch.tensor(synth_prompt(B, S), dtype=torch.int64))
        st.pos.fill_(S)
        st.prefill_graph.replay()
        step = st.step or st.tstep or (lambda: eng._decode_step(st))
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.launches):
            step()
        e.record()
        e.synchronize()
        torch.cuda.nvtx.range_push("decode_step")  # one more step, as an NVTX range for launch-list captures
        step()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    eng.check_device_errors(st)
    us = s.elapsed_time(e) / a.launches * 1e3
    nbytes = weight_bytes(cfg) + B * kv_bytes_per_token(cfg) * (S + 3 + a.launches / 2 + 1)
    peak, kind = _peaks()
    mode = "step" if st.step else ("tc_step" if st.tstep else "tc_chain")
    print(json.dumps({"kernel": mode, "layers": a.layers, "batch": B, "launches": a.launches, "avg_us": round(us, 2),
                      "algorithmic_bytes": int(nbytes), "achieved_GBs": round(nbytes / us / 1e3, 1),
                      "frac_of_peak": round(nbytes / us / 1e3 / peak, 4), "peak": peak, "peak_kind": kind}))
    if a.trace and st.step is not None:
        print(json.dumps(step_timeline(eng, st, cfg, peak)))


OPS = ("qkv", "attn", "o", "gate_up", "down")


def step_timeline(eng, st, cfg, peak):
    """One persistent decode step (batch 1-3) with its timeline stamps on: per CTA and op, %globaltimer at
    0 = input ready (its dependency wait passed), 1 = input staged in shared memory, 2 = the op's blocks
    consumed and its segments flushed (finalize epilogues included), 3 = the producer issued the op's
    last weight block. Summarised over the middle layers (first and last two left out) as times
    relative to the previous op's last `done` (the critical path), and the interval the producer spent
    issuing each projection's blocks against that projection's streaming time at the peak."""
    import statistics

    import torch

    from decode_b200 import ops

    L, G = eng.n_layers, ops.sm_count()
    nops = 2 + 5 * L
    trace = torch.zeros((G * nops * 4,), dtype=torch.int64, device=eng.device)
    traced = ops.DecodeStep(eng, st, trace=trace)
    with torch.inference_mode():
        st.step()
        traced()
        torch.cuda.synchronize()
    eng.check_device_errors(st)
    t = trace.view(G, nops, 4).cpu().double()
    t0 = float(t[:, 0, 2].min())  # embedding done on the first CTA
    t = (t - t0) / 1e3               # microseconds from the step's start
    H, I, nq, nkv = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"]
    wbytes = {"qkv": 2 * (nq + 2 * nkv) * 128 * H, "attn": 0, "o": 2 * H * nq * 128, "gate_up": 4 * I * H,
              "down": 2 * H * I}
    layers = list(range(2, L - 2)) if L > 5 else list(range(1, L))
    med = lambda v: round(statistics.median(v), 2) if v else None  # noqa: E731
    rows = {}
    def pct5(v):  # min, quartiles, max of the per-CTA values
        v = sorted(v)
        n = len(v)
        return [v[0], v[n // 4], v[n // 2], v[(3 * n) // 4], v[-1]]

    for k, name in enumerate(OPS):
        wait, stage, work, issue, span, done_dist, issue_dist = [], [], [], [], [], [], []
        for l in layers:
            op, prev = 1 + 5 * l + k, 1 + 5 * l + k - 1
            prev_done = float(t[:, prev, 2].max())
            ready = float(t[:, op, 0].max())
            done = float(t[:, op, 2].max())
            wait.append(ready - prev_done)
            span.append(done - prev_done)
            done_dist.append(pct5((t[:, op, 2] - prev_done).tolist()))
            if name != "attn":
                issue_dist.append(pct5((t[:, op, 3] - prev_done).tolist()))
            if name != "attn":  # the attention op records no `staged` stamp and streams no weights
                staged = float(t[:, op, 1].max())
                stage.append(staged - ready)
                work.append(done - staged)
                prev_proj = {0: 1 + 5 * (l - 1) + 4, 2: 1 + 5 * l, 3: 1 + 5 * l + 2, 4: 1 + 5 * l + 3}[k]
                issue.append(float(t[:, op, 3].max()) - float(t[:, prev_proj, 3].max()))
        rows[name] = {"wait_us": med(wait), "stage_us": med(stage), "work_us": med(work), "span_us": med(span),
                      "producer_issue_interval_us": med(issue),
                      "stream_us_at_peak": round(wbytes[name] / (peak * 1e3), 2),
                      # per-CTA spread, each quantile the median over the layers, relative to the previous
                      # op's last done: when the CTAs finished (flushes and epilogues included) and when
                      # their producers issued the op's last weight block
                      "cta_done_min_q1_med_q3_max_us": [med([d[i] for d in done_dist]) for i in range(5)],
                      "cta_last_block_issued_min_q1_med_q3_max_us":
                          [med([d[i] for d in issue_dist]) for i in range(5)] if issue_dist else None}
    layer_us = [float(t[:, 1 + 5 * (l + 1), 0].max()) - float(t[:, 1 + 5 * l, 0].max()) for l in layers[:-1]]
    lm = 1 + 5 * L
    return {"timeline": "persistent step, per-op medians over layers %d..%d" % (layers[0], layers[-1]),
            "layer_us": med(layer_us), "layer_stream_us_at_peak": round(sum(wbytes.values()) / (peak * 1e3), 2),
            "ops": rows, "lm_head_span_us": round(float(t[:, lm, 2].max()) - float(t[:, lm - 1, 2].max()), 2),
            "step_us": round(float(t[:, lm, 2].max()), 2),
            "definitions": {"wait": "last CTA past its dependency wait - previous op's last done",
                            "stage": "last CTA staged - last CTA ready", "work": "last done - last staged",
                            "span": "last done - previous op's last done",
                            "producer_issue_interval": "producer's last block of this projection issued - its last "
                                                       "block of the previous projection (max over CTAs)"}}


def _time_cycle(fn, copies, launches):
    """Average device time of fn(i) in ms, cycling over `copies` operand sets (CUDA events on the
    launching stream, after warm-up)."""
    import torch

    for i in range(min(3, launches)):
        fn(i % copies)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(launches):
        fn(i % copies)
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / launches


def _time_graph(fn, copies, launches):
    """Average device time of fn(i) in ms with the launches captured in one CUDA graph (as the engine
    replays them: no host launch cost), cycling over `copies` operand sets."""
    import torch

    for i in range(min(3, launches)):
        fn(i % copies)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(launches):
            fn(i % copies)
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(3):
        g.replay()
    e.record()
    e.synchronize()
    del g
    return s.elapsed_time(e) / (3 * launches)


def run_sweep_linear(a):
    """the five decode projections (K -> N) at M in {1, 4, 16, 64}, each with its plain
    BF16 store and with its fused epilogue, on three paths:
      cuda_core  the streaming GEMV (qd_gemv / qd_qkv_rope_append / qd_lm_head_argmax), M > 8 as
                 ceil(M / 8) launches of 8 rows (each re-streams the weights)
      tc         the tcgen05 kernels (qd_tc_*), timed alone and with the activation packing launch
      cublas     torch F.linear on row-major weights (store only), the library baseline
    Weights N(0, 0.02), activations N(0, 1), seed 1; every case cycles over enough weight copies to
    exceed twice the L2. Bytes = 2NK + 2MK + 2MN (+ 2MN for a residual read); flops = 2MNK."""
    import torch
    import torch.nn.functional as F

    from decode_b200 import ops
    from engine import rope_tables

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    peak, kind = _peaks()
    tpeak = _tensor_peak()
    H, I, V, nq, nkv, D = 2560, 9728, 151936, 32, 8, 128
    shapes = [("qkv", (nq + 2 * nkv) * D, H), ("o", H, nq * D), ("gu", 2 * I, H), ("down", H, I), ("lm", V, H)]
    g = torch.Generator(device=dev).manual_seed(1)
    err = torch.zeros((1,), dtype=torch.int32, device=dev)
    cap = 64
    cos, sin = (t.to(dev) for t in rope_tables(cap, D, 5e6))
    pos = torch.tensor([cap - 1], dtype=torch.int64, device=dev)
    ones_d = torch.ones(D, dtype=torch.bfloat16, device=dev)
    launches = max(a.launches, 24)
    for name, n, k in shapes:
        copies = max(2, -(-(300 << 20) // (2 * n * k)))
        wrm = [(torch.randn((n, k), generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(copies)]
        wpk = [ops.pack_matrix(w) for w in wrm]
        ones_k = torch.ones(k, dtype=torch.bfloat16, device=dev)
        for M in (1, 4, 16, 64):
            x = torch.randn((M, k), generator=g, device=dev).to(torch.bfloat16)
            base = 2 * n * k + 2 * M * k + 2 * M * n
            cases = []
            # ---- cuda-core GEMV path (chunks of at most 8 rows)
            chunks = [(r, min(M, r + 8)) for r in range(0, M, 8)]
            for epi in ("store", "fused"):
                outb = torch.zeros((M, n), dtype=torch.bfloat16, device=dev)
                if name == "lm" and epi == "fused":
                    plans = [ops.LmHeadArgmax(r1 - r0, V, k, dev) for r0, r1 in chunks]
                    tok = torch.zeros((M,), dtype=torch.int64, device=dev)

                    def fn(i, plans=plans, tok=tok, x=x):
                        for (r0, r1), p in zip(chunks, plans):
                            p(x[r0:r1], wpk[i], ones_k, tok[r0:r1], err=err, pdl=False)
                elif name == "qkv" and epi == "fused":
                    plans = [ops.QkvRopeAppend(r1 - r0, k, nq, nkv, dev) for r0, r1 in chunks]
                    kc = torch.zeros((M, nkv, cap, D), dtype=torch.bfloat16, device=dev)
                    vc, q = torch.zeros_like(kc), torch.empty((M, nq, D), dtype=torch.bfloat16, device=dev)

                    def fn(i, plans=plans, kc=kc, vc=vc, q=q, x=x):
                        for (r0, r1), p in zip(chunks, plans):
                            p(x[r0:r1], wpk[i], ones_k, ones_d, ones_d, cos, sin, pos, q[r0:r1], kc[r0:r1],
                              vc[r0:r1], err=err, pdl=False)
                else:
                    e = ops.Gemv.STORE
                    if epi == "fused":
                        e = {"o": ops.Gemv.RES, "down": ops.Gemv.RES, "gu": ops.Gemv.SWIGLU}[name]
                    plans = [ops.Gemv(r1 - r0, n, k, e, dev) for r0, r1 in chunks]

                    def fn(i, plans=plans, e=e, outb=outb, x=x):
                        for (r0, r1), p in zip(chunks, plans):
                            if e == ops.Gemv.RES:
                                p(x[r0:r1], wpk[i], outb[r0:r1], res=outb[r0:r1], err=err, pdl=False)
                            elif e == ops.Gemv.SWIGLU:
                                p(x[r0:r1], wpk[i], outb[r0:r1, : n // 2], norm_w=ones_k, err=err, pdl=False)
                            else:
                                p(x[r0:r1], wpk[i], outb[r0:r1], err=err, pdl=False)
                cases.append(("cuda_core", epi, fn, len(chunks)))
            # ---- tensor-core path
            xp = ops.PackedActivations(M, k, dev)
            xp.pack(x)
            for epi in ("store", "fused"):
                outb = torch.zeros((M, n), dtype=torch.bfloat16, device=dev)
                norm = None
                if name == "lm" and epi == "fused":
                    p = ops.TcLmHeadArgmax(M, V, k, dev)
                    tok = torch.zeros((M,), dtype=torch.int64, device=dev)
                    op = lambda i, p=p, tok=tok: p(xp, wpk[i], tok, err=err, pdl=False)  # noqa: E731
                    norm = ones_k
                elif name == "qkv" and epi == "fused":
                    p = ops.TcQkvRopeAppend(M, k, nq, nkv, dev)
                    kc = torch.zeros((M, nkv, cap, D), dtype=torch.bfloat16, device=dev)
                    vc, q = torch.zeros_like(kc), torch.empty((M, nq, D), dtype=torch.bfloat16, device=dev)
                    op = lambda i, p=p, kc=kc, vc=vc, q=q: p(xp, wpk[i], ones_d, ones_d, cos, sin, pos, q, kc,  # noqa: E731
                                                             vc, err=err, pdl=False)
                    norm = ones_k
                else:
                    e = ops.TcGemv.STORE
                    if epi == "fused":
                        e = {"o": ops.TcGemv.RES, "down": ops.TcGemv.RES, "gu": ops.TcGemv.SWIGLU}[name]
                        norm = ones_k if name == "gu" else None
                    p = ops.TcGemv(M, n, k, e, dev)
                    if e == ops.TcGemv.RES:
                        op = lambda i, p=p, o=outb: p(xp, wpk[i], o, res=o, err=err, pdl=False)  # noqa: E731
                    elif e == ops.TcGemv.SWIGLU:
                        op = lambda i, p=p, o=outb: p(xp, wpk[i], o[:, : n // 2], err=err, pdl=False)  # noqa: E731
                    else:
                        op = lambda i, p=p, o=outb: p(xp, wpk[i], o, err=err, pdl=False)  # noqa: E731
                cases.append(("tc_kernel", epi, op, 1))
                cases.append(("tc", epi, lambda i, op=op, norm=norm, x=x: (xp.pack(x, norm, 1e-6, False), op(i)), 2))
            # ---- cuBLAS
            outc = torch.empty((M, n), dtype=torch.bfloat16, device=dev)
            cases.append(("cublas", "store", lambda i, x=x, o=outc: torch.matmul(x, wrm[i].t(), out=o), 1))
            for path, epi, fn, nl in cases:
                ms = _time_cycle(fn, copies, launches)
                nbytes = base + (2 * M * n if epi == "fused" and name in ("o", "down") else 0)
                if epi == "fused" and name == "gu":
                    nbytes = 2 * n * k + 2 * M * k + M * n  # output is M x n/2
                if epi == "fused" and name == "lm":
                    nbytes = 2 * n * k + 2 * M * k + 8 * M  # argmax only, no logits written
                flops = 2 * M * n * k
                gbs = nbytes / (ms / 1e3) / 1e9
                print(json.dumps({"sweep": "linear", "shape": name, "n": n, "k": k, "M": M, "path": path,
                                  "epilogue": epi, "launches": nl, "us": round(ms * 1e3, 2), "GBs": round(gbs, 1),
                                  "frac_hbm": round(gbs / peak, 4), "TFLOPs": round(flops / (ms / 1e3) / 1e12, 2),
                                  "frac_tensor": round(flops / (ms / 1e3) / 1e12 / tpeak, 4),
                                  "peak_hbm": peak, "peak_kind": kind}), flush=True)
            assert int(err.item()) == 0
        del wrm, wpk
        torch.cuda.empty_cache()


def run_sweep_attn(a):
    """GQA decode attention (32 q / 8 KV heads, D 128) at B in {1, 8, 32} and cache
    length L in {1024, 8192, 32768}, Q/K/V N(0, 1) seed 2: ours_tc (qd_attn_decode_tc, tcgen05),
    ours_stream (qd_attn_decode_stream, CUDA cores), ours_team (qd_attn_decode, the per-unit kernel whose arithmetic
    the persistent step kernel shares) and torch SDPA with enable_gqa (the library baseline).
    Bytes = 4096 B L (K + V) + 2 x 8192 B (q, out)."""
    import torch
    import torch.nn.functional as F

    from decode_b200 import ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    peak, kind = _peaks()
    nq, nkv, D = 32, 8, 128
    g = torch.Generator(device=dev).manual_seed(2)
    err = torch.zeros((1,), dtype=torch.int32, device=dev)
    launches = max(a.launches, 24)
    for B in (1, 8, 32):
        for L in (1024, 8192, 32768):
            per = 2 * B * nkv * L * D * 2
            copies = max(2, -(-(300 << 20) // per))
            kc = [torch.randn((B, nkv, L, D), generator=g, device=dev).to(torch.bfloat16) for _ in range(copies)]
            vc = [torch.randn((B, nkv, L, D), generator=g, device=dev).to(torch.bfloat16) for _ in range(copies)]
            q = torch.randn((B, nq, D), generator=g, device=dev).to(torch.bfloat16)
            out = torch.empty((B, nq, D), dtype=torch.bfloat16, device=dev)
            attn = ops.DecodeAttention(B, nq, nkv, L, dev)
            stream = ops.DecodeAttentionStream(B, nq, nkv, L, dev)
            tca = ops.DecodeAttentionTc(B, nq, nkv, L, dev)
            pos = torch.tensor([L - 1], dtype=torch.int64, device=dev)
            q4 = q.view(B, nq, 1, D)
            nbytes = 4096 * B * L + 2 * 8192 * B
            for path, fn in (("ours_tc", lambda i: tca(q, kc[i], vc[i], pos, out, err=err, pdl=False)),
                             ("ours_stream", lambda i: stream(q, kc[i], vc[i], pos, out, err=err, pdl=False)),
                             ("ours_team", lambda i: attn(q, kc[i], vc[i], pos, out, err=err, pdl=False)),
                             ("torch_sdpa", lambda i: F.scaled_dot_product_attention(
                                 q4, kc[i], vc[i], scale=D ** -0.5, enable_gqa=True))):
                ms = _time_cycle(fn, copies, launches)
                gbs = nbytes / (ms / 1e3) / 1e9
                print(json.dumps({"sweep": "attn", "B": B, "L": L, "path": path,
                                  "us": round(ms * 1e3, 2), "GBs": round(gbs, 1), "frac_hbm": round(gbs / peak, 4),
                                  "peak_hbm": peak, "peak_kind": kind}), flush=True)
            assert int(err.item()) == 0
            del kc, vc
            torch.cuda.empty_cache()


def run_sweep_prefill(a):
    """Prompt projections (prefill, engine/engine.py:550-592) at M tokens in {128, 1024, 16384} (the
    prompt of config 1, one config-4 sequence, a full 16384-token prefill chunk): qd_tc_gemm over the
    packed weights (plain store and fused epilogue) against cuBLAS (torch.matmul on row-major
    weights, store only), each timed as a CUDA graph replay over weight copies that exceed the L2.
    Flops = 2MNK, against the measured dense BF16 peak. Then the engine's whole
    prompt forward for configs 1 and 4 (one GPU's shard: 8 x 1024), timed by CUDA events around the
    prefill graph."""
    import torch

    from decode_b200 import ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    tpeak = _tensor_peak()
    H, I, nq, nkv, D = 2560, 9728, 32, 8, 128
    shapes = [("qkv", (nq + 2 * nkv) * D, H), ("o", H, nq * D), ("gu", 2 * I, H), ("down", H, I)]
    g = torch.Generator(device=dev).manual_seed(1)
    err = torch.zeros((1,), dtype=torch.int32, device=dev)
    launches = max(a.launches, 12)
    for name, n, k in shapes:
        # enough weight copies to exceed twice the L2, so every launch streams its weights from HBM as the
        # prompt forward's layers do
        copies = max(1, -(-2 * 126 * 2 ** 20 // (2 * n * k)))
        ws = [(torch.randn((n, k), generator=g, device=dev) * 0.02).to(torch.bfloat16) for _ in range(copies)]
        wps = [ops.pack_matrix(w) for w in ws]
        for M in (128, 1024, 16384):
            x = torch.randn((M, k), generator=g, device=dev).to(torch.bfloat16)
            out = torch.empty((M, n), dtype=torch.bfloat16, device=dev)
            epi = {"o": ops.Gemv.RES, "down": ops.Gemv.RES, "gu": ops.Gemv.SWIGLU}.get(name, ops.Gemv.STORE)
            grid, bn, ks, nb = ops.tc_gemm_plan(M, n, k)
            sc = torch.zeros((max(nb, 1),), dtype=torch.uint8, device=dev)
            cases = [("tc_gemm", "store", lambda i: ops.tc_gemm(x, wps[i], n, out, err=err, scratch=sc))]
            if epi == ops.Gemv.RES:
                cases.append(("tc_gemm", "fused", lambda i: ops.tc_gemm(x, wps[i], n, out, res=out, epilogue=epi,
                                                                       err=err, scratch=sc)))
            elif epi == ops.Gemv.SWIGLU:
                cases.append(("tc_gemm", "fused", lambda i: ops.tc_gemm(x, wps[i], n, out[:, : n // 2], epilogue=epi,
                                                                       err=err, scratch=sc)))
            cases.append(("cublas", "store", lambda i: torch.matmul(x, ws[i].t(), out=out)))
            for path, ep, fn in cases:
                ms = _time_graph(fn, copies, max(launches, copies))
                tf = 2 * M * n * k / (ms / 1e3) / 1e12
                print(json.dumps({"sweep": "prefill", "shape": name, "n": n, "k": k, "M": M, "path": path,
                                  "epilogue": ep, "tile_n": bn if path == "tc_gemm" else None,
                                  "ksplit": ks if path == "tc_gemm" else None,
                                  "grid": grid if path == "tc_gemm" else None, "us": round(ms * 1e3, 2),
                                  "TFLOPs": round(tf, 1), "frac_tensor": round(tf / tpeak, 4),
                                  "peak_tflops": tpeak}), flush=True)
            assert int(err.item()) == 0
            del x, out
        del ws, wps
        torch.cuda.empty_cache()
    # causal prompt attention: qd_prefill_attn against PyTorch's flash SDPA (the reference's call)
    nq, nkv, D = 32, 8, 128
    for b, S in ((1, 128), (8, 1024), (16, 1024), (1, 8192)):
        q = torch.randn((b * S, nq * D), generator=g, device=dev).to(torch.bfloat16)
        kc = torch.randn((b, nkv, S, D), generator=g, device=dev).to(torch.bfloat16)
        vc = torch.randn((b, nkv, S, D), generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty((b * S, nq * D), dtype=torch.bfloat16, device=dev)
        q4 = q.view(b, S, nq, D).transpose(1, 2)
        flops = 4 * b * nq * (S * (S + 1) // 2) * D
        for path, fn in (("qd_prefill_attn", lambda i: ops.prefill_attn(q, b, S, nq, nkv, kc, vc, out, err=err)),
                         ("torch_flash_sdpa", lambda i: torch.nn.functional.scaled_dot_product_attention(
                             q4, kc, vc, is_causal=True, scale=D ** -0.5, enable_gqa=True))):
            ms = _time_graph(fn, 1, launches)
            tf = flops / (ms / 1e3) / 1e12
            print(json.dumps({"sweep": "prefill_attn", "batch": b, "prompt": S, "path": path, "us": round(ms * 1e3, 2),
                              "TFLOPs": round(tf, 1), "frac_tensor": round(tf / tpeak, 4)}), flush=True)
        assert int(err.item()) == 0
        del q, kc, vc, out
    # whole prompt forward through the engine (random-init weights)
    import engine as E

    state, cfg = make_model(a.layers)
    eng = E.Engine.from_state_dict(state, cfg, "cuda:0")
    del state
    for B, S in ((1, 128), (8, 1024)):
        st = eng._build(B, S, 2)
        with torch.inference_mode():
            st.ids.copy_(torch.tensor(synth_prompt(B, S), dtype=torch.int64))
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.prefill_graph.replay()
        torch.cuda.synchronize()
        s.record()
        for _ in range(3):
            st.prefill_graph.replay()
        e.record()
        e.synchronize()
        ms = s.elapsed_time(e) / 3
        # the last layer continues only the last position (o, gate/up, down, LM head on B rows)
        rest = 4096 * 2560 + 2560 * 19456 + 9728 * 2560
        flops = 2 * B * S * (a.layers * 2560 * 6144 + (a.layers - 1) * rest) + 2 * B * (rest + 151936 * 2560)
        eng.check_device_errors(st)
        print(json.dumps({"sweep": "prefill_forward", "layers": a.layers, "batch": B, "prompt": S, "ms": round(ms, 3),
                          "tokens_per_s": round(B * S / (ms / 1e3), 1),
                          "projection_TFLOPs": round(flops / (ms / 1e3) / 1e12, 1)}), flush=True)


def _tensor_peak():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


def synth_prompt(B, S):
    from decode_b200 import synth

    return synth.random_prompt(B, S, 151936, seed=0)


def main():
    a = _args()
    if a.sweep == "linear":
        run_sweep_linear(a)
    elif a.sweep == "attn":
        run_sweep_attn(a)
    elif a.sweep == "prefill":
        run_sweep_prefill(a)
    elif a.kernel:
        run_kernel(a)
    elif a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
