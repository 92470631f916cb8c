"""CPU oracle for the Qwen3 greedy decode path.

TEST INFRASTRUCTURE ONLY. Nothing in the product (`htn-2026_b200/`) imports this package; only
`tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm use it, and
only as the checker or as the timed CPU baseline, never as the thing measured on the GPU.

  qwen3_cpu  torch-CPU restatement of the reference's eager decode path (engine/engine.py tier 1,
             :501-514, :550-643) op by op, with every BF16 rounding point of transformers'
             modeling_qwen3; also the per-op checkers for the CUDA kernels.
  native     the reference's tier 0: the plain Transformers greedy loop with a KV cache
             (engine/engine.py:963-972) and its teacher-forced margin (:974-996).

Pinned against tests/golden/*.json, which tests/golden/make_golden.py produced by running the
reference engine itself (tiers 0 and 1) on CPU.
"""
