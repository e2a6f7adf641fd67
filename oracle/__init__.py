"""CPU oracle for the mini_vllm decode path -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

This package restates, in plain PyTorch on the CPU, the reference's own
algorithm for the decode step (``mini_vllm/models/model.py``, the pure-PyTorch
model that ``MINI_VLLM_BACKEND=pytorch`` selects, ``mini_vllm/ops/_utils.py:74``),
its paged KV-cache manager (``mini_vllm/engine/kv_cache.py``), its engine step
(``mini_vllm/engine/engine.py:241-360``) and its sampling semantics
(``mini_vllm/ops/sampling.py``, ``mini_vllm/engine/sampler.py``).

Pinning: the restatement is checked against fixtures that the reference itself
produced on this code's behalf (``tests/golden/make_golden.py`` runs the
unmodified reference and writes ``tests/golden/*.pt|json``); see
``tests/test_oracle_golden.py``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package, and only as the checker / the timed CPU baseline.  The
CUDA product path (``llm_pytorch_inference_b200``) never imports it.
"""
