"""CPU oracle for the paged/packed attention hot path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, what the reference engine
(pedrosilva-a11y/llm-engineering, ``serving/engine/``) computes on this path, so that the
CUDA kernels can be checked against it. Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm may import it, and only as the checker or the
timed CPU baseline: the product path (``llm-engineering_b200``) never imports it and has
no CPU fallback.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here against
fixtures produced by running the reference itself (``tests/golden/make_golden.py``).
The attention arithmetic of the reference is third-party (HF transformers
``sdpa_attention_forward`` / ``eager_attention_forward`` over torch SDPA; the reference
pins torch 2.14.0 and transformers 5.17.0 in ``uv.lock``); it is restated here as fp32
``softmax(q k^T * scale + mask) v`` with grouped-query heads, and pinned against the
reference's own packed path run on this machine's transformers.
"""
