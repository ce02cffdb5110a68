"""CPU oracle for the W4A16 MoE layer and its expert-prefetch path.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this
directory: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may use it, and only as the checker (or, for
``bench.py --impl reference``, as the timed reference CPU path).

Each module restates one piece of the reference algorithm on the CPU, citing
the reference file:line it follows (paths are relative to the reference
project root, HUSRCF/MTP "mtp-expert-prefetch"; vLLM paths are relative to the
installed vLLM 0.22.0 package):

* ``gptq``      - int4 pack / unpack / dequantise (numpy, integer + fp32).
* ``router``    - softmax / top-k / renormalise (numpy fp32).
* ``align``     - moe_align_block_size in canonical order (numpy, integer).
* ``layer``     - the routed SiLU-MLP sum + sigmoid-gated shared expert
                  (torch fp32 on the CPU), the reference ``moe_tokens`` form.
* ``cache``     - LRU and ready-time expert-cache managers (pure Python).
* ``predictor`` - MTP expert-demand predictor MLP + per-layer top-k (torch fp32).

Parity pins: ``tests/golden/`` holds fixtures produced by running the
reference's own Python code (``tests/golden/make_golden.py``); the oracle is
checked against them in ``tests/test_oracle_golden.py``. The vLLM compiled ops
(``topk_softmax``, ``moe_align_block_size``) cannot run on a CPU; the router
and align restatements are pinned by the reference's CPU torch fallback
(vllm_router_trace.py:4201-4227) and by the worked example in the vLLM
wrapper's docstring respectively.
"""
