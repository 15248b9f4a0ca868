"""CPU oracle for the Flash-Cache / Flash-Verify hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in plain torch fp32 on the CPU, what the reference
VILA-Lab/Flash-dLLM computes on its hot path:

* ``flash_cache_oracle`` -- the five Triton kernels of
  ``llada/flash_cache_triton.py`` (QKV+RoPE+cache scatter, masked attention
  with raw-score tracking, tracked attention, verify QKV, verify attention)
  and the per-layer driver ``flash_fused_elastic_cache``;
* ``decode_oracle`` -- the decode bookkeeping of ``llada/generate.py``
  (block tables, confidence/accept, verify mask and query build, verify
  acceptance scan, top-k selective refresh) and the whole
  ``generate_with_Flash_dLLM`` loop;
* ``tiny_model`` -- seeded weights and a CPU LLaDA forward that calls the
  oracle layer, used to drive the decode loop at small sizes.

Parity is pinned against the reference itself: ``tests/golden/make_golden.py``
runs the reference kernels under ``TRITON_INTERPRET=1`` (fp32) and the
reference ``generate_with_Flash_dLLM`` on a tiny random-init model, and the
committed fixtures in ``tests/golden/`` are checked against this package by
``tests/test_oracle_golden.py``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
arm may import this package, and only as the checker / the timed CPU
baseline.  The product (``flash-dllm_b200/``) never imports it.
"""
