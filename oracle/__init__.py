"""CPU oracle for the MJOLNIR decode-attention hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference algorithms that the CUDA
product path must reproduce:

* ``oracle.quant``     -- the e2m3 (6-bit, 4 codes per 3 bytes) and fp8-e4m3
                          quantize-on-write, bit for bit (numpy, integer/fp32);
* ``oracle.attention`` -- the dequantise-then-attend fp32 attention over a paged
                          KV cache (torch fp32 on the CPU), the split-KV planner
                          restated for comparison, and the LSE split merge.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import it, and only as the checker (or as the timed CPU baseline). The
product package ``mjolnir_b200`` never imports it and has no CPU fallback.

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference's own
Python implementation (GoBrrr-ai/mjolnir ``src/mjolnir/mjolnir/quant.py``,
``kvfp6.py``, ``arch/thor/harness.py``, ``arch/orin/harness.py``,
``arch/thor/plan.py``) on seeded inputs and committed the outputs as fixtures
under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this oracle
against them.
"""
