"""CPU oracle for the USAF MoE expert hot path.

TEST INFRASTRUCTURE ONLY.  This package restates, on the CPU, the algorithm of
the reference (tsuyu122/usaf) for the MoE expert training step so that the
CUDA path in ``usaf_b200`` can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it, and only as the checker or as the timed CPU
baseline.  The product path (``usaf_b200``) never imports this package and has
no CPU fallback.

Modules
-------
quant      packed int4 (HQQ-style) quantize / dequantize, numpy
           (usaf/quantization.py:21-132)
moe        router, dense-masked experts, batched sparse dispatch, capture
           stores, SparseAdam, selectors, RigL merge (torch on the CPU)
           (usaf/qwen3moe_dml.py, usaf/moe_loader.py, usaf/sparse_optim.py,
           usaf/selector.py, train.py, benchmarks/kaggle_t4_bench.py)
inputs     the seeded synthetic inputs of the benchmark configurations

The oracle is pinned against the reference itself: ``tests/golden/make_golden.py``
imports the reference in the build container, runs it on seeded inputs and
stores its outputs as fixtures; ``tests/test_oracle_golden.py`` checks the
oracle against those fixtures.
"""
