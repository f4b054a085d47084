"""CPU oracle for the IRON LLM-operator hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, what IRON's own golden models compute for each
operator on the hot path (each function cites the reference file:line it
follows). It is the checker for the CUDA kernels in ``iron_b200``: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl
reference`` legs of ``bench.py`` may import or run it. The ``iron_b200``
package never imports it and has no CPU fallback.

Pinning: ``tests/test_oracle_golden.py`` checks every function here against
fixtures in ``tests/golden/`` that ``tests/golden/make_golden.py`` produced by
running IRON's own Python goldens (``iron/operators/*/reference.py``,
``iron/applications/llama_3.2_1b/llama_cpu.py``) from the reference checkout.
The uint4 Dequant golden calls the absent third-party ``mlir_aie`` function
``expand_ref``; its restatement here is pinned by IRON's own input packer
(``dequant/reference.py:21-94``): packed inputs are exact quantizations, so the
expected output of each element is known exactly.
"""
