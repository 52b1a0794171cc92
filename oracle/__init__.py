"""CPU oracle of the quantised-linear hot path.

TEST INFRASTRUCTURE ONLY. The product (``cuda_force_b200``) never imports,
links or executes anything in this directory. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs
use it, and only as the checker or the timed CPU baseline.

* ``quant_ref``  — numpy restatement of the reference's block-INT8 quantise /
  dequantise (python/cudaforge/ops.py:215-240, cpp/src/bindings.cpp:298-329).
* ``quant_ref.c`` — the same restatement in plain C (built by ``Makefile`` into
  ``_build/``), a second independent checker used on large inputs.
* ``linear_ref`` — fp32/fp64 restatement of the LoRA linear
  (python/cudaforge/ops.py:178-185, cpp/src/bindings.cpp:255-258).
* ``norm_ref``   — torch restatement of RMSNorm and residual add + RMSNorm
  (python/cudaforge/ops.py:164-171, 188-192, cpp/src/bindings.cpp:238-271).
* ``build_ref``  — compiles the reference's own CPU operators
  (cpp/src/bindings.cpp) into ``_ref/`` as ``torch.ops.cudaforge_ref.*``.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference's Python
implementation (imported from the reference tree in the build container) and
its compiled CPU operators on seeded inputs and commits the results under
``tests/golden/``; ``tests/test_oracle.py`` checks both restatements against
those fixtures bit for bit.
"""
