"""CPU oracle for the `cuda` target of ml-graph-compiler.

TEST INFRASTRUCTURE ONLY. Nothing in the product (``ml-graph-compiler_b200/mgc_cuda``, the CUDA
kernels, the C ABI) imports, links or executes anything in this directory. Only ``tests/``,
``__graft_entry__.smoke()`` (as the checker) and ``bench.py`` (the ``cpu_baseline`` leg and the
``--impl reference`` arm) use it.

Contents:

* ``semantics.py`` / ``runner.py``: a numpy restatement of the reference's operator semantics
  (``src/ml_graph_compiler/ops.py``) for every operator the cuda target lowers, and a graph
  runner over the scheduled node list. Floating point work is done in float64 and rounded to the
  tensor's dtype, so the oracle is at least as exact as the reference interpreter it restates.
* ``Makefile``: compiles the reference's own C runtime kernels
  (``codegen/runtime/mgc_kernels.c``) from the sources where they lie into ``oracle/_ref/``, a
  second, independent arithmetic reference for the GEMM epilogue, softmax, layer norm, pooling
  and depthwise kernels.

Pinning: ``tests/golden/make_golden.py`` runs the reference's interpreter
(``interpreter.run_graph``) and C backend on seeded graphs and stores their outputs as fixtures;
``tests/test_oracle.py`` checks this oracle against every fixture.
"""
