"""CPU oracle of CIGN's sparse message-passing hot path -- TEST INFRASTRUCTURE.

This package restates, on the CPU, the algorithms of the reference
implementation (rabbit-art/CIGN) for every op of the hot path, each function
citing the reference file:line it follows.  It is the checker, never the
thing measured or shipped: only ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import
it.  The product package ``cign_b200`` never imports it and has no CPU path.

Pinning (how the oracle itself is checked):
  * CSR / CSR^T / normalised-operator construction, SpMM and the k-hop
    recurrence, the pack family and the block ops are compared against
    golden fixtures produced by running the reference's own Python code on
    the CPU (tests/golden/make_golden.py, fixtures in tests/golden/);
  * splitmix64 is checked against the published SplitMix64 outputs;
  * the collapsed GAT has no CPU-runnable reference (CUDA-only kernel,
    PyG/dgNN absent): its restatement is cross-checked against an
    independent formulation of GATConv(concat=False) + bias + SiLU.
"""
