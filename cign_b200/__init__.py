"""cign_b200 -- B200-native (sm_100a) kernels for CIGN's sparse message-passing
hot path behind the reference's Python module API.

Modules named after the reference's (drop-in replacements):
    multihop_csr_pipeline, collapsed_gat, fused_gat_sideops,
    fused_clifford_pack, fused_clifford_switch_pack, fused_clifford_cign_pack,
    fused_clifford_cign_generic, fused_block_ops
plus graph_operator (FixedCSR operator / selected_sparse_powers), model_cign
(the CIGN caller used by the benchmark) and synth (seeded workloads).

All compute goes through libcign_sm100.so (C ABI in include/cign_sm100.h);
there is no CPU fallback.  Importing the package does not load the library.
"""
__version__ = "0.1.0"
