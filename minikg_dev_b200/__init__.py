"""minikg_dev_b200 — MiniKG's relation-typed sparse message passing on B200 (sm_100a).

Public surface:
* ``fastlog_bridge``: the reference operator API (FastLogFunctionSparse3DTopK,
  build_csr_structure, sum_sp_3d, sum_sparse3d_concat) and ``kernel_ops()``;
* ``proof``: the fused multi-hop engine (``kernel_sparse_scores``, ``proof_scores``,
  ``decode_max``, ``decode_topk``);
* ``rules``: the rule-weight producer (``build_rule_logits``, ``rule_weights``: the per-rule
  bidirectional LSTMs, linear layer and per-hop softmax on the device);
* ``graph``: device CSR build and ``DeviceGraph``;
* ``synth``: seeded synthetic knowledge graphs of the benchmark shapes.
The CUDA code lives in ``csrc/`` and is built into ``_lib/libminikg_b200.so`` by
``python -m minikg_dev_b200.build``.
"""
__version__ = "0.1.0"
