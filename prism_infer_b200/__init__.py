"""B200-native (sm_100a) Qwen3-MoE sparse block, a drop-in for prism-infer's ``MoE`` layer.

Public surface (mirrors the reference's module layout):

* ``prism_infer_b200.layers.moe.MoE`` — the block (router -> route/top-k -> dispatch ->
  grouped SwiGLU experts -> weighted combine), same constructor and ``forward(hidden_states)``
  as ``prism_infer/layers/moe.py:31-100``;
* ``prism_infer_b200.engine.parallel.expert_parallel`` — expert-parallel helpers with the
  reference's names (``set_expert_parallel_size``, ``build_dispatch_plan``, ...);
* ``prism_infer_b200.capi`` — the ctypes binding of the C-ABI library ``libprism_moe.so``
  (declared in ``include/prism_moe.h``).

Importing the package does not load CUDA code; the library loads on first use and raises if
it is missing.
"""
__version__ = "0.1.0"
