"""FlashNS on B200 (sm_100a): fused FP64 jet-PINN loss + parameter-gradient evaluation.

Host API mirrors the reference ``flashns`` package (``jet_spec``, ``jet_packed``,
``ns_seed``, ``pinn_packed``, ``distributed_contract``); the compute runs in the
hand-written CUDA kernels of ``libflashns_b200.so`` through its C ABI
(``include/flashns_b200.h``).
"""

__all__ = ["build", "evaluator", "jet_spec", "ns_seed", "distributed_contract", "problems"]
