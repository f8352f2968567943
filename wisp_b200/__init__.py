"""wisp_b200 -- B200-native (sm_100a) routed-expert int4 FFN hot path of the
WISP MoE inference engine.

The product is the C ABI in include/wisp_b200.h, implemented by
libwisp_b200.so (CUDA kernels in wisp_b200/csrc). This package holds the
in-tree build (``python -m wisp_b200.build``), a ctypes view of the ABI
(``abi``), the MoE layer wrapper (``moe``), the expert-parallel driver
(``ep``), seeded synthetic weights (``synth``) and the expert blob format
(``blob``).
"""
__all__ = ["abi", "blob", "synth", "moe", "ep", "build"]
