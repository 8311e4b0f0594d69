"""anedvd_b200: a B200-native CUDA backend for ANEDVD's quantized-weight hot path.

The product is the C-ABI library ``libcuq.so`` (``include/cuq.h``) built from
``anedvd_b200/csrc``; this package holds its ctypes binding (``runtime``), the
host-side mirror of the reference engine's interface (``engine``), the GGUF
container code (``gguf``) and the seeded synthetic-model generator (``synth``,
``quant``).
"""
