"""apsi_b200 -- Apsi's low-bit quantized linear layer, rebuilt for NVIDIA B200 (sm_100a).

Submodules:
  kernels    torch-level wrappers of the C ABI (include/apsi_lowbit.h)
  precision  the public entry points of apsi/precision.py (QTensor, quantize, dequantize, qmatmul, ...)
  lowbit     the public entry points of apsi/lowbit.py (parse, round_weights, matmul, ...)
  hub        a hub_gpu-compatible device ops object (qmatrix / linear / gemv / gemm)
  sharded    column-sharded multi-GPU linear with an NCCL all-gather of the outputs
"""
__version__ = "1.0.0"
