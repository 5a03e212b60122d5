"""GEMM-side API mirroring the reference's ``cutlass_gemm`` package:
``quantization.quantize/dequantize`` and ``backend.gemm`` with the same
arguments, layouts and error behaviour, on the sm_100a kernels."""
