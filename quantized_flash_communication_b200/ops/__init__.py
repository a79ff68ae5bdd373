"""Single-GPU operators (quantization, packing, GEMM, normalisation, attention)."""
from .quant import quantize, dequantize, pack_int4, unpack_int4  # noqa: F401
