"""torobi_b200: a B200-native (sm_100a) backend for Torobi's quantized-weight
QLoRA path -- MLX-style affine quantize/dequantize, quantized_matmul with the
LoRA up-projection added in its tensor-memory accumulator (the down-projection
is a separate skinny pass per shared input), and the data-parallel LoRA step --
behind the C ABI of include/torobi_b200.h.
"""
from ._lib import LIB_PATH, TqError, device_status, header_symbols, lib
from .ops import (adamw_, dequantize, dequantize_batch, lora_down, lora_grad, qlora_matmul,
                  quantize, quantize_batch, quantized_matmul, sumsq, transpose_to_bf16)

__all__ = [
    "LIB_PATH", "TqError", "device_status", "header_symbols", "lib", "adamw_", "dequantize",
    "dequantize_batch", "lora_down", "lora_grad", "qlora_matmul", "quantize", "quantize_batch",
    "quantized_matmul", "sumsq", "transpose_to_bf16",
]
