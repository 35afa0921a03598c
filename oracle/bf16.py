"""bfloat16 helpers for the oracle (test infrastructure).

numpy has no bfloat16 type, so bf16 tensors are carried as uint16 bit
patterns.  Conversion float32 -> bf16 is round-to-nearest-even on the raw
bits, which is what torch's ``tensor.to(torch.bfloat16)`` and CUDA's
``__float2bfloat16_rn`` do for finite values.
"""
import numpy as np


def f32_to_bf16_bits(a):
    """Round float32 values to bf16 (RNE) and return the uint16 bit patterns."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    rounding_bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding_bias) >> 16).astype(np.uint16)
    r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def bf16_bits_to_f32(b):
    """Expand uint16 bf16 bit patterns to float32."""
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(a):
    """float32 -> nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(a))
