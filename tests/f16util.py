"""f16 bit patterns for the kernel-level tests (the step's 16-bit operands are IEEE half)."""
import numpy as np


def f16_bits(x):
    """Round to nearest-even f16; return the uint16 bit patterns."""
    return np.ascontiguousarray(np.asarray(x, np.float32).astype(np.float16)).view(np.uint16)


def bits_to_f32(b):
    """uint16 f16 bit patterns -> float32 values (exact)."""
    return np.ascontiguousarray(b).view(np.float16).astype(np.float32)
