"""bfloat16 helpers for the numpy oracle (test infrastructure only).

bf16 values are carried either as float32 arrays whose values are exactly
representable in bf16, or as uint16 bit patterns (the wire / device format).
Rounding is round-to-nearest-even, the mode torch uses for
``Tensor.to(torch.bfloat16)`` and the mode the reference kernels set
(``set_rounding(rounding_mode::conv_even)``, aie_kernels/aie2p/decode_attn.cc:126).
"""

import numpy as np


def round_bits(x) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round-to-nearest-even; NaN stays NaN."""
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint32)
    nan = np.isnan(f)
    if nan.any():
        r = np.where(nan, ((u >> 16) | 0x40).astype(np.uint32), r)
    return r.astype(np.uint16)


def from_bits(b) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 values."""
    b = np.ascontiguousarray(np.asarray(b, dtype=np.uint16))
    return (b.astype(np.uint32) << 16).view(np.float32)


def rnd(x) -> np.ndarray:
    """Round float values to the nearest bf16 value, returned as float32."""
    return from_bits(round_bits(x))


def rnd64(x) -> np.ndarray:
    """Round a float64 array to float32 first (one rounding), then to bf16.

    Used where the reference computes in float32 and stores bf16."""
    return rnd(np.asarray(x, dtype=np.float64).astype(np.float32))
