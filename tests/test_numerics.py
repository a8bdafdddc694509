"""CPU: exhaustive checks of arithmetic shortcuts the kernels rely on."""
import numpy as np


def _bf(x):
    b = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def test_kivi_scale_reciprocal_multiply_is_exact():
    """bf16(fp32(d / 15)) == bf16(fp32(d * fp32(1/15))) for every finite bf16 d.
    d/15 has a binary expansion repeating a 4-bit pattern, so it never lies
    within the multiply's ~2^-23 relative error of a bf16 rounding midpoint;
    the kernels use the multiply for the KIVI scale (mx - mn) / 15."""
    f = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    f = f[np.isfinite(f)]
    div = _bf((f / np.float32(15)).astype(np.float32))
    mul = _bf((f * np.float32(1.0 / 15.0)).astype(np.float32))
    assert np.array_equal(div, mul)
