"""FP8 E4M3FN codec restated in numpy (oracle; test infrastructure only).

Decode follows ``flash_attn_mps/kernels/attention_decode.metal:9-16`` (the same
rule as ``attention.metal:4-10``): exponent field 0 is subnormal with step
2^-9, 0x7F/0xFF are NaN, everything else is (1 + m/8) * 2^(e-7).

Encode follows ``flash_attn_mps/kernels/cache.metal:8-18``: saturating
round-to-nearest-even. NaN keeps its sign with payload 0x7F, |x| >= 448
saturates to 0x7E, values below 2^-6 round on the subnormal grid
(rint(|x| * 512)), the rest round their 3-bit mantissa to even. The reference
test pins this as ``x.clamp(-448, 448).to(torch.float8_e4m3fn)``
(``tests/test_cache.py:52``).
"""

import numpy as np


def e4m3_decode(bits):
    """uint8 array -> float64 array (attention_decode.metal:9-16)."""
    b = np.asarray(bits, dtype=np.uint8).astype(np.int64)
    exponent = (b >> 3) & 15
    mantissa = b & 7
    normal = np.ldexp(1.0 + mantissa * 0.125, (exponent - 7).astype(np.int32))
    value = np.where(exponent == 0, mantissa * 2.0 ** -9, normal)
    value = np.where((exponent == 15) & (mantissa == 7), np.nan, value)
    return np.where(b & 128, -value, value)


def e4m3_encode(values):
    """float32-representable array -> uint8 codes (cache.metal:8-18)."""
    x = np.asarray(values, dtype=np.float32)
    sign = ((x.view(np.uint32) >> 24) & 128).astype(np.int64)
    a = np.abs(x.astype(np.float64))
    code = np.zeros(x.shape, dtype=np.int64)
    nan = np.isnan(a)
    big = ~nan & (a >= 448.0)
    small = ~nan & ~big & (a < 0.015625)
    normal = ~nan & ~big & ~small
    code[nan] = 127
    code[big] = 126
    code[small] = np.rint(a[small] * 512.0).astype(np.int64)
    if normal.any():
        frac, exp2 = np.frexp(a[normal])      # a = frac * 2**exp2, frac in [0.5, 1)
        exponent = exp2.astype(np.int64) - 1  # floor(log2(a)), exact
        mantissa = np.rint(np.ldexp(a[normal], (3 - exponent).astype(np.int32))).astype(np.int64) - 8
        code[normal] = np.minimum(((exponent + 7) << 3) + mantissa, 126)
    return (sign | code).astype(np.uint8)
