"""fp8 raw weights restated in numpy — TEST INFRASTRUCTURE ONLY (the CPU checker for the CUDA fp8 path).

selas keeps fp8 sources as stored (``encode_raw``, ``selas/convert.py:178-180``) and casts them to the
compute dtype at use (``decode`` for ``raw``, ``selas/codecs.py:270-271``: ``x.to(dtype)``). The cast is
exact for both formats, so the decoded value is the format's value:

* e4m3fn: sign, 4-bit exponent (bias 7), 3-bit mantissa; exponent 0 is subnormal (m * 2^-9); the all-ones
  exponent is a normal binade except the mantissa 7, which is NaN (no infinities);
* e5m2: sign, 5-bit exponent (bias 15), 2-bit mantissa; exponent 0 is subnormal (m * 2^-16); the all-ones
  exponent holds inf (mantissa 0) and NaN.

Pinned by ``tests/test_oracle_golden.py`` against torch's own cast, the operation selas performs.
"""

from __future__ import annotations

import numpy as np


def decode(codes: np.ndarray, e5m2: bool) -> np.ndarray:
    """fp32 values of fp8 byte codes."""
    c = np.asarray(codes, dtype=np.uint8).astype(np.int64)
    sign = np.where(c & 0x80, -1.0, 1.0)
    if e5m2:
        e, m, bias, mbits = (c >> 2) & 0x1F, c & 0x3, 15, 2
        special = e == 0x1F
        out = np.where(e == 0, m * 2.0 ** (1 - bias - mbits), (1 + m / 2.0 ** mbits) * 2.0 ** (e - bias))
        out = np.where(special, np.where(m == 0, np.inf, np.nan), out)
    else:
        e, m, bias, mbits = (c >> 3) & 0xF, c & 0x7, 7, 3
        out = np.where(e == 0, m * 2.0 ** (1 - bias - mbits), (1 + m / 2.0 ** mbits) * 2.0 ** (e - bias))
        out = np.where((e == 0xF) & (m == 0x7), np.nan, out)
    return (sign * out).astype(np.float32)
