"""E4M3 (fp8) emulation for the oracle (TEST INFRASTRUCTURE ONLY).

The reference's precision policy names fp8 for aligned GEMMs and 1x1 convs
(c32/strategy.py:124-160) and its decompositions emit ``matmul_f8``
(c32/decompositions.py:18-27), but the reference has no fp8 kernel: its
``lookup`` (c32/kernel_registry.py:42-66) raises for that name.  So there is no
reference behaviour to pin against; this module pins the *format* instead: the
OCP 8-bit floating point E4M3 encoding (1 sign bit, 4 exponent bits with bias 7,
3 mantissa bits, subnormals below 2^-6, largest finite 448, no infinities),
round to nearest even, saturating to +-448.  ``tests/test_oracle.py`` checks it
against the code points of that specification and against torch's
``float8_e4m3fn`` conversion; ``tests/test_gpu_kernels.py`` checks the CUDA
quantiser against it byte for byte.

The quantisation scheme of the fp8 path (rowwise, per-tensor-row scales):
``scale[m] = max|x[m,:]| / 448`` in fp32 (1 for an all-zero row) and
``q[m,k] = e4m3(x[m,k] / scale[m])`` with an fp32 division.
"""

from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> E4M3 bytes, round to nearest even, saturating (NaN -> 0x7F)."""
    x = np.asarray(x, np.float32)
    a = np.abs(x).astype(np.float64)
    nan = np.isnan(a)
    a = np.where(nan, 0.0, np.minimum(a, E4M3_MAX))
    # exponent of the grid: floor(log2 a) for normals, -6 for subnormals
    _, ex = np.frexp(a)
    e = np.maximum(ex.astype(np.int64) - 1, -6)
    step = np.ldexp(1.0, e - 3)
    m = np.minimum(np.rint(a / step) * step, E4M3_MAX)  # rint: ties to even
    # re-derive the fields from the rounded value (rounding may enter the next binade)
    _, ex2 = np.frexp(m)
    e2 = np.maximum(ex2.astype(np.int64) - 1, -6)
    sub = m < 2.0 ** -6
    mant = np.where(sub, m / 2.0 ** -9, m / np.ldexp(1.0, e2 - 3) - 8.0)
    expf = np.where(sub, 0, e2 + 7)
    bits = (expf.astype(np.int64) << 3) | np.rint(mant).astype(np.int64)
    bits = np.where(m == 0.0, 0, bits)
    sign = np.signbit(x).astype(np.int64) << 7
    out = (bits | sign).astype(np.uint8)
    return np.where(nan, np.uint8(0x7F), out).astype(np.uint8)


def _decode_table() -> np.ndarray:
    t = np.zeros(256, np.float64)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        mnt = b & 7
        if e == 0xF and mnt == 7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * mnt * 2.0 ** -9
        else:
            t[b] = s * (1.0 + mnt / 8.0) * 2.0 ** (e - 7)
    return t


_TABLE = _decode_table()


def e4m3_decode(q: np.ndarray) -> np.ndarray:
    """E4M3 bytes -> float64 values."""
    return _TABLE[np.asarray(q, np.uint8)]


def quant_rows(x: np.ndarray):
    """Rowwise quantisation of a 2-D array: (q uint8 [M,K], scale float32 [M])."""
    x = np.asarray(x, np.float32)
    amax = np.max(np.abs(x), axis=1) if x.shape[1] else np.zeros(x.shape[0], np.float32)
    scale = np.where(amax > 0, (amax / np.float32(448.0)).astype(np.float32), np.float32(1.0)).astype(np.float32)
    q = e4m3_encode((x / scale[:, None]).astype(np.float32))
    return q, scale


def gemm_fp8(qa, sa, qb, sb, bias=None, act: int = 0) -> np.ndarray:
    """(decode(qa) . decode(qb)^T) * sa[m] * sb[n] (+ bias), act 1 = ReLU, 2 = GELU (erf)."""
    y = e4m3_decode(qa) @ e4m3_decode(qb).T
    y = y * np.asarray(sa, np.float64)[:, None] * np.asarray(sb, np.float64)[None, :]
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :]
    if act == 1:
        y = np.maximum(y, 0.0)
    elif act == 2:
        from math import erf
        y = 0.5 * y * (1.0 + np.vectorize(erf)(y / np.sqrt(2.0)))
    return y
