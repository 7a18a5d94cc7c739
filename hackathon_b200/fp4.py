"""Host-side FP4 (E2M1) weight quantisation for the W4A16 precision path.

Same scheme as ``C3B_K_QUANT_FP4``: groups of 16 K elements per weight row,
``scale = max|group| / 6`` (fp32 division; 1 for an all-zero group), codes
E2M1(w / scale) rounded to the nearest magnitude of {0, .5, 1, 1.5, 2, 3, 4, 6}
with ties to the even code, element 2i in the low nibble of byte i, scales
stored [K/64][N][4] for the GEMM's tensor map.
"""

from __future__ import annotations

import numpy as np

_MAG = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
# midpoints between consecutive magnitudes; a tie goes to the even code
_MID = (_MAG[1:] + _MAG[:-1]) / 2


def _codes(v: np.ndarray) -> np.ndarray:
    a = np.minimum(np.abs(v).astype(np.float64), 6.0)
    c = np.searchsorted(_MID, a, side="left").astype(np.int64)   # a <= mid -> lower code
    tie = np.isin(a, _MID)
    up = np.searchsorted(_MID, a, side="right").astype(np.int64)  # a == mid -> upper code
    c = np.where(tie & (up % 2 == 0), up, c)
    return (c | np.where(np.signbit(v), 8, 0)).astype(np.uint8)


def quant_groups_fp4(w: np.ndarray):
    """[N, K] float -> (uint8 [N, K/2] packed codes, float32 [K/64, N, 4] scales)."""
    w = np.ascontiguousarray(w, np.float32)
    N, K = w.shape
    if K % 64:
        raise ValueError("W4A16 needs K % 64 == 0")
    g = w.reshape(N, K // 16, 16)
    amax = np.max(np.abs(g), axis=2)
    s = np.where(amax > 0, amax / np.float32(6.0), np.float32(1.0)).astype(np.float32)
    codes = _codes((g / s[:, :, None]).astype(np.float32)).reshape(N, K)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed, s.reshape(N, K // 64, 4).transpose(1, 0, 2).copy()
