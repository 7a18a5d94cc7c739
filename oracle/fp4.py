"""FP4 (E2M1) / W4A16 emulation for the oracle (TEST INFRASTRUCTURE ONLY).

The reference's policy names fp4 as W4A16 — FP4 constant weights, 16-bit
activations (c32/strategy.py:98-119 and 150-154) — but has no fp4 kernel, so,
as for fp8, this module pins the *format*: OCP E2M1 (1 sign bit, 2 exponent
bits with bias 1, 1 mantissa bit; magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6),
round to nearest with ties to the even code, saturating to +-6.  The tests
check it against those code points, against the package's host encoder and
against the CUDA quantiser byte for byte.

Scheme of the W4A16 path: groups of 16 consecutive K elements of a weight row
share ``scale = max|group| / 6`` (fp32; 1 for an all-zero group); codes are
E2M1(w / scale), element 2i in the low nibble of byte i; scales are stored
[K/64][N][4].  The GEMM uses ``W_eff = bf16(E2M1 value * scale)`` (the fp32
product is exact, then rounded to bf16) against bf16 activations.
"""

from __future__ import annotations

import numpy as np

from .bf16 import round_bf16

GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def e2m1_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> 4-bit codes (uint8, 0..15), nearest with ties to the even code."""
    x = np.asarray(x, np.float32)
    a = np.abs(x).astype(np.float64)
    a = np.where(np.isnan(a), 6.0, np.minimum(a, 6.0))
    hi = np.clip(np.searchsorted(GRID, a, side="left"), 0, 7)
    lo = np.clip(hi - 1, 0, 7)
    dlo, dhi = a - GRID[lo], GRID[hi] - a
    code = np.where(dlo < dhi, lo, np.where(dhi < dlo, hi, np.where(lo % 2 == 0, lo, hi)))
    code = np.where(a == GRID[hi], hi, code)
    sign = np.where(np.signbit(x) & ~np.isnan(x), 8, 0)
    return (code | sign).astype(np.uint8)


def e2m1_decode(c: np.ndarray) -> np.ndarray:
    c = np.asarray(c, np.uint8)
    v = GRID[c & 7]
    return np.where(c & 8, -v, v)


def quant_groups(w: np.ndarray):
    """[N, K] -> (packed uint8 [N, K/2], scales float32 [K/64, N, 4])."""
    w = np.asarray(w, np.float32)
    N, K = w.shape
    g = w.reshape(N, K // 16, 16)
    amax = np.max(np.abs(g), axis=2)
    s = np.where(amax > 0, (amax / np.float32(6.0)).astype(np.float32), np.float32(1.0)).astype(np.float32)
    codes = e2m1_encode((g / s[:, :, None]).astype(np.float32)).reshape(N, K)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    scales = s.reshape(N, K // 64, 4).transpose(1, 0, 2).copy()
    return packed, scales


def dequant(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """W_eff [N, K] float32 = bf16(E2M1 value * group scale)."""
    N, K2 = packed.shape
    K = 2 * K2
    codes = np.empty((N, K), np.uint8)
    codes[:, 0::2] = packed & 0xF
    codes[:, 1::2] = packed >> 4
    s = scales.transpose(1, 0, 2).reshape(N, K // 16)
    w = (e2m1_decode(codes).reshape(N, K // 16, 16) * s[:, :, None]).astype(np.float32).reshape(N, K)
    return round_bf16(w)


def gemm_w4a16(a_bf16: np.ndarray, packed, scales, bias=None) -> np.ndarray:
    y = np.asarray(a_bf16, np.float64) @ dequant(packed, scales).astype(np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :]
    return y
