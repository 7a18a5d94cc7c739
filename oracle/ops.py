"""CPU oracle: NumPy restatement of the reference C3.5 operator semantics.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import this package, and only as the
checker / the timed CPU baseline.  The product path (``hackathon_b200``) never
imports it and fails loudly when its CUDA library is missing.

Every function restates one operator of the reference's CuPy engine
(``c35/engine.py``) or kernel registry (``c32/kernel_registry.py``) in plain
float32 NumPy, citing the file:line it follows.  Pinning: the golden fixtures
under ``tests/golden/`` were produced by running the reference's own engine
ops (with NumPy standing in for CuPy, the trick of
c32/test_kernel_registry.py:14-25) on the same seeded inputs; the CPU test suite
checks this module against them.
"""

from __future__ import annotations

import math
from typing import Any, Dict, List, Optional, Sequence

import numpy as np

F32 = np.float32

# Abramowitz & Stegun 7.1.26 (published rational approximation), used by the
# reference's unfused Erf (c35/engine.py:201-223, c32/kernel_registry.py:179-192).
_AS_P = 0.3275911
_AS_A = (0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)


def erf_as(x: np.ndarray) -> np.ndarray:
    """c35/engine.py:201-223 — A&S 7.1.26 erf approximation in float32."""
    x = np.asarray(x, dtype=F32)
    sign = np.sign(x)
    ax = np.abs(x)
    t = (1.0 / (1.0 + F32(_AS_P) * ax)).astype(F32)
    poly = np.zeros_like(t)
    tp = t.copy()
    for c in _AS_A:
        poly = poly + F32(c) * tp
        tp = tp * t
    return (sign * (1.0 - poly * np.exp(-ax * ax))).astype(F32)


def erf_exact(x: np.ndarray) -> np.ndarray:
    """Exact erf (the fused EW chain calls CUDA ``erff``, c35/engine.py:965)."""
    from scipy.special import erf as _erf
    return _erf(np.asarray(x, dtype=np.float64)).astype(F32)


# ------------------------------------------------------------------ basic ops

def gemm(a, b, c=None, alpha=1.0, beta=1.0, transA=0, transB=0) -> np.ndarray:
    """c35/engine.py:247-279 (op_gemm): alpha*op(A)op(B) + beta*C."""
    a = np.asarray(a, F32)
    b = np.asarray(b, F32)
    if transA:
        a = a.T
    if transB:
        b = b.T
    r = F32(alpha) * (a @ b)
    if c is not None:
        r = r + F32(beta) * np.asarray(c, F32)
    return r.astype(F32)


def conv2d(x, w, b=None, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1),
           group=1, **_: Any) -> np.ndarray:
    """c35/engine.py:288-440 (op_conv): NCHW conv as im2col x weight contraction."""
    x = np.asarray(x, F32)
    w = np.asarray(w, F32)
    N, C, H, W = x.shape
    O, Cg, kH, kW = w.shape
    sH, sW = int(strides[0]), int(strides[-1])
    dH, dW = int(dilations[0]), int(dilations[-1])
    pT, pL, pB, pR = (int(p) for p in pads)
    Ho = (H + pT + pB - (dH * (kH - 1) + 1)) // sH + 1
    Wo = (W + pL + pR - (dW * (kW - 1) + 1)) // sW + 1
    xp = np.pad(x, ((0, 0), (0, 0), (pT, pB), (pL, pR)))
    outs = []
    og = O // group
    for gi in range(group):
        xs = xp[:, gi * Cg:(gi + 1) * Cg]
        cols = np.empty((N, Ho, Wo, Cg, kH, kW), F32)
        for r in range(kH):
            for s in range(kW):
                cols[..., r, s] = xs[:, :, r * dH: r * dH + sH * (Ho - 1) + 1: sH,
                                     s * dW: s * dW + sW * (Wo - 1) + 1: sW].transpose(0, 2, 3, 1)
        a2 = cols.reshape(N * Ho * Wo, Cg * kH * kW)
        w2 = w[gi * og:(gi + 1) * og].reshape(og, -1).T
        outs.append((a2 @ w2).reshape(N, Ho, Wo, og).transpose(0, 3, 1, 2))
    out = np.concatenate(outs, axis=1) if group > 1 else outs[0]
    if b is not None:
        out = out + np.asarray(b, F32).reshape(1, O, 1, 1)
    return np.ascontiguousarray(out, dtype=F32)


def batchnorm(x, scale, bias, mean, var, epsilon=1e-5) -> np.ndarray:
    """c32/kernel_registry.py:573-584 / c35/engine.py:858-879 (inference BN)."""
    sh = [1, -1] + [1] * (x.ndim - 2)
    r = (x - mean.reshape(sh)) / np.sqrt(var.reshape(sh) + F32(epsilon)) * scale.reshape(sh) + bias.reshape(sh)
    return r.astype(F32)


def fold_conv_bn(w, scale, bias, mean, var, conv_bias=None, epsilon=1e-5):
    """c35/executor.py:400-411: w' = w*g/sqrt(v+eps), b' = (b-mu)*g/sqrt(v+eps)+beta."""
    factor = (scale / np.sqrt(var + F32(epsilon))).astype(F32)
    if conv_bias is None:
        conv_bias = np.zeros_like(mean)
    wf = (w * factor.reshape((-1,) + (1,) * (w.ndim - 1))).astype(F32)
    bf = ((conv_bias - mean) * factor + bias).astype(F32)
    return wf, bf


def global_average_pool(x) -> np.ndarray:
    """c35/engine.py:450-459: mean over spatial axes, keepdims."""
    return x.mean(axis=tuple(range(2, x.ndim)), keepdims=True, dtype=F32).astype(F32)


def gather(data, indices, axis=0) -> np.ndarray:
    """c35/engine.py:462-481 / c32/kernel_registry.py:744-752 (np.take)."""
    return np.take(data, np.asarray(indices, np.int64), axis=int(axis))


def layer_norm(x, scale, bias=None, axis=-1, epsilon=1e-5) -> np.ndarray:
    """c35/engine.py:484-532: two-pass LayerNormalization over axes [axis, rank)."""
    axis = int(axis) % x.ndim
    axes = tuple(range(axis, x.ndim))
    mean = x.mean(axis=axes, keepdims=True, dtype=F32)
    xc = x - mean
    var = (xc * xc).mean(axis=axes, keepdims=True, dtype=F32)
    r = xc * (1.0 / np.sqrt(var + F32(epsilon))).astype(F32) * scale
    if bias is not None:
        r = r + bias
    return r.astype(F32)


def softmax(x, axis=-1) -> np.ndarray:
    """c35/engine.py:634-650: max-subtracted softmax."""
    m = x.max(axis=axis, keepdims=True)
    e = np.exp(x - m)
    return (e / e.sum(axis=axis, keepdims=True)).astype(F32)


def split(x, sizes, axis=0) -> List[np.ndarray]:
    """c35/engine.py:557-601."""
    idx = list(np.cumsum([int(s) for s in sizes])[:-1])
    return [np.ascontiguousarray(p) for p in np.split(x, idx, axis=int(axis))]


def resolve_reshape(in_shape: Sequence[int], target: Sequence[int], allowzero: int = 0):
    """c35/engine.py:72-111 (_resolve_reshape_shape)."""
    out: List[int] = []
    infer = None
    known = 1
    for i, d in enumerate(int(v) for v in target):
        if d == 0 and not allowzero:
            d = int(in_shape[i])
        if d == -1:
            infer = i
            out.append(-1)
        else:
            out.append(d)
            known *= d
    total = int(np.prod(in_shape))
    if infer is not None:
        out[infer] = total // known
    return tuple(out)


# ---------------------------------------------------------- fused kernels

def gemm_epilogue(a, b, bias=None, *, alpha=1.0, beta=1.0, transA=0, transB=0,
                  relu=False, flatten_axis=None, matmul=False) -> np.ndarray:
    """c35/engine.py:722-849: act(alpha*op(A)op(B) + beta*bias) with Flatten absorb."""
    a = np.asarray(a, F32)
    if flatten_axis is not None:
        ax = int(flatten_axis) % (a.ndim + 1)
        a = a.reshape(int(np.prod(a.shape[:ax])), -1)
    lead = ()
    if matmul:
        lead = a.shape[:-1]
        a = a.reshape(-1, a.shape[-1])
        transA = transB = 0
    r = gemm(a, b, None, alpha, 1.0, transA, transB)
    if bias is not None:
        c = np.asarray(bias, F32)
        while c.ndim > 2 and c.shape[0] == 1:
            c = c[0]
        r = r + F32(beta) * c
    if relu:
        r = np.maximum(r, F32(0))
    if matmul:
        r = r.reshape(lead + (r.shape[-1],))
    return r.astype(F32)


def attention_scores(q, kT, divisor, mask) -> np.ndarray:
    """c35/engine.py:1250-1380: softmax(Q @ K^T / divisor + mask) along the last axis."""
    s = (np.matmul(q, kT) / F32(np.asarray(divisor).reshape(()))) + mask
    return softmax(s.astype(F32), -1)


def residual_layer_norm(x, residual, scale, bias=None, axis=-1, epsilon=1e-5):
    """c35/engine.py:1078-1167: LayerNorm(x + residual)."""
    return layer_norm((x + residual).astype(F32), scale, bias, axis, epsilon)


def causal_attention(q, k, v, scale: float) -> np.ndarray:
    """The flash-style node's contract: softmax(QK^T*scale + causal) @ V.

    Equals ``attention_scores`` with a 0/-1e9 upper-triangular mask followed by
    the P@V MatMul (c35/engine.py:535-543); q,k,v are [B,H,S,D].
    """
    s = np.matmul(q, k.transpose(0, 1, 3, 2)) * F32(scale)
    S = s.shape[-1]
    s = s + np.triu(np.full((S, S), -1e9, F32), 1)
    return np.matmul(softmax(s.astype(F32), -1), v).astype(F32)


def gelu_erf(x) -> np.ndarray:
    """The 5-op GELU chain x*0.5*(1+erf(x/sqrt2)) executed by fused_ew (erff)."""
    x = np.asarray(x, F32)
    return ((x * (F32(1.0) + erf_exact(x / F32(math.sqrt(2.0))))) * F32(0.5)).astype(F32)


def im2col(x, kernel_shape, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1)) -> np.ndarray:
    """c32/kernel_registry.py:399-453: [N*Ho*Wo, C*kH*kW] patch matrix."""
    x = np.asarray(x, F32)
    N, C, H, W = x.shape
    kH, kW = int(kernel_shape[0]), int(kernel_shape[-1])
    sH, sW = int(strides[0]), int(strides[-1])
    dH, dW = int(dilations[0]), int(dilations[-1])
    pT, pL, pB, pR = (int(p) for p in pads)
    Ho = (H + pT + pB - (dH * (kH - 1) + 1)) // sH + 1
    Wo = (W + pL + pR - (dW * (kW - 1) + 1)) // sW + 1
    xp = np.pad(x, ((0, 0), (0, 0), (pT, pB), (pL, pR)))
    cols = np.empty((N, Ho, Wo, C, kH, kW), F32)
    for r in range(kH):
        for s in range(kW):
            cols[..., r, s] = xp[:, :, r * dH: r * dH + sH * (Ho - 1) + 1: sH,
                                 s * dW: s * dW + sW * (Wo - 1) + 1: sW].transpose(0, 2, 3, 1)
    return cols.reshape(N * Ho * Wo, C * kH * kW)


def ew_chain(ops: List[Dict[str, Any]], inputs: List[np.ndarray]) -> np.ndarray:
    """c35/engine.py:948-1013: interpret a FusedEWChain ``_ops`` program."""
    vals: Dict[str, np.ndarray] = {}
    last = None
    for e in ops:
        args = [inputs[r] if isinstance(r, int) else vals[r] for r in e.get("inputs", [])]
        op = e["op"]
        if op == "Add":
            r = args[0] + args[1]
        elif op == "Sub":
            r = args[0] - args[1]
        elif op == "Mul":
            r = args[0] * args[1]
        elif op == "Div":
            r = args[0] / args[1]
        elif op == "Relu":
            r = np.maximum(args[0], F32(0))
        elif op == "Erf":
            r = erf_exact(args[0])
        elif op == "Sqrt":
            r = np.sqrt(args[0])
        elif op == "Exp":
            r = np.exp(args[0])
        else:
            raise ValueError(op)
        last = np.asarray(r, F32)
        if e.get("output"):
            vals[e["output"]] = last
    return last
