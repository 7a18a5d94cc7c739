"""Launch preparation for every reference kernel name.

``prepare(name, inputs, outputs, params)`` turns one C3.4 ``KernelStep`` — the
reference kernel name, its input tensors, its pre-allocated output slots and
its ``operator_params`` — into native launches of ``libc3b200.so`` plus the
logical output shapes.  It is shared by the eager registry
(``kernel_registry.py``, the drop-in for c32/kernel_registry.py) and by the
plan adapter (``c34_plan.py``), which resolves everything once at plan-build
time.  Semantics follow the reference kernel each builder cites.

Tensors are described by :class:`Desc` (device pointer or arena offset, dtype,
shape, and host values when the tensor is a constant such as a Reshape shape).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib as L


@dataclass
class Desc:
    ptr: int
    dtype: int
    shape: Tuple[int, ...]
    arena: bool = False
    host: Optional[np.ndarray] = None  # host copy of small constants (shapes, split sizes)
    # "nhwc": a logical [N, C, H, W] tensor stored channels-last ([N*H*W, C]),
    # as the tensor-core convolutions read and write it
    layout: str = "plain"

    @property
    def numel(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64)) if self.shape else 1

    def t(self, shape: Optional[Sequence[int]] = None) -> L.Tensor:
        return L.make_tensor(self.ptr, self.dtype, tuple(self.shape if shape is None else shape), self.arena)


@dataclass
class Launch:
    kid: int
    ins: List[L.Tensor]
    outs: List[L.Tensor]
    params: Any


@dataclass
class Prepared:
    launches: List[Launch] = field(default_factory=list)
    out_shapes: List[Tuple[int, ...]] = field(default_factory=list)


_BUILDERS: Dict[str, Callable[..., Prepared]] = {}


def builder(*names: str):
    def deco(fn):
        for n in names:
            _BUILDERS[n] = fn
        return fn
    return deco


def resolve(name: str) -> Callable[..., Prepared]:
    """Alias rules of c32/kernel_registry.py:42-67 (fail closed)."""
    if name in _BUILDERS:
        return _BUILDERS[name]
    if f"{name}_f32" in _BUILDERS:
        return _BUILDERS[f"{name}_f32"]
    if name.endswith("_f32") and name[:-4] in _BUILDERS:
        return _BUILDERS[name[:-4]]
    if name.endswith("_fp32"):
        bare = name[:-5]
        if f"{bare}_f32" in _BUILDERS:
            return _BUILDERS[f"{bare}_f32"]
        if bare in _BUILDERS:
            return _BUILDERS[bare]
    raise RuntimeError(f"Unknown kernel: {name!r}.  Registered kernels: {sorted(_BUILDERS)}")


def registered() -> List[str]:
    return sorted(_BUILDERS)


def prepare(name: str, ins: Sequence[Optional[Desc]], outs: Sequence[Desc], params: Dict[str, Any]) -> Prepared:
    return resolve(name)(list(ins), list(outs), dict(params or {}))


# ------------------------------------------------------------------ helpers

def _out(outs: Sequence[Desc], i: int, shape: Sequence[int], dtype: int = L.F32) -> L.Tensor:
    o = outs[i]
    need = int(np.prod(shape, dtype=np.int64)) if len(shape) else 1
    if need * L.DTYPE_SIZE[dtype] > o.numel * L.DTYPE_SIZE[o.dtype]:
        raise ValueError(f"Output arena too small: need {need} elements, have {o.numel}")
    return L.make_tensor(o.ptr, dtype, tuple(shape), o.arena)


def _host_ints(d: Optional[Desc]) -> Optional[List[int]]:
    if d is None or d.host is None:
        return None
    return [int(v) for v in np.asarray(d.host).reshape(-1).tolist()]


def _ew_program(ops: Sequence[Tuple[int, int, int]], imm: Sequence[float] = ()) -> L.EwParams:
    p = L.EwParams()
    if len(ops) > L.EW_MAX_OPS:
        raise ValueError("elementwise program too long")
    p.n_ops = len(ops)
    for k, (op, a, b) in enumerate(ops):
        p.op[k], p.a[k], p.b[k] = op, a, b
    for k, v in enumerate(imm):
        p.imm[k] = float(v)
    return p


def _ew(ins: Sequence[Desc], outs, ops, imm=(), views: Optional[Sequence[Sequence[int]]] = None) -> Prepared:
    shapes = [tuple(v) for v in views] if views else [d.shape for d in ins]
    out_shape = tuple(np.broadcast_shapes(*shapes)) if shapes else ()
    tin = [d.t(s) for d, s in zip(ins, shapes)]
    return Prepared([Launch(L.K_EW, tin, [_out(outs, 0, out_shape)], _ew_program(ops, imm))], [out_shape])


def _copy_launch(src: Desc, dst: L.Tensor, strides: Sequence[int], offset: int = 0) -> Launch:
    p = L.CopyParams()
    p.in_offset = int(offset)
    for i, s in enumerate(strides):
        p.in_stride[i] = int(s)
    return Launch(L.K_COPY, [src.t()], [dst], p)


def _contig_strides(shape: Sequence[int]) -> List[int]:
    st, acc = [], 1
    for d in reversed(shape):
        st.append(acc)
        acc *= int(d)
    return list(reversed(st))


def _identity_copy(src: Desc, outs, shape) -> Prepared:
    n = src.numel
    flat = _out(outs, 0, (n,), src.dtype)
    return Prepared([_copy_launch(Desc(src.ptr, src.dtype, (n,), src.arena), flat, [1])], [tuple(shape)])


def _permute(src: Desc, perm: Sequence[int], outs, final_shape=None) -> Prepared:
    st = _contig_strides(src.shape)
    tshape = tuple(src.shape[p] for p in perm)
    dst = _out(outs, 0, tshape, src.dtype)
    return Prepared([_copy_launch(src, dst, [st[p] for p in perm])], [tuple(final_shape or tshape)])


# ------------------------------------------------------------ elementwise
# c32/kernel_registry.py:200-265

@builder("add", "add_f32")
def _b_add(ins, outs, p):
    if "epsilon" in p and len(ins) == 1:
        return _ew(ins[:1], outs, [(L.OP_ADD_IMM, 0, 0)], [p["epsilon"]])
    return _ew(ins[:2], outs, [(L.OP_ADD, 0, 1)])


@builder("mul", "mul_f32")
def _b_mul(ins, outs, p):
    return _ew(ins[:2], outs, [(L.OP_MUL, 0, 1)])


@builder("div", "div_f32")
def _b_div(ins, outs, p):
    return _ew(ins[:2], outs, [(L.OP_DIV, 0, 1)])


@builder("sub", "sub_f32")
def _b_sub(ins, outs, p):
    return _ew(ins[:2], outs, [(L.OP_SUB, 0, 1)])


@builder("relu_f32")
def _b_relu(ins, outs, p):
    return _ew(ins[:1], outs, [(L.OP_RELU, 0, 0)])


@builder("erf_f32")
def _b_erf(ins, outs, p):
    # The registry's Erf is the A&S 7.1.26 approximation (kernel_registry.py:179-192).
    return _ew(ins[:1], outs, [(L.OP_ERF_AS, 0, 0)])


@builder("exp", "exp_f32")
def _b_exp(ins, outs, p):
    return _ew(ins[:1], outs, [(L.OP_EXP, 0, 0)])


@builder("sqrt", "sqrt_f32")
def _b_sqrt(ins, outs, p):
    return _ew(ins[:1], outs, [(L.OP_SQRT, 0, 0)])


@builder("reciprocal", "reciprocal_f32")
def _b_recip(ins, outs, p):
    return _ew(ins[:1], outs, [(L.OP_RECIP, 0, 0)])


@builder("add_bias_f32")
def _b_add_bias(ins, outs, p):
    """kernel_registry.py:379-392: data + beta * bias broadcast along bias_axis."""
    data, bias = ins[0], ins[1]
    axis = int(p.get("bias_axis", -1)) % len(data.shape)
    bshape = [1] * len(data.shape)
    bshape[axis] = bias.numel
    return _ew([data, bias], outs, [(L.OP_MUL_IMM, 1, 0), (L.OP_ADD, 0, -1)],
               [float(p.get("beta", 1.0))], views=[data.shape, bshape])


@builder("batchnorm_f32")
def _b_bn(ins, outs, p):
    """kernel_registry.py:573-584: (x - mean) / sqrt(var + eps) * scale + bias."""
    x = ins[0]
    ch = [1, -1] + [1] * (len(x.shape) - 2)
    c = x.shape[1]
    vs = [tuple(c if v == -1 else v for v in ch)] * 4
    ops = [(L.OP_ADD_IMM, 4, 0), (L.OP_SQRT, -1, 0), (L.OP_SUB, 0, 3), (L.OP_DIV, -3, -2),
           (L.OP_MUL, -4, 1), (L.OP_ADD, -5, 2)]
    return _ew(ins[:5], outs, ops, [float(p.get("epsilon", 1e-5))], views=[x.shape] + vs)


@builder("fused_residual_relu_f32")
def _b_res_relu(ins, outs, p):
    """kernel_registry.py:654-662: max(conv + residual, 0)."""
    return _ew(ins[:2], outs, [(L.OP_ADD, 0, 1), (L.OP_RELU, -1, 0)])


_EW_OPCODE = {"Add": L.OP_ADD, "Sub": L.OP_SUB, "Mul": L.OP_MUL, "Div": L.OP_DIV, "Relu": L.OP_RELU,
              "Erf": L.OP_ERF, "Sqrt": L.OP_SQRT, "Exp": L.OP_EXP}


@builder("fused_ew_f32")
def _b_fused_ew(ins, outs, p):
    """c35/engine.py:948-1013: interpret the ``_ops`` chain (Erf is CUDA erff there)."""
    ops = p.get("_ops") or []
    if not ops:
        raise ValueError("FusedEWChain has no elementwise program")
    names: Dict[str, int] = {}
    prog = []
    for k, e in enumerate(ops):
        refs = []
        for r in e.get("inputs", []):
            if isinstance(r, int) and 0 <= r < len(ins):
                refs.append(r)
            elif isinstance(r, str) and r in names:
                refs.append(-names[r] - 1)
            else:
                raise ValueError(f"FusedEWChain cannot resolve operand {r!r}")
        op = e.get("op", "")
        if op not in _EW_OPCODE:
            raise ValueError(f"Unknown op in FusedEWChain: {op}")
        arity = 1 if op in ("Relu", "Erf", "Sqrt", "Exp") else 2
        if len(refs) != arity:
            raise ValueError(f"FusedEWChain {op} expects {arity} operands")
        prog.append((_EW_OPCODE[op], refs[0], refs[1] if arity == 2 else 0))
        if e.get("output"):
            names[e["output"]] = k
    return _ew(ins, outs, prog)


# ------------------------------------------------------------ reductions
# c32/kernel_registry.py:268-311

def _red_axes(p, ndim):
    axes, axis = p.get("axes"), p.get("axis")
    keep = bool(p.get("keepdims", False))
    if axes is not None:
        ax = [int(a) % ndim for a in (axes if isinstance(axes, list) else [axes])]
    elif axis is not None:
        ax = [int(axis) % ndim]
    else:
        ax = list(range(ndim))
    return sorted(set(ax)), keep


def _reduce(ins, outs, p, op):
    x = ins[0]
    ax, keep = _red_axes(p, len(x.shape))
    if ax != list(range(ax[0], ax[-1] + 1)):
        raise ValueError("reduce: non-contiguous reduction axes are not supported")
    outer = int(np.prod(x.shape[:ax[0]], dtype=np.int64))
    red = int(np.prod(x.shape[ax[0]:ax[-1] + 1], dtype=np.int64))
    inner = int(np.prod(x.shape[ax[-1] + 1:], dtype=np.int64))
    shape = tuple(1 if i in ax else d for i, d in enumerate(x.shape)) if keep else \
        tuple(d for i, d in enumerate(x.shape) if i not in ax)
    rp = L.ReduceParams(outer, red, inner, op, 0)
    return Prepared([Launch(L.K_REDUCE, [x.t()], [_out(outs, 0, shape)], rp)], [shape])


@builder("reduce_mean", "reduce_mean_f32")
def _b_rmean(ins, outs, p):
    return _reduce(ins, outs, p, L.RED_MEAN)


@builder("reduce_sum", "reduce_sum_f32")
def _b_rsum(ins, outs, p):
    return _reduce(ins, outs, p, L.RED_SUM)


@builder("reduce_max", "reduce_max_f32")
def _b_rmax(ins, outs, p):
    return _reduce(ins, outs, p, L.RED_MAX)


# ------------------------------------------------------------ contractions

def _gemm_params(M, N, K, *, batch=1, sa=0, sb=0, sc=0, ta=0, tb=0, alpha=1.0, beta=1.0, bias=L.BIAS_NONE,
                 act=L.ACT_NONE, res=0) -> L.GemmParams:
    g = L.GemmParams()
    g.M, g.N, g.K, g.batch = M, N, K, batch
    g.stride_a, g.stride_b, g.stride_c = sa, sb, sc
    g.trans_a, g.trans_b, g.alpha, g.beta = ta, tb, alpha, beta
    g.bias_mode, g.act, g.has_residual = bias, act, res
    return g


@builder("matmul_f32")
def _b_matmul(ins, outs, p):
    """kernel_registry.py:318-358 (cuBLAS via cp.dot / cp.matmul in the reference)."""
    a, b = ins[0], ins[1]
    ta, tb = int(p.get("transA", 0)), int(p.get("transB", 0))
    alpha = float(p.get("alpha", 1.0))
    if p.get("lowering_kind", "matmul") == "conv_contract":
        # a [M, CK]; b [O, C, kh, kw] -> b2d [O, CK]; result a @ b2d.T
        M, K = (a.shape[1], a.shape[0]) if ta else (a.shape[0], a.shape[1])
        if len(b.shape) == 4:
            O = b.shape[0]
            bt = 0 if tb else 1  # b2d is [O, CK] (N x K); transB flips it
        else:
            O = b.shape[1] if not tb else b.shape[0]
            bt = tb
        N = O
        g = _gemm_params(M, N, K, ta=ta, tb=bt, alpha=alpha)
        shape = (M, N)
        return Prepared([Launch(L.K_GEMM, [a.t(), b.t()], [_out(outs, 0, shape)], g)], [shape])
    if ta or tb:
        if len(a.shape) != 2 or len(b.shape) != 2:
            raise ValueError("matmul: transA/transB need rank-2 operands")
    if len(a.shape) == 2 and len(b.shape) == 2:
        M, K = (a.shape[1], a.shape[0]) if ta else a.shape
        N = b.shape[0] if tb else b.shape[1]
        g = _gemm_params(M, N, K, ta=ta, tb=tb, alpha=alpha)
        return Prepared([Launch(L.K_GEMM, [a.t(), b.t()], [_out(outs, 0, (M, N))], g)], [(M, N)])
    # batched matmul with NumPy broadcasting of leading dims
    ash = a.shape if len(a.shape) >= 2 else (1,) + a.shape
    bsh = b.shape if len(b.shape) >= 2 else b.shape + (1,)
    M, K = ash[-2], ash[-1]
    N = bsh[-1]
    lead = tuple(np.broadcast_shapes(ash[:-2], bsh[:-2]))
    batch = int(np.prod(lead, dtype=np.int64)) if lead else 1
    abat = int(np.prod(ash[:-2], dtype=np.int64)) if len(ash) > 2 else 1
    bbat = int(np.prod(bsh[:-2], dtype=np.int64)) if len(bsh) > 2 else 1
    if abat not in (1, batch) or bbat not in (1, batch):
        raise ValueError("matmul: partially broadcast batch dimensions are not supported")
    g = _gemm_params(M, N, K, batch=batch, sa=M * K if abat > 1 else 0, sb=K * N if bbat > 1 else 0, sc=M * N,
                     alpha=alpha)
    shape = lead + (M, N)
    return Prepared([Launch(L.K_GEMM, [a.t(), b.t()], [_out(outs, 0, shape)], g)], [shape])


def _gemm_epilogue(ins, outs, p, matmul_semantics: bool) -> Prepared:
    """c35/engine.py:722-844 (_execute_gemm_epilogue)."""
    a, b = ins[0], ins[1]
    ash = a.shape
    fa = p.get("_flatten_axis")
    if fa is not None:
        ax = int(fa) + len(ash) if int(fa) < 0 else int(fa)
        if not 0 <= ax <= len(ash):
            raise ValueError("Fused GEMM Flatten axis is out of range")
        ash = (int(np.prod(ash[:ax], dtype=np.int64)), int(np.prod(ash[ax:], dtype=np.int64)))
    if matmul_semantics:
        lead = tuple(ash[:-1])
        ash = (int(np.prod(lead, dtype=np.int64)), ash[-1])
        ta = tb = 0
    else:
        if len(ash) != 2:
            raise ValueError("Fused Gemm requires rank-2 A after Flatten")
        lead = ()
        ta, tb = int(p.get("transA", 0)), int(p.get("transB", 0))
    m = ash[1] if ta else ash[0]
    k = ash[0] if ta else ash[1]
    bk = b.shape[1] if tb else b.shape[0]
    n = b.shape[0] if tb else b.shape[1]
    if k != bk:
        raise ValueError(f"Fused GEMM inner dimensions differ: {k} and {bk}")
    mode = L.BIAS_NONE
    tin = [Desc(a.ptr, a.dtype, ash, a.arena).t(), b.t()]
    if len(ins) >= 3 and ins[2] is not None:
        c = ins[2]
        cs = list(c.shape)
        while len(cs) > 2 and cs[0] == 1:
            cs.pop(0)
        if len(cs) == 0:
            cr, cc = 1, 1
        elif len(cs) == 1:
            cr, cc = 1, cs[0]
        elif len(cs) == 2:
            cr, cc = cs
        else:
            raise ValueError("Fused GEMM bias rank is not broadcastable")
        if cr not in (1, m) or cc not in (1, n):
            raise ValueError(f"Fused GEMM bias shape {c.shape} cannot broadcast to {(m, n)}")
        mode = {(True, True): L.BIAS_SCALAR, (True, False): L.BIAS_COL, (False, True): L.BIAS_ROW,
                (False, False): L.BIAS_FULL}[(cr == 1, cc == 1)]
        if cr == 1 and cc == 1 and m == 1 and n == 1:
            mode = L.BIAS_SCALAR
        tin.append(c.t((c.numel,)))
    act = L.ACT_RELU if p.get("_activation") == "Relu" else L.ACT_NONE
    g = _gemm_params(m, n, k, ta=ta, tb=tb, alpha=float(p.get("alpha", 1.0)), beta=float(p.get("beta", 1.0)),
                     bias=mode, act=act)
    shape = lead + (n,) if matmul_semantics else (m, n)
    return Prepared([Launch(L.K_GEMM, tin, [_out(outs, 0, shape)], g)], [shape])


@builder("fused_gemm_epilogue_f32")
def _b_gemm_epi(ins, outs, p):
    return _gemm_epilogue(ins, outs, p, False)


@builder("fused_matmul_bias_f32")
def _b_matmul_bias(ins, outs, p):
    return _gemm_epilogue(ins, outs, p, True)


@builder("b200linearepilogue_f32")
def _b_b200_linear(ins, outs, p):
    """The fused node of hackathon_b200.c33_passes.fuse_linear_epilogue in fp32:
    MatMul + bias [+ exact-erf GELU | + residual] in one launch (the GELU
    chain's constants are checked by the caller)."""
    a, b = ins[0], ins[1]
    lead = tuple(a.shape[:-1])
    M, K = int(np.prod(lead, dtype=np.int64)), a.shape[-1]
    if b.shape[0] != K:
        raise ValueError(f"linear: inner dimensions differ: {K} and {b.shape[0]}")
    N = b.shape[1]
    ri = p.get("_residual_input_index")
    res = ins[int(ri)] if ri is not None else None
    bias = ins[2] if len(ins) > 2 and ins[2] is not None else None
    act = {"Relu": L.ACT_RELU, "Gelu": L.ACT_GELU}.get(p.get("_activation"), L.ACT_NONE)
    g = _gemm_params(M, N, K, bias=L.BIAS_COL if bias is not None else L.BIAS_NONE, act=act,
                     res=int(res is not None))
    tin = [a.t((M, K)), b.t()] + ([bias.t((N,))] if bias is not None else []) + \
        ([res.t((M, N))] if res is not None else [])
    shape = lead + (N,)
    return Prepared([Launch(L.K_GEMM, tin, [_out(outs, 0, shape)], g)], [shape])


# ------------------------------------------------------------ convolution

def conv_geometry(p: Dict[str, Any], H: int, W: int, kh: int, kw: int) -> Tuple[L.ConvGeom, int, int]:
    """Geometry of c35/engine.py:288-440 (pads / auto_pad / strides / dilations)."""
    ks = p.get("kernel_shape") or [kh, kw]
    kh, kw = int(ks[0]), int(ks[-1])
    st = list(p.get("strides", [1, 1]))
    sh, sw = int(st[0]), int(st[-1])
    dl = list(p.get("dilations", [1, 1]))
    dh, dw = int(dl[0]), int(dl[-1])
    ap = p.get("auto_pad", "NOTSET")
    ap = (ap.decode() if isinstance(ap, bytes) else str(ap)).upper()
    eh, ew = dh * (kh - 1) + 1, dw * (kw - 1) + 1
    if ap in ("SAME_UPPER", "SAME_LOWER"):
        oh, ow = math.ceil(H / sh), math.ceil(W / sw)
        th, tw = max((oh - 1) * sh + eh - H, 0), max((ow - 1) * sw + ew - W, 0)
        if ap == "SAME_UPPER":
            pt, pl = th // 2, tw // 2
        else:
            pt, pl = (th + 1) // 2, (tw + 1) // 2
        pb, pr = th - pt, tw - pl
    elif ap == "VALID":
        pt = pl = pb = pr = 0
    else:
        pads = list(p.get("pads", [0, 0, 0, 0]))
        pt, pl, pb, pr = (int(v) for v in pads)
    Ho = (H + pt + pb - eh) // sh + 1
    Wo = (W + pl + pr - ew) // sw + 1
    if Ho <= 0 or Wo <= 0:
        raise ValueError("Conv attributes produce a non-positive output dimension")
    g = L.ConvGeom(kh, kw, sh, sw, pt, pl, pb, pr, dh, dw)
    return g, Ho, Wo


@builder("im2col_f32")
def _b_im2col(ins, outs, p):
    """kernel_registry.py:399-453."""
    x = ins[0]
    N, C, H, W = x.shape
    ks = p.get("kernel_shape", [3, 3])
    g, Ho, Wo = conv_geometry({**p, "auto_pad": "NOTSET"}, H, W, int(ks[0]), int(ks[-1]))
    shape = (N * Ho * Wo, C * g.kh * g.kw)
    return Prepared([Launch(L.K_IM2COL, [x.t()], [_out(outs, 0, shape)], g)], [shape])


def _conv_nchw(x: Desc, w: Desc, bias: Optional[Desc], res: Optional[Desc], outs, p, act=L.ACT_NONE) -> Prepared:
    N, C, H, W = x.shape
    O, Cg, kh, kw = w.shape
    if int(p.get("group", 1)) != 1 or Cg != C:
        raise ValueError("conv: grouped convolution is not supported")
    g, Ho, Wo = conv_geometry(p, H, W, kh, kw)
    cp = L.ConvParams()
    cp.n, cp.c, cp.h, cp.w, cp.cout, cp.ho, cp.wo, cp.layout = N, C, H, W, O, Ho, Wo, 0
    cp.g = g
    cp.has_bias = int(bias is not None)
    cp.has_residual = int(res is not None)
    cp.act = act
    tin = [x.t(), w.t()] + ([bias.t((O,))] if bias is not None else []) + ([res.t()] if res is not None else [])
    shape = (N, O, Ho, Wo)
    return Prepared([Launch(L.K_CONV, tin, [_out(outs, 0, shape)], cp)], [shape])


@builder("winograd_forward_f32")
def _b_winograd(ins, outs, p):
    """kernel_registry.py:460-566 is meant to compute a 3x3 stride-1 Conv but
    raises at its first einsum (line 534); this is the Conv it stands for."""
    return _conv_nchw(ins[0], ins[1], None, None, outs, p)


@builder("conv2d_bias_act_f32")
def _b_conv_f32(ins, outs, p):
    bias = ins[2] if len(ins) > 2 and ins[2] is not None else None
    res = ins[3] if len(ins) > 3 else None
    act = L.ACT_RELU if p.get("_activation") == "Relu" else L.ACT_NONE
    return _conv_nchw(ins[0], ins[1], bias, res, outs, p, act)


@builder("b200convbiasact_f32")
def _b_b200_conv(ins, outs, p):
    """The fused node of hackathon_b200.c33_passes.fuse_conv_bias_act in fp32:
    conv (BN folded into w, b) + bias [+ residual] [+ ReLU] in one launch."""
    ri = p.get("_residual_input_index")
    res = ins[int(ri)] if ri is not None else None
    bias = ins[2] if len(ins) > 2 and ins[2] is not None else None
    act = L.ACT_RELU if p.get("_activation") == "Relu" else L.ACT_NONE
    return _conv_nchw(ins[0], ins[1], bias, res, outs, p, act)


@builder("conv_reshape_f32")
def _b_conv_reshape(ins, outs, p):
    """kernel_registry.py:105-175, 365-372: NHWO contract -> NCHW."""
    src = ins[0]
    if len(src.shape) != 2:
        return _identity_copy(src, outs, src.shape)
    M, O = src.shape
    N = int(p.get("_batch_size") or 0)
    if not N or M % N:
        return _identity_copy(src, outs, src.shape)
    HW = M // N
    hw = None
    osp = p.get("_output_spatial")
    if osp and len(osp) == 2 and int(osp[0]) * int(osp[1]) == HW and int(osp[0]) > 0:
        hw = (int(osp[0]), int(osp[1]))
    if hw is None:
        isp = p.get("_input_spatial")
        if isp and len(isp) == 2:
            ks = p.get("kernel_shape", [3, 3])
            g, Ho, Wo = conv_geometry({**p, "auto_pad": "NOTSET"}, int(isp[0]), int(isp[1]), int(ks[0]), int(ks[-1]))
            if Ho * Wo == HW:
                hw = (Ho, Wo)
    if hw is None:
        h = int(math.isqrt(HW))
        while h > 0 and HW % h:
            h -= 1
        hw = (h, HW // h)
    Ho, Wo = hw
    dst = _out(outs, 0, (N, O, Ho, Wo))
    return Prepared([_copy_launch(src, dst, [Ho * Wo * O, 1, Wo * O, O])], [(N, O, Ho, Wo)])


# ------------------------------------------------------------ normalisation / softmax

def _ln(x: Desc, res: Optional[Desc], scale: Desc, bias: Optional[Desc], outs, axis, eps) -> Prepared:
    ax = int(axis) % len(x.shape)
    cols = int(np.prod(x.shape[ax:], dtype=np.int64))
    rows = x.numel // cols if cols else 0
    if scale.numel != cols:
        raise ValueError("LayerNorm scale size does not match normalized shape")
    lp = L.LayerNormParams(rows, cols, float(eps), int(res is not None), int(bias is not None), 0)
    tin = [x.t()] + ([res.t()] if res is not None else []) + [scale.t((cols,))] + \
          ([bias.t((cols,))] if bias is not None else [])
    return Prepared([Launch(L.K_LAYERNORM, tin, [_out(outs, 0, x.shape)], lp)], [x.shape])


@builder("fused_layer_norm_f32")
def _b_ln(ins, outs, p):
    """c35/engine.py:1170-1247."""
    bias = ins[2] if len(ins) > 2 and ins[2] is not None else None
    return _ln(ins[0], None, ins[1], bias, outs, p.get("axis", -1), p.get("epsilon", 1e-5))


@builder("fused_residual_norm_f32")
def _b_res_ln(ins, outs, p):
    """c35/engine.py:1078-1167: LayerNorm(x + residual)."""
    if ins[0].shape != ins[1].shape:
        raise ValueError("FusedResidualNorm requires equal residual input shapes")
    bias = ins[3] if len(ins) > 3 and ins[3] is not None else None
    return _ln(ins[0], ins[1], ins[2], bias, outs, p.get("axis", -1), p.get("epsilon", 1e-5))


@builder("fused_softmax_f32")
def _b_softmax(ins, outs, p):
    """c35/engine.py:1016-1075."""
    x = ins[0]
    ax = int(p.get("axis", -1)) % len(x.shape)
    sp = L.SoftmaxParams(int(np.prod(x.shape[:ax], dtype=np.int64)), x.shape[ax],
                         int(np.prod(x.shape[ax + 1:], dtype=np.int64)))
    return Prepared([Launch(L.K_SOFTMAX, [x.t()], [_out(outs, 0, x.shape)], sp)], [x.shape])


@builder("fused_attention_scores_f32")
def _b_attn(ins, outs, p):
    """c35/engine.py:1250-1380: softmax(Q K^T / divisor + mask), [B,H,S,S]."""
    q, k, div, mask = ins[:4]
    if len(q.shape) != 4 or len(k.shape) != 4:
        raise ValueError("FusedAttentionScores requires rank-4 MatMul inputs")
    q0, q1, rows, inner = q.shape
    k0, k1, kin, cols = k.shape
    if inner != kin:
        raise ValueError("FusedAttentionScores MatMul inner dimensions differ")
    out0, out1 = max(q0, k0), max(q1, k1)
    ms = [1] * (4 - len(mask.shape)) + list(mask.shape)
    ap = L.AttnScoresParams()
    for n, v in zip(("q0", "q1", "k0", "k1", "rows", "cols", "inner", "out0", "out1"),
                    (q0, q1, k0, k1, rows, cols, inner, out0, out1)):
        setattr(ap, n, int(v))
    for i in range(4):
        ap.m[i] = int(ms[i])
    shape = (out0, out1, rows, cols)
    return Prepared([Launch(L.K_ATTN_SCORES, [q.t(), k.t(), div.t(), mask.t()], [_out(outs, 0, shape)], ap)],
                    [shape])


# ------------------------------------------------------------ data movement
# kernel_registry.py:669-759, engine.py:1383-1445

def flash_params_from_node(qkv: Desc, heads_shape: Desc, divisor: Desc, mask: Desc, p) -> L.FlashParams:
    """FlashParams for a B200FlashAttention node (hackathon_b200.c33_passes):
    qkv [B, S, 3*H*D] split into Q, K, V in that order along the last axis,
    heads from the Reshape target [., S, H, D], scale 1/divisor, and a mask
    that must be all zero or causal (0 on and below the diagonal, -1e9 above;
    the seeded graphs' mask, c35/engine.py:1250-1380 adds it before softmax)."""
    if list(p.get("_qkv_order", [0, 1, 2])) != [0, 1, 2]:
        raise ValueError("flash attention: Q, K, V must be the Split outputs 0, 1, 2")
    hs = _host_ints(heads_shape)
    if hs is None or len(hs) != 4 or divisor.host is None or mask.host is None:
        raise ValueError("flash attention: heads shape, divisor and mask must be constants")
    if len(qkv.shape) != 3:
        raise ValueError("flash attention: qkv must be [B, S, 3*H*D]")
    B, S, three_hd = qkv.shape
    H, D = hs[2], hs[3]
    if 3 * H * D != three_hd:
        raise ValueError("flash attention: qkv width is not 3 * heads * head_dim")
    m = np.asarray(mask.host, np.float32)
    if m.size == S * S:
        m2 = m.reshape(S, S)
        causal = np.array_equal(m2, np.triu(np.full((S, S), -1e9, np.float32), 1))
        if not causal and np.any(m2):
            raise ValueError("flash attention: only an all-zero or causal (0/-1e9) mask is supported")
    elif np.any(m):
        raise ValueError("flash attention: the mask must be [.., S, S]")
    else:
        causal = False
    div = float(np.asarray(divisor.host).reshape(-1)[0])
    return L.FlashParams(B, S, H, D, 1.0 / div, int(causal))


@builder("b200flashattention_f32")
def _b_b200_flash(ins, outs, p):
    """The fused node of hackathon_b200.c33_passes.fuse_flash_attention in fp32:
    softmax(Q K^T / divisor + mask) V with heads merged, read from the packed
    QKV projection, no score tensor."""
    qkv = ins[0]
    fp = flash_params_from_node(qkv, ins[1], ins[2], ins[3], p)
    shape = (fp.batch, fp.seq, fp.heads * fp.head_dim)
    return Prepared([Launch(L.K_FLASH_ATTN, [qkv.t()], [_out(outs, 0, shape, qkv.dtype)], fp)], [shape])


def resolve_reshape(in_shape, target, allowzero=0) -> Tuple[int, ...]:
    out, infer, known = [], None, 1
    for i, d in enumerate(int(v) for v in target):
        if d == 0 and not allowzero:
            d = int(in_shape[i])
        if d == -1:
            infer = i
            out.append(-1)
        else:
            out.append(d)
            known *= d
    total = int(np.prod(in_shape, dtype=np.int64))
    if infer is not None:
        out[infer] = total // known
    elif int(np.prod(out, dtype=np.int64)) != total:
        raise ValueError("Reshape target element count does not match input")
    return tuple(out)


@builder("reshape")
def _b_reshape(ins, outs, p):
    x = ins[0]
    tgt = _host_ints(ins[1]) if len(ins) > 1 and ins[1] is not None and ins[1].numel > 0 else None
    if tgt is None:
        tgt = list(p.get("_reshape_shape", x.shape))
    shape = resolve_reshape(x.shape, tgt, int(p.get("allowzero", 0)))
    return _identity_copy(x, outs, shape)


@builder("transpose")
def _b_transpose(ins, outs, p):
    x = ins[0]
    perm = p.get("perm") or list(range(len(x.shape) - 1, -1, -1))
    return _permute(x, [int(v) for v in perm], outs)


@builder("fused_transpose_reshape_f32")
def _b_transpose_reshape(ins, outs, p):
    x = ins[0]
    perm = [int(v) for v in (p.get("perm") or range(len(x.shape) - 1, -1, -1))]
    tshape = tuple(x.shape[i] for i in perm)
    tgt = _host_ints(ins[1])
    if tgt is None:
        raise ValueError("FusedTransposeReshape needs the shape tensor's host values")
    return _permute(x, perm, outs, resolve_reshape(tshape, tgt, int(p.get("allowzero", 0))))


@builder("flatten")
def _b_flatten(ins, outs, p):
    x = ins[0]
    ax = int(p.get("axis", 1))
    if ax < 0:
        ax += len(x.shape)
    shape = (int(np.prod(x.shape[:ax], dtype=np.int64)), int(np.prod(x.shape[ax:], dtype=np.int64)))
    return _identity_copy(x, outs, shape)


@builder("split")
def _b_split(ins, outs, p):
    """kernel_registry.py:713-741 (+ split sizes from the second input, engine.py:557-601)."""
    x = ins[0]
    ax = int(p.get("axis", 0)) % len(x.shape)
    sizes = _host_ints(ins[1]) if len(ins) > 1 and ins[1] is not None and ins[1].numel > 0 else None
    if not sizes:
        sizes = [int(s) for s in (p.get("split") or [])]
    nout = int(p.get("_num_outputs", len(outs)))
    if not sizes:
        if nout <= 0 or x.shape[ax] % nout:
            raise ValueError("Split requires equal division")
        sizes = [x.shape[ax] // nout] * nout
    st = _contig_strides(x.shape)
    res = Prepared()
    off = 0
    for i, sz in enumerate(sizes):
        shape = tuple(sz if d == ax else x.shape[d] for d in range(len(x.shape)))
        if i < len(outs):
            dst = _out(outs, i, shape, x.dtype)
            res.launches.append(_copy_launch(x, dst, st, off * st[ax]))
            res.out_shapes.append(shape)
        off += sz
    return res


@builder("gather")
def _b_gather(ins, outs, p):
    """kernel_registry.py:744-752: np.take(data, indices, axis)."""
    x, idx = ins[0], ins[1]
    ax = int(p.get("axis", 0)) % len(x.shape)
    gp = L.GatherParams(int(np.prod(x.shape[:ax], dtype=np.int64)), x.shape[ax], idx.numel,
                        int(np.prod(x.shape[ax + 1:], dtype=np.int64)))
    shape = tuple(x.shape[:ax]) + tuple(idx.shape) + tuple(x.shape[ax + 1:])
    return Prepared([Launch(L.K_GATHER, [x.t(), idx.t((idx.numel,))], [_out(outs, 0, shape, x.dtype)], gp)],
                    [shape])


@builder("constant")
def _b_constant(ins, outs, p):
    """Constants are pre-loaded by H2D; the kernel is a no-op (kernel_registry.py:755-759)."""
    return Prepared([], [])
