"""Drop-in replacement for the reference's ``c32/kernel_registry.py``.

Same public surface — ``register``, ``lookup``, ``is_registered``,
``list_registered`` and one function per kernel name with the reference
signature (c32/kernel_registry.py:6-16)::

    kernel(inputs, outputs, params, tuning) -> None

``inputs`` / ``outputs`` are device arrays: anything exposing
``__cuda_array_interface__`` (CuPy arrays, which is what the reference's
executor passes) or torch CUDA tensors.  As in the reference, ``outputs[i]`` is
a pre-allocated float32 arena view of the full planned capacity and is replaced
by a view of the written result with its logical shape (the contract of
``_write_result``, c32/kernel_registry.py:84-102).  Every computation runs in
``libc3b200.so``; nothing here computes on the host, and an unknown name fails
closed with ``RuntimeError("Unknown kernel: ...")`` (kernel_registry.py:65-67).
The launch stream is the caller's current stream (CuPy's or torch's), as in
``with stream:`` at c35/executor.py:843-846.
"""

from __future__ import annotations

from typing import Any, Callable, Dict, List, Optional

import numpy as np

from . import _lib as L
from .kernels import Desc, prepare, registered as _prepared_names, resolve as _resolve_builder

KernelFunc = Callable[..., None]
_registry: Dict[str, KernelFunc] = {}

_TYPESTR = {"<f4": L.F32, "<i8": L.I64, "<i4": L.I32, "<f2": L.F16, "|u1": L.U8, "<V2": L.BF16}


def register(name: str) -> Callable[[KernelFunc], KernelFunc]:
    def decorator(fn: KernelFunc) -> KernelFunc:
        _registry[name] = fn
        return fn
    return decorator


def lookup(name: str) -> KernelFunc:
    """Name resolution of c32/kernel_registry.py:42-67 (verbatim, +_f32, -_f32, _fp32)."""
    if name in _registry:
        return _registry[name]
    cand = f"{name}_f32"
    if cand in _registry:
        return _registry[cand]
    if name.endswith("_f32") and name[:-4] in _registry:
        return _registry[name[:-4]]
    if name.endswith("_fp32"):
        bare = name[:-5]
        if f"{bare}_f32" in _registry:
            return _registry[f"{bare}_f32"]
        if bare in _registry:
            return _registry[bare]
    raise RuntimeError(f"Unknown kernel: {name!r}.  Registered kernels: {sorted(_registry)}")


def is_registered(name: str) -> bool:
    try:
        lookup(name)
        return True
    except RuntimeError:
        return False


def list_registered() -> List[str]:
    return sorted(_registry)


# ------------------------------------------------------------------ arrays

def _is_torch(x: Any) -> bool:
    return type(x).__module__.startswith("torch")


def describe(x: Any) -> Desc:
    """Device array -> Desc (pointer, dtype, shape); must be C-contiguous."""
    if _is_torch(x):
        import torch
        if not x.is_cuda:
            raise TypeError("kernel arrays must live on the GPU")
        if not x.is_contiguous():
            raise ValueError("kernel arrays must be C-contiguous")
        dmap = {torch.float32: L.F32, torch.bfloat16: L.BF16, torch.float16: L.F16, torch.int64: L.I64,
                torch.int32: L.I32, torch.uint8: L.U8}
        return Desc(int(x.data_ptr()), dmap[x.dtype], tuple(int(d) for d in x.shape))
    cai = getattr(x, "__cuda_array_interface__", None)
    if cai is None:
        raise TypeError(f"unsupported array type {type(x).__name__}: need a device array")
    shape = tuple(int(d) for d in cai["shape"])
    st = cai.get("strides")
    if st is not None:
        es = np.dtype(cai["typestr"]).itemsize
        exp = []
        acc = es
        for d in reversed(shape):
            exp.append(acc)
            acc *= d
        if tuple(reversed(exp)) != tuple(st) and int(np.prod(shape)) > 1:
            raise ValueError("kernel arrays must be C-contiguous")
    ts = cai["typestr"]
    if ts not in _TYPESTR:
        raise TypeError(f"unsupported dtype {ts}")
    return Desc(int(cai["data"][0]), _TYPESTR[ts], shape)


def _host_values(x: Any) -> np.ndarray:
    if _is_torch(x):
        return x.detach().cpu().numpy()
    if hasattr(x, "get"):
        return x.get()
    return np.asarray(x)


def _current_stream(arrays: List[Any]) -> int:
    for a in arrays:
        if a is None:
            continue
        if _is_torch(a):
            import torch
            return int(torch.cuda.current_stream(a.device).cuda_stream)
        mod = type(a).__module__
        if mod.startswith("cupy"):
            import cupy  # noqa: F401  (only when the caller already uses CuPy)
            return int(cupy.cuda.get_current_stream().ptr)
    return 0


def _view(arr: Any, shape) -> Any:
    n = int(np.prod(shape, dtype=np.int64)) if len(shape) else 1
    flat = arr.reshape(-1)
    return flat[:n].reshape(tuple(shape))


# Names whose second input is a small shape / size tensor read on the host
# (the reference does the same blocking read, kernel_registry.py:675).
_HOST_SECOND = {"reshape", "split", "fused_transpose_reshape_f32"}


def _make(name: str) -> KernelFunc:
    def kernel(inputs: List[Any], outputs: List[Any], params: Dict[str, Any],
               tuning: Optional[Dict[str, int]] = None) -> None:
        ins: List[Optional[Desc]] = []
        for i, x in enumerate(inputs):
            if x is None:
                ins.append(None)
                continue
            d = describe(x)
            if i == 1 and name in _HOST_SECOND:
                d.host = _host_values(x)
            ins.append(d)
        outs = [describe(o) for o in outputs]
        prep = prepare(name, ins, outs, params or {})
        stream = _current_stream(list(inputs) + list(outputs))
        for ln in prep.launches:
            L.launch(ln.kid, ln.ins, ln.outs, ln.params, stream)
        for i, shape in enumerate(prep.out_shapes):
            if i < len(outputs):
                dt = ln_out_dtype(prep, i)
                out = outputs[i]
                if dt is not None and dt != describe(out).dtype:
                    out = _retype(out, dt)
                outputs[i] = _view(out, shape)
    kernel.__name__ = f"kernel_{name}"
    kernel.__qualname__ = kernel.__name__
    return kernel


def ln_out_dtype(prep, i: int) -> Optional[int]:
    k = 0
    for ln in prep.launches:
        for t in ln.outs:
            if k == i:
                return int(t.dtype)
            k += 1
    return None


def _retype(arr: Any, dt: int) -> Any:
    """Reinterpret an arena view as another dtype (gather/split keep their data dtype)."""
    if _is_torch(arr):
        import torch
        tmap = {L.F32: torch.float32, L.BF16: torch.bfloat16, L.F16: torch.float16, L.I64: torch.int64,
                L.I32: torch.int32, L.U8: torch.uint8}
        return arr.view(tmap[dt])
    npmap = {L.F32: np.float32, L.F16: np.float16, L.I64: np.int64, L.I32: np.int32, L.U8: np.uint8}
    return arr.view(npmap[dt])


for _name in _prepared_names():
    register(_name)(_make(_name))


# ------------------------------------------------------------- fp8 precision path
#
# The reference's policy selects fp8 for aligned GEMMs (c32/strategy.py:147-157)
# and its decompositions then emit "matmul_f8" (c32/decompositions.py:18-27),
# which the reference's lookup cannot resolve.  Here the name executes:
# operands are quantised rowwise to E4M3 on the device (C3B_K_QUANT_E4M3) and
# multiplied on tcgen05 kind::f8f6f4 (C3B_K_GEMM_FP8), fp32 output.  The
# temporaries come from the caller's own array library (torch or CuPy) on the
# caller's stream.

def _scratch(like: Any, shape, np_dtype):
    if _is_torch(like):
        import torch
        tmap = {np.uint8: torch.uint8, np.float32: torch.float32, np.uint16: torch.bfloat16}
        return torch.empty(tuple(shape), dtype=tmap[np_dtype], device=like.device)
    import cupy
    return cupy.empty(tuple(shape), dtype=np_dtype)


@register("matmul_f8")
def kernel_matmul_f8(inputs: List[Any], outputs: List[Any], params: Dict[str, Any],
                     tuning: Optional[Dict[str, int]] = None) -> None:
    a, b = inputs[0], inputs[1]
    da, db = describe(a), describe(b)
    if len(da.shape) != 2 or len(db.shape) != 2:
        raise ValueError("matmul_f8: 2-D operands")
    ta, tb = int(params.get("transA", 0)), int(params.get("transB", 0))
    alpha = float(params.get("alpha", 1.0))
    M, K = (da.shape[1], da.shape[0]) if ta else da.shape
    N = db.shape[0] if tb else db.shape[1]
    if (db.shape[1] if tb else db.shape[0]) != K:
        raise ValueError("matmul_f8: inner dimensions differ")
    if K % 16 or N % 32:
        raise ValueError("matmul_f8: needs K % 16 == 0 and N % 32 == 0")
    stream = _current_stream([a, b] + list(outputs))

    def k_major(x, d, rows, cols, trans):
        # [rows, cols] K-major operand; transposed through a strided copy when needed
        if not trans:
            return d
        t = _scratch(x, (rows, cols), np.float32)
        cp = L.CopyParams()
        cp.in_offset = 0
        cp.in_stride[0], cp.in_stride[1] = 1, rows
        L.launch(L.K_COPY, [L.make_tensor(d.ptr, d.dtype, d.shape)], [L.make_tensor(int(t.data_ptr() if _is_torch(t)
                 else t.data.ptr), L.F32, (rows, cols))], cp, stream)
        keep.append(t)
        return describe(t)

    def ptr(t):
        return int(t.data_ptr()) if _is_torch(t) else int(t.data.ptr)

    keep: List[Any] = []
    A = k_major(a, da, M, K, ta)             # A^T stored [K, M] -> [M, K]
    Bk = k_major(b, db, N, K, not tb)        # B stored [K, N] -> [N, K]
    qa, sa = _scratch(a, (M, K), np.uint8), _scratch(a, (M,), np.float32)
    qb, sb = _scratch(a, (N, K), np.uint8), _scratch(a, (N,), np.float32)
    for src, q, s, rows in ((A, qa, sa, M), (Bk, qb, sb, N)):
        L.launch(L.K_QUANT_E4M3, [L.make_tensor(src.ptr, src.dtype, (rows, K))],
                 [L.make_tensor(ptr(q), L.U8, (rows, K)), L.make_tensor(ptr(s), L.F32, (rows,))],
                 L.QuantParams(rows, K), stream)
    g = L.GemmTcParams()
    g.M, g.N, g.K, g.bias_mode, g.act, g.has_residual, g.block_n = M, N, K, L.BIAS_NONE, 0, 0, 0
    do = describe(outputs[0])
    if do.numel < M * N or do.dtype != L.F32:
        raise ValueError("matmul_f8: output must be an f32 arena of at least M*N elements")
    L.launch(L.K_GEMM_FP8, [L.make_tensor(ptr(qa), L.U8, (M, K)), L.make_tensor(ptr(qb), L.U8, (N, K)),
                            L.make_tensor(ptr(sa), L.F32, (M,)), L.make_tensor(ptr(sb), L.F32, (N,))],
             [L.make_tensor(do.ptr, L.F32, (M, N))], g, stream)
    if alpha != 1.0:
        from .kernels import _ew_program
        L.launch(L.K_EW, [L.make_tensor(do.ptr, L.F32, (M * N,))], [L.make_tensor(do.ptr, L.F32, (M * N,))],
                 _ew_program([(L.OP_MUL_IMM, 0, 0)], [alpha]), stream)
    outputs[0] = _view(outputs[0], (M, N))


@register("matmul_f4")
def kernel_matmul_f4(inputs: List[Any], outputs: List[Any], params: Dict[str, Any],
                     tuning: Optional[Dict[str, int]] = None) -> None:
    """The policy's fp4 GEMM as W4A16 (c32/strategy.py:98-119): the weight
    operand (inputs[1]) is quantised to FP4 E2M1 in groups of 16 on the device
    (C3B_K_QUANT_FP4), the activations are cast to bf16, and the tcgen05 GEMM
    expands the weights next to the MMA (C3B_K_GEMM_W4A16); fp32 output."""
    a, b = inputs[0], inputs[1]
    da, db = describe(a), describe(b)
    if len(da.shape) != 2 or len(db.shape) != 2:
        raise ValueError("matmul_f4: 2-D operands")
    ta, tb = int(params.get("transA", 0)), int(params.get("transB", 0))
    if float(params.get("alpha", 1.0)) != 1.0:
        raise NotImplementedError("matmul_f4: alpha != 1")
    M, K = (da.shape[1], da.shape[0]) if ta else da.shape
    N = db.shape[0] if tb else db.shape[1]
    if (db.shape[1] if tb else db.shape[0]) != K:
        raise ValueError("matmul_f4: inner dimensions differ")
    if K % 64 or N % 32:
        raise ValueError("matmul_f4: needs K % 64 == 0 and N % 32 == 0")
    stream = _current_stream([a, b] + list(outputs))

    def ptr(t):
        return int(t.data_ptr()) if _is_torch(t) else int(t.data.ptr)

    def copy_to(src, rows, cols, trans, dtype, np_dtype):
        t = _scratch(a, (rows, cols), np_dtype)
        cp = L.CopyParams()
        if trans:
            cp.in_stride[0], cp.in_stride[1] = 1, rows
        else:
            cp.in_stride[0], cp.in_stride[1] = cols, 1
        L.launch(L.K_COPY, [L.make_tensor(src.ptr, src.dtype, src.shape)], [L.make_tensor(ptr(t), dtype, (rows, cols))],
                 cp, stream)
        return t

    abf = copy_to(da, M, K, ta, L.BF16, np.uint16)           # bf16 activations [M, K]
    bk = copy_to(db, N, K, not tb, L.F32, np.float32)        # weights [N, K]
    q, s = _scratch(a, (N, K // 2), np.uint8), _scratch(a, (K // 64, N, 4), np.float32)
    L.launch(L.K_QUANT_FP4, [L.make_tensor(ptr(bk), L.F32, (N, K))],
             [L.make_tensor(ptr(q), L.U8, (N, K // 2)), L.make_tensor(ptr(s), L.F32, (K // 64, N, 4))],
             L.QuantParams(N, K), stream)
    g = L.GemmTcParams()
    g.M, g.N, g.K, g.bias_mode, g.act, g.has_residual, g.block_n = M, N, K, L.BIAS_NONE, 0, 0, 0
    do = describe(outputs[0])
    if do.numel < M * N or do.dtype != L.F32:
        raise ValueError("matmul_f4: output must be an f32 arena of at least M*N elements")
    L.launch(L.K_GEMM_W4A16, [L.make_tensor(ptr(abf), L.BF16, (M, K)), L.make_tensor(ptr(q), L.U8, (N, K // 2)),
                              L.make_tensor(ptr(s), L.F32, (K // 64, N, 4))],
             [L.make_tensor(do.ptr, L.F32, (M, N))], g, stream)
    outputs[0] = _view(outputs[0], (M, N))
