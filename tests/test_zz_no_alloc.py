"""The allocation-free stem convolution (c3b_stem_conv_noalloc).

It serves callers that may not allocate device memory themselves; its patch
matrix lives in a fixed array inside the library.  Its results must match the
regular two-launch stem path (stem_im2col + tcgen05 GEMM into a caller-owned
patch matrix) on consecutive calls, so a call never sees the previous call's
scratch contents.  Collected last on purpose (file name), and self-contained so
it also passes alone in a fresh process.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _setup():
    import torch
    from hackathon_b200 import _lib as L
    lib = L.lib()
    T = C.POINTER(L.Tensor)
    lib.c3b_stem_conv_noalloc.argtypes = [T, T, T, T, C.POINTER(L.StemParams), C.c_int, C.c_void_p]
    return torch, L, lib


def _params(L, n):
    p = L.StemParams()
    p.n, p.c, p.h, p.w, p.ho, p.wo, p.kpad = n, 3, 32, 32, 32, 32, 64
    p.g = L.ConvGeom(3, 3, 1, 1, 1, 1, 1, 1, 1, 1)
    return p


def _reference_path(torch, L, x, w, b, p, act):
    M = p.n * p.ho * p.wo
    cols = torch.empty((M, p.kpad), dtype=torch.bfloat16, device="cuda")
    out = torch.empty((M, w.shape[0]), dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    L.launch(L.K_STEM_IM2COL, [L.make_tensor(x.data_ptr(), L.F32, tuple(x.shape))],
             [L.make_tensor(cols.data_ptr(), L.BF16, (M, p.kpad))], p, s)
    g = L.GemmTcParams()
    g.M, g.N, g.K, g.bias_mode, g.act, g.has_residual, g.block_n = M, w.shape[0], p.kpad, L.BIAS_COL, act, 0, 0
    L.launch(L.K_GEMM_TC, [L.make_tensor(cols.data_ptr(), L.BF16, (M, p.kpad)),
                           L.make_tensor(w.data_ptr(), L.BF16, tuple(w.shape)),
                           L.make_tensor(b.data_ptr(), L.F32, tuple(b.shape))],
             [L.make_tensor(out.data_ptr(), L.BF16, (M, w.shape[0]))], g, s)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def _noalloc(torch, L, lib, x, w, b, p, act):
    M = p.n * p.ho * p.wo
    out = torch.full((M, w.shape[0]), float("nan"), dtype=torch.bfloat16, device="cuda")
    tx = L.make_tensor(x.data_ptr(), L.F32, tuple(x.shape))
    tw = L.make_tensor(w.data_ptr(), L.BF16, tuple(w.shape))
    tb = L.make_tensor(b.data_ptr(), L.F32, tuple(b.shape))
    to = L.make_tensor(out.data_ptr(), L.BF16, (M, w.shape[0]))
    rc = lib.c3b_stem_conv_noalloc(C.byref(tx), C.byref(tw), C.byref(tb), C.byref(to), C.byref(p), act,
                                   C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, L.last_error()
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def _oracle_conv(x, w_bf16, b, act):
    """The stem convolution on the CPU from the same bf16-rounded operands:
    NCHW conv (oracle.ops.conv2d, c35/engine.py Conv) with the weights
    unpacked from the [Cout, kpad] (r, s, c)-ordered patch layout."""
    from oracle import ops as O
    from oracle.bf16 import round_bf16
    wk = w_bf16[:, :27].reshape(-1, 3, 3, 3).transpose(0, 3, 1, 2)  # [Cout, c, r, s]
    y = O.conv2d(round_bf16(x), np.ascontiguousarray(wk), b, strides=[1, 1], pads=[1, 1, 1, 1],
                 dilations=[1, 1])
    y = y.transpose(0, 2, 3, 1).reshape(-1, w_bf16.shape[0])
    return np.maximum(y, 0) if act == 1 else y


def test_noalloc_stem_matches_regular_path_on_consecutive_calls():
    torch, L, lib = _setup()
    rng = np.random.default_rng(99)
    w = torch.from_numpy(rng.standard_normal((64, 64), dtype=np.float32) * 0.2).cuda().to(torch.bfloat16)
    b = torch.from_numpy(rng.standard_normal(64, dtype=np.float32)).cuda()
    for n, act in ((16, L.ACT_RELU), (5, L.ACT_NONE)):  # second call is smaller: stale rows must not matter
        p = _params(L, n)
        x = torch.from_numpy(rng.standard_normal((n, 3, 32, 32), dtype=np.float32)).cuda()
        ref = _reference_path(torch, L, x, w, b, p, act)
        got = _noalloc(torch, L, lib, x, w, b, p, act)
        assert np.isfinite(got).all()
        # same kernels on the same operands: bit-identical to the regular path
        assert np.array_equal(got, ref)
        # and the convolution itself, against the CPU oracle on the same bf16
        # operands (fp32 accumulation-order differences plus the bf16 output
        # rounding: within 2^-8 of each value's magnitude, plus a tiny floor)
        want = _oracle_conv(x.cpu().numpy(), w.float().cpu().numpy(), b.cpu().numpy(), act)
        assert np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -8 + 1e-3)
    assert L.device_status() == 0


def test_noalloc_stem_rejected_call_launches_nothing():
    """A call with an invalid weight tensor fails before queuing any work: the
    output stays untouched and the next valid call is still exact."""
    torch, L, lib = _setup()
    rng = np.random.default_rng(5)
    n = 4
    p = _params(L, n)
    x = torch.from_numpy(rng.standard_normal((n, 3, 32, 32), dtype=np.float32)).cuda()
    w = torch.from_numpy(rng.standard_normal((64, 64), dtype=np.float32) * 0.2).cuda().to(torch.bfloat16)
    b = torch.from_numpy(rng.standard_normal(64, dtype=np.float32)).cuda()
    M = n * 1024
    out = torch.full((M, 64), 7.0, dtype=torch.bfloat16, device="cuda")
    bad_w = torch.zeros((48, 64), dtype=torch.bfloat16, device="cuda")  # Cout not a multiple of 32
    tx = L.make_tensor(x.data_ptr(), L.F32, tuple(x.shape))
    tb = L.make_tensor(b.data_ptr(), L.F32, (64,))
    to = L.make_tensor(out.data_ptr(), L.BF16, (M, 64))
    for tw in (L.make_tensor(bad_w.data_ptr(), L.BF16, (48, 64)),          # bad Cout
               L.make_tensor(w.data_ptr(), L.F32, (64, 64))):              # wrong dtype
        rc = lib.c3b_stem_conv_noalloc(C.byref(tx), C.byref(tw), C.byref(tb), C.byref(to), C.byref(p), 1,
                                       C.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc != 0 and "stem_conv_noalloc" in L.last_error()
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
    ref = _reference_path(torch, L, x, w, b, p, L.ACT_RELU)
    assert np.array_equal(_noalloc(torch, L, lib, x, w, b, p, L.ACT_RELU), ref)


def test_noalloc_stem_rejects_oversized_batches():
    torch, L, lib = _setup()
    p = _params(L, 129)  # 129 * 1024 * 64 * 2 bytes > 16 MiB
    x = torch.zeros((129, 3, 32, 32), dtype=torch.float32, device="cuda")
    w = torch.zeros((64, 64), dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(64, dtype=torch.float32, device="cuda")
    out = torch.zeros((129 * 1024, 64), dtype=torch.bfloat16, device="cuda")
    tx = L.make_tensor(x.data_ptr(), L.F32, tuple(x.shape))
    tw = L.make_tensor(w.data_ptr(), L.BF16, (64, 64))
    tb = L.make_tensor(b.data_ptr(), L.F32, (64,))
    to = L.make_tensor(out.data_ptr(), L.BF16, (129 * 1024, 64))
    rc = lib.c3b_stem_conv_noalloc(C.byref(tx), C.byref(tw), C.byref(tb), C.byref(to), C.byref(p), 0, None)
    assert rc == -1
    assert "fixed scratch" in L.last_error()
