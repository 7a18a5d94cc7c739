"""Per-kernel parity on the GPU, through the reference kernel ABI.

Each test calls a registry kernel exactly as the reference executor would
(``lookup(name)(inputs, outputs, params, tuning)``, c35/executor.py:576-581),
with pre-allocated float32 arena views as outputs, and compares with the
oracle restatement of the same reference kernel.  FP32 tolerance: 1e-4 relative
(max|a-b| / max|b|).  bf16 tensor-core kernels are checked against the oracle
evaluated on the same bf16-rounded operands with fp32 accumulation.
"""

import math

import numpy as np
import pytest

from oracle import ops as O
from oracle.bf16 import round_bf16

pytestmark = pytest.mark.gpu

RTOL = 1e-4


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    from hackathon_b200 import _lib
    _lib.lib()
    return torch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def arena(torch, n):
    return torch.full((int(n),), float("nan"), dtype=torch.float32, device="cuda")


def call(name, ins, outs, params):
    from hackathon_b200.kernel_registry import lookup
    lookup(name)(ins, outs, params, {"block_x": 256, "grid_x": 1, "smem_bytes": 0})
    import torch
    torch.cuda.synchronize()
    return outs


def host(t):
    return t.detach().cpu().numpy()


RNG = np.random.default_rng(1234)


def randn(*s):
    return RNG.standard_normal(s, dtype=np.float32)


def test_elementwise_family(torch_cuda):
    t = torch_cuda
    a, b = randn(2, 3, 4), randn(3, 1)
    for name, ref in [("add_f32", a + b), ("sub", a - b), ("mul_f32", a * b), ("div", a / (np.abs(b) + 0.5))]:
        bb = b if name != "div" else np.abs(b) + 0.5
        outs = call(name, [dev(t, a), dev(t, bb)], [arena(t, 64)], {})
        assert tuple(outs[0].shape) == ref.shape
        assert rel(host(outs[0]), ref) < RTOL
    x = randn(5, 7)
    for name, ref in [("relu_f32", np.maximum(x, 0)), ("erf_f32", O.erf_as(x)), ("exp", np.exp(x)),
                      ("sqrt", np.sqrt(np.abs(x))), ("reciprocal", 1.0 / (np.abs(x) + 1))]:
        xin = np.abs(x) if name == "sqrt" else (np.abs(x) + 1 if name == "reciprocal" else x)
        outs = call(name, [dev(t, xin)], [arena(t, 64)], {})
        assert rel(host(outs[0]), ref) < RTOL, name
    outs = call("add", [dev(t, x)], [arena(t, 64)], {"epsilon": 1e-3})
    assert rel(host(outs[0]), x + np.float32(1e-3)) < RTOL


def test_bias_bn_residual(torch_cuda):
    t = torch_cuda
    x, bias = randn(2, 4, 3, 3), randn(4)
    outs = call("add_bias_f32", [dev(t, x), dev(t, bias)], [arena(t, 100)], {"bias_axis": 1, "beta": 0.5})
    assert rel(host(outs[0]), x + 0.5 * bias.reshape(1, 4, 1, 1)) < RTOL
    sc, be, mu = randn(4), randn(4), randn(4)
    var = np.abs(randn(4)) + 0.5
    outs = call("batchnorm_f32", [dev(t, v) for v in (x, sc, be, mu, var)], [arena(t, 100)], {"epsilon": 1e-5})
    assert rel(host(outs[0]), O.batchnorm(x, sc, be, mu, var, 1e-5)) < RTOL
    r = randn(2, 4, 3, 3)
    outs = call("fused_residual_relu_f32", [dev(t, x), dev(t, r)], [arena(t, 100)], {})
    assert rel(host(outs[0]), np.maximum(x + r, 0)) < RTOL


def test_fused_ew_gelu_chain(torch_cuda):
    t = torch_cuda
    f = randn(8, 16)
    ops = [{"op": "Div", "inputs": [0, 1], "output": "d"}, {"op": "Erf", "inputs": ["d"], "output": "e"},
           {"op": "Add", "inputs": ["e", 2], "output": "a"}, {"op": "Mul", "inputs": [0, "a"], "output": "m"},
           {"op": "Mul", "inputs": ["m", 3], "output": "o"}]
    consts = [np.array([math.sqrt(2)], np.float32), np.array([1.0], np.float32), np.array([0.5], np.float32)]
    outs = call("fused_ew_f32", [dev(t, f)] + [dev(t, c) for c in consts], [arena(t, 200)], {"_ops": ops})
    assert rel(host(outs[0]), O.ew_chain(ops, [f] + consts)) < RTOL
    assert rel(host(outs[0]), O.gelu_erf(f)) < RTOL


def test_reductions_softmax(torch_cuda):
    t = torch_cuda
    x = randn(3, 5, 4, 6)
    outs = call("reduce_mean_f32", [dev(t, x)], [arena(t, 100)], {"axes": [-2, -1], "keepdims": True})
    assert tuple(outs[0].shape) == (3, 5, 1, 1)
    assert rel(host(outs[0]), O.global_average_pool(x)) < RTOL
    outs = call("reduce_max", [dev(t, x)], [arena(t, 100)], {"axis": 1})
    assert rel(host(outs[0]), x.max(axis=1)) < RTOL
    outs = call("reduce_sum", [dev(t, x)], [arena(t, 400)], {"axis": -1, "keepdims": True})
    assert rel(host(outs[0]), x.sum(axis=-1, keepdims=True)) < RTOL
    for axis in (-1, 1):
        outs = call("fused_softmax_f32", [dev(t, x)], [arena(t, x.size)], {"axis": axis})
        assert rel(host(outs[0]), O.softmax(x, axis)) < RTOL


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_gemm_epilogue(torch_cuda, ta, tb):
    t = torch_cuda
    M, N, K = 67, 45, 131
    a = randn(K, M) if ta else randn(M, K)
    b = randn(N, K) if tb else randn(K, N)
    for bias in (randn(N), randn(1, N), randn(M, 1), randn(M, N)):
        p = {"transA": ta, "transB": tb, "alpha": 0.7, "beta": 1.3, "_activation": "Relu"}
        outs = call("fused_gemm_epilogue_f32", [dev(t, a), dev(t, b), dev(t, bias)], [arena(t, M * N)], p)
        ref = O.gemm_epilogue(a, b, bias, alpha=0.7, beta=1.3, transA=ta, transB=tb, relu=True)
        assert rel(host(outs[0]), ref) < RTOL


def test_gemm_flatten_and_matmul_bias(torch_cuda):
    t = torch_cuda
    x, w, b = randn(6, 8, 2, 2), randn(10, 32), randn(10)
    outs = call("fused_gemm_epilogue_f32", [dev(t, x), dev(t, w), dev(t, b)], [arena(t, 60)],
                {"transB": 1, "_flatten_axis": 1})
    assert rel(host(outs[0]), O.gemm_epilogue(x, w, b, transB=1, flatten_axis=1)) < RTOL
    x3, w2, b2 = randn(3, 17, 40), randn(40, 24), randn(24)
    outs = call("fused_matmul_bias_f32", [dev(t, x3), dev(t, w2), dev(t, b2)], [arena(t, 3 * 17 * 24)], {})
    assert tuple(outs[0].shape) == (3, 17, 24)
    assert rel(host(outs[0]), O.gemm_epilogue(x3, w2, b2, matmul=True)) < RTOL


def test_matmul_batched_and_conv_contract(torch_cuda):
    t = torch_cuda
    a, b = randn(2, 3, 9, 16), randn(2, 3, 16, 5)
    outs = call("matmul_f32", [dev(t, a), dev(t, b)], [arena(t, 2 * 3 * 45)], {"lowering_kind": "matmul"})
    assert rel(host(outs[0]), np.matmul(a, b)) < RTOL
    z = np.load(_golden("registry_kat.npz"))
    outs = call("matmul_f32", [dev(t, z["im2col"]), dev(t, z["w"])], [arena(t, z["contract"].size)],
                {"lowering_kind": "conv_contract"})
    assert rel(host(outs[0]), z["contract"]) < RTOL


def _golden(name):
    import os
    return os.path.join(os.path.dirname(__file__), "golden", name)


def test_registry_conv_chain_matches_reference_kat(torch_cuda):
    """im2col -> conv_contract -> conv_reshape -> add_bias, against the outputs
    the reference registry produced on the same inputs (registry_kat.npz)."""
    t = torch_cuda
    import json
    z = np.load(_golden("registry_kat.npz"))
    p = json.loads(str(z["params"]))
    col = call("im2col_f32", [dev(t, z["x"])], [arena(t, z["im2col"].size)], p)[0]
    assert np.array_equal(host(col), z["im2col"])
    mm = call("matmul_f32", [col, dev(t, z["w"])], [arena(t, z["contract"].size)],
              {**p, "lowering_kind": "conv_contract"})[0]
    n, o, ho, wo = z["nchw"].shape
    rs = call("conv_reshape_f32", [mm], [arena(t, z["nchw"].size)], {**p, "_output_spatial": [ho, wo]})[0]
    assert rel(host(rs), z["nchw"]) < RTOL
    ob = call("add_bias_f32", [rs, dev(t, z["b"])], [arena(t, z["nchw"].size)], {"bias_axis": 1})[0]
    assert rel(host(ob), z["biased"]) < RTOL
    er = call("erf_f32", [dev(t, z["x"])], [arena(t, z["x"].size)], {})[0]
    assert np.abs(host(er) - z["erf_as"]).max() < 1e-6


@pytest.mark.parametrize("stride,k,pads", [(1, 3, [1, 1, 1, 1]), (2, 3, [1, 1, 1, 1]), (2, 1, [0, 0, 0, 0]),
                                           (1, 3, [0, 1, 2, 0])])
def test_winograd_stands_for_conv(torch_cuda, stride, k, pads):
    t = torch_cuda
    x, w = randn(2, 5, 9, 8), randn(7, 5, k, k)
    p = {"kernel_shape": [k, k], "strides": [stride, stride], "pads": pads, "dilations": [1, 1], "group": 1}
    ref = O.conv2d(x, w, None, **p)
    outs = call("winograd_forward_f32", [dev(t, x), dev(t, w)], [arena(t, ref.size)], p)
    assert tuple(outs[0].shape) == ref.shape
    assert rel(host(outs[0]), ref) < RTOL


def test_layernorm_and_residual_norm(torch_cuda):
    t = torch_cuda
    for cols in (7, 64, 256, 1024, 2000):
        x, r, g, b = randn(5, cols), randn(5, cols), randn(cols), randn(cols)
        outs = call("fused_layer_norm_f32", [dev(t, x), dev(t, g), dev(t, b)], [arena(t, x.size)],
                    {"axis": -1, "epsilon": 1e-5})
        assert rel(host(outs[0]), O.layer_norm(x, g, b)) < RTOL
        outs = call("fused_residual_norm_f32", [dev(t, x), dev(t, r), dev(t, g), dev(t, b)], [arena(t, x.size)],
                    {"axis": -1, "epsilon": 1e-5})
        assert rel(host(outs[0]), O.residual_layer_norm(x, r, g, b)) < RTOL


def test_attention_scores(torch_cuda):
    t = torch_cuda
    B, H, S, D = 2, 3, 37, 16
    q, kT = randn(B, H, S, D), randn(B, H, D, S)
    div = np.array([4.0], np.float32)
    mask = np.triu(np.full((S, S), -1e9, np.float32), 1).reshape(1, 1, S, S)
    outs = call("fused_attention_scores_f32", [dev(t, q), dev(t, kT), dev(t, div), dev(t, mask)],
                [arena(t, B * H * S * S)], {"axis": -1})
    assert rel(host(outs[0]), O.attention_scores(q, kT, div, mask)) < RTOL


def test_layout_kernels(torch_cuda):
    t = torch_cuda
    x = randn(2, 6, 4, 8)
    outs = call("transpose", [dev(t, x)], [arena(t, x.size)], {"perm": [0, 2, 1, 3]})
    assert np.array_equal(host(outs[0]), x.transpose(0, 2, 1, 3))
    outs = call("fused_transpose_reshape_f32", [dev(t, x), dev(t, np.array([0, 0, 48], np.int64))],
                [arena(t, x.size)], {"perm": [0, 2, 1, 3]})
    assert np.array_equal(host(outs[0]), x.transpose(0, 2, 1, 3).reshape(2, 4, 48))
    outs = call("reshape", [dev(t, x), dev(t, np.array([0, -1], np.int64))], [arena(t, x.size)], {})
    assert np.array_equal(host(outs[0]), x.reshape(2, -1))
    outs = call("flatten", [dev(t, x)], [arena(t, x.size)], {"axis": 2})
    assert np.array_equal(host(outs[0]), x.reshape(12, 32))
    y = randn(2, 5, 12)
    outs = call("split", [dev(t, y), dev(t, np.array([3, 4, 5], np.int64))],
                [arena(t, 100), arena(t, 100), arena(t, 100)], {"axis": -1})
    for o, r in zip(outs, O.split(y, [3, 4, 5], -1)):
        assert np.array_equal(host(o), r)
    outs = call("split", [dev(t, y)], [arena(t, 100), arena(t, 100)], {"axis": -1, "_num_outputs": 2})
    for o, r in zip(outs, O.split(y, [6, 6], -1)):
        assert np.array_equal(host(o), r)
    mm = randn(2 * 3 * 4, 5)
    outs = call("conv_reshape_f32", [dev(t, mm)], [arena(t, mm.size)], {"_batch_size": 2, "_output_spatial": [3, 4]})
    assert np.array_equal(host(outs[0]), mm.reshape(2, 3, 4, 5).transpose(0, 3, 1, 2))


def test_gather(torch_cuda):
    t = torch_cuda
    table = randn(50, 12)
    ids = RNG.integers(-50, 50, size=(3, 7)).astype(np.int64)
    outs = call("gather", [dev(t, table), dev(t, ids)], [arena(t, 3 * 7 * 12)], {"axis": 0})
    assert np.array_equal(host(outs[0]), O.gather(table, ids, 0))
    x = randn(4, 9, 6)
    outs = call("gather", [dev(t, x), dev(t, np.array([8], np.int64))], [arena(t, 24)], {"axis": 1})
    assert np.array_equal(host(outs[0]), O.gather(x, [8], 1))


def test_unknown_kernel_fails_closed(torch_cuda):
    from hackathon_b200.kernel_registry import lookup
    with pytest.raises(RuntimeError, match="Unknown kernel"):
        lookup("sigmoid_f32")


# ---------------------------------------------------------------- tensor cores

def _bf16(t, a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K,act,res", [(128, 64, 64, 0, 0), (300, 128, 192, 1, 0), (1000, 256, 512, 2, 1),
                                           (257, 96, 72, 0, 1), (4096, 512, 1024, 1, 1)])
def test_gemm_tc(torch_cuda, M, N, K, act, res):
    import torch
    from hackathon_b200 import _lib as L
    a, w, b = round_bf16(randn(M, K)), round_bf16(randn(N, K) * 0.1), randn(N)
    r = randn(M, N)
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    g = L.GemmTcParams()
    g.M, g.N, g.K, g.bias_mode, g.act, g.has_residual, g.block_n = M, N, K, L.BIAS_COL, act, res, 0
    ta, tw, tb, tr = _bf16(torch, a), _bf16(torch, w), dev(torch, b), dev(torch, r)
    ins = [L.make_tensor(ta.data_ptr(), L.BF16, (M, K)), L.make_tensor(tw.data_ptr(), L.BF16, (N, K)),
           L.make_tensor(tb.data_ptr(), L.F32, (N,))]
    if res:
        ins.append(L.make_tensor(tr.data_ptr(), L.F32, (M, N)))
    L.launch(L.K_GEMM_TC, ins, [L.make_tensor(out.data_ptr(), L.F32, (M, N))], g,
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    ref = a.astype(np.float64) @ w.astype(np.float64).T + b
    if res:
        ref = ref + r
    if act == 1:
        ref = np.maximum(ref, 0)
    elif act == 2:
        ref = O.gelu_erf(ref.astype(np.float32))
    assert rel(host(out), ref) < 2e-5


@pytest.mark.parametrize("mode", [0, 1, 2, 3])
@pytest.mark.parametrize("n,h,cin,cout,k,stride,res", [(2, 32, 64, 64, 3, 1, 0), (3, 16, 64, 128, 3, 2, 0),
                                                       (4, 16, 128, 128, 3, 1, 1), (8, 8, 128, 256, 1, 2, 0),
                                                       (10, 4, 256, 512, 3, 1, 1), (16, 8, 256, 512, 3, 2, 0),
                                                       (9, 32, 64, 64, 3, 1, 1), (3, 8, 64, 128, 3, 1, 1),
                                                       (5, 4, 128, 64, 3, 1, 0), (33, 16, 128, 128, 3, 1, 0),
                                                       (17, 32, 64, 64, 3, 1, 1), (40, 16, 64, 64, 3, 1, 0),
                                                       (16, 32, 64, 64, 3, 1, 1), (8, 16, 64, 128, 3, 2, 1),
                                                       (12, 16, 64, 128, 1, 2, 0)])
def test_conv_tc(torch_cuda, n, h, cin, cout, k, stride, res, mode):
    """mode 0: fastest eligible variant (row ring / halo); 1: one TMA window per tap; 2/3: halo tiles."""
    import torch
    from hackathon_b200 import _lib as L
    pad = k // 2
    x = round_bf16(randn(n, cin, h, h))
    w = round_bf16(randn(cout, cin, k, k) * 0.05)
    b = randn(cout)
    ref = O.conv2d(x, w, b, strides=[stride, stride], pads=[pad] * 4)
    ho = ref.shape[2]
    r = round_bf16(randn(n, cout, ho, ho)) if res else None
    if res:
        ref = np.maximum(ref + r, 0)
    xn = _bf16(torch, x.transpose(0, 2, 3, 1))
    wn = _bf16(torch, w.transpose(0, 2, 3, 1))
    tb = dev(torch, b)
    out = torch.empty((n, ho, ho, cout), dtype=torch.bfloat16, device="cuda")
    cp = L.ConvTcParams()
    cp.n, cp.h, cp.w, cp.cin, cp.cout, cp.ho, cp.wo, cp.k, cp.stride, cp.pad = n, h, h, cin, cout, ho, ho, k, stride, pad
    cp.has_residual, cp.act, cp.block_n, cp.mode = res, 1 if res else 0, 0, mode
    ins = [L.make_tensor(xn.data_ptr(), L.BF16, (n, h, h, cin)), L.make_tensor(wn.data_ptr(), L.BF16, (cout, k, k, cin)),
           L.make_tensor(tb.data_ptr(), L.F32, (cout,))]
    if res:
        rn = _bf16(torch, r.transpose(0, 2, 3, 1))
        ins.append(L.make_tensor(rn.data_ptr(), L.BF16, (n, ho, ho, cout)))
    L.launch(L.K_CONV_TC, ins, [L.make_tensor(out.data_ptr(), L.BF16, (n, ho, ho, cout))], cp,
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    got = out.float().cpu().numpy().transpose(0, 3, 1, 2)
    # bf16 output rounding: half an ulp of bf16 relative to the largest value
    assert rel(got, ref) < 8e-3


@pytest.mark.parametrize("n,h,cin,cout,k,stride,res", [(160, 32, 64, 128, 3, 2, 0), (160, 32, 64, 128, 1, 2, 1),
                                                       (300, 16, 256, 512, 1, 2, 0), (150, 16, 128, 256, 1, 2, 1)])
def test_conv_tc_resident_weights(torch_cuda, n, h, cin, cout, k, stride, res):
    """Stride-2 convolutions with at least two tiles per SM: tc_gemm_kernel
    stages the whole weight block once per CTA (one or two column blocks)."""
    test_conv_tc(torch_cuda, n, h, cin, cout, k, stride, res, 0)


@pytest.mark.parametrize("n,h,cin,cout,h16", [(8, 32, 64, 128, 0), (160, 32, 64, 128, 0), (6, 16, 128, 64, 0),
                                               (5, 8, 64, 128, 1)])
def test_conv_tc_fused_shortcut(torch_cuda, n, h, cin, cout, h16):
    """3x3 stride-2 conv + ReLU with the block's 1x1 stride-2 shortcut in the
    same launch (has_shortcut): both outputs against the oracle's two convs."""
    import torch
    from hackathon_b200 import _lib as L
    rnd = _round_f16 if h16 else round_bf16
    t16, conv = (L.F16, lambda a: _f16(torch, a)) if h16 else (L.BF16, lambda a: _bf16(torch, a))
    x = rnd(randn(n, cin, h, h))
    w = rnd(randn(cout, cin, 3, 3) * 0.05)
    ws = rnd(randn(cout, cin, 1, 1) * 0.1)
    b, bs = randn(cout), randn(cout)
    ref = np.maximum(O.conv2d(x, w, b, strides=[2, 2], pads=[1] * 4), 0)
    ref_s = O.conv2d(x, ws, bs, strides=[2, 2], pads=[0] * 4)
    ho = h // 2
    xn, wn = conv(x.transpose(0, 2, 3, 1)), conv(w.transpose(0, 2, 3, 1))
    wsn = conv(ws.reshape(cout, cin))
    tb, tbs = dev(torch, b), dev(torch, bs)
    dt = torch.float16 if h16 else torch.bfloat16
    out = torch.empty((n, ho, ho, cout), dtype=dt, device="cuda")
    out_s = torch.full((n, ho, ho, cout), float("nan"), dtype=dt, device="cuda")
    cp = L.ConvTcParams()
    cp.n, cp.h, cp.w, cp.cin, cp.cout, cp.ho, cp.wo, cp.k, cp.stride, cp.pad = n, h, h, cin, cout, ho, ho, 3, 2, 1
    cp.has_residual, cp.act, cp.block_n, cp.mode, cp.has_shortcut = 0, 1, 0, 0, 1
    ins = [L.make_tensor(xn.data_ptr(), t16, (n, h, h, cin)), L.make_tensor(wn.data_ptr(), t16, (cout, 3, 3, cin)),
           L.make_tensor(tb.data_ptr(), L.F32, (cout,)), L.make_tensor(wsn.data_ptr(), t16, (cout, cin)),
           L.make_tensor(tbs.data_ptr(), L.F32, (cout,))]
    outs = [L.make_tensor(out.data_ptr(), t16, (n, ho, ho, cout)), L.make_tensor(out_s.data_ptr(), t16, (n, ho, ho, cout))]
    L.launch(L.K_CONV_TC, ins, outs, cp, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    got = out.float().cpu().numpy().transpose(0, 3, 1, 2)
    got_s = out_s.float().cpu().numpy().transpose(0, 3, 1, 2)
    assert rel(got, ref) < 8e-3
    assert rel(got_s, ref_s) < 8e-3
    # the same shortcut as its own launch gives the same bits (one K block of
    # four MMAs either way)
    cp1 = L.ConvTcParams()
    cp1.n, cp1.h, cp1.w, cp1.cin, cp1.cout, cp1.ho, cp1.wo, cp1.k, cp1.stride, cp1.pad = n, h, h, cin, cout, ho, ho, 1, 2, 0
    cp1.has_residual, cp1.act, cp1.block_n, cp1.mode = 0, 0, 0, 0
    alone = torch.empty_like(out_s)
    L.launch(L.K_CONV_TC, [ins[0], L.make_tensor(wsn.data_ptr(), t16, (cout, 1, 1, cin)), ins[4]],
             [L.make_tensor(alone.data_ptr(), t16, (n, ho, ho, cout))], cp1, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(alone, out_s)


@pytest.mark.parametrize("shift", [0, 64])
def test_conv_tc_rowslide_residual_offsets(torch_cuda, shift):
    """Stage-1 convolution with a residual (sliding-window kernel) on operands
    at 64-byte offsets inside one arena, as the reference C3.4 plans place
    them: three launches agree bit for bit and with the reference conv.  The
    residual slots are refilled by TMA after the epilogue's generic reads; a
    missing proxy fence there showed up exactly in this configuration as rows
    read after their slot had been refilled."""
    import torch
    from hackathon_b200 import _lib as L
    n, h, c = 512, 32, 64
    x = round_bf16(randn(n, h, h, c))
    r = round_bf16(randn(n, h, h, c))
    w = round_bf16(randn(c, 3, 3, c) * 0.05)
    b = randn(c)
    nb = n * h * h * c * 2
    arena = torch.zeros(3 * nb + 8192, dtype=torch.uint8, device="cuda")
    ox, orr, oo = shift, nb + 2048 + shift, 2 * nb + 4096 + shift
    arena[ox:ox + nb].copy_(_bf16(torch, x).view(-1).view(torch.uint8))
    arena[orr:orr + nb].copy_(_bf16(torch, r).view(-1).view(torch.uint8))
    tw, tb = _bf16(torch, w), dev(torch, b)
    cp = L.ConvTcParams()
    cp.n, cp.h, cp.w, cp.cin, cp.cout, cp.ho, cp.wo, cp.k, cp.stride, cp.pad = n, h, h, c, c, h, h, 3, 1, 1
    cp.has_residual, cp.act, cp.block_n, cp.mode = 1, 1, 0, 0
    base = arena.data_ptr()
    ins = [L.make_tensor(base + ox, L.BF16, (n, h, h, c)), L.make_tensor(tw.data_ptr(), L.BF16, (c, 3, 3, c)),
           L.make_tensor(tb.data_ptr(), L.F32, (c,)), L.make_tensor(base + orr, L.BF16, (n, h, h, c))]
    outs = []
    for i in range(3):
        arena[oo:oo + nb].fill_(i + 1)
        L.launch(L.K_CONV_TC, ins, [L.make_tensor(base + oo, L.BF16, (n, h, h, c))], cp,
                 torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        outs.append(arena[oo:oo + nb].clone())
    assert L.device_status() == 0
    assert all(bool((o == outs[0]).all()) for o in outs[1:])
    got = outs[0].view(torch.bfloat16).float().cpu().numpy().reshape(n, h, h, c)[:16].transpose(0, 3, 1, 2)
    ref = np.maximum(O.conv2d(x[:16].transpose(0, 3, 1, 2), w.transpose(0, 3, 1, 2), b, strides=[1, 1],
                              pads=[1, 1, 1, 1]) + r[:16].transpose(0, 3, 1, 2), 0)
    assert rel(got, ref) < 8e-3


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("B,S,H", [(2, 128, 4), (1, 200, 2), (3, 64, 1), (2, 512, 3), (1, 384, 16)])
def test_flash_attention(torch_cuda, dt, B, S, H):
    import torch
    from hackathon_b200 import _lib as L
    D = 64
    qkv = randn(B, S, 3, H, D)
    if dt == "bf16":
        qkv = round_bf16(qkv)
    q, k, v = (qkv[:, :, i].transpose(0, 2, 1, 3) for i in range(3))
    ref = O.causal_attention(q, k, v, 1.0 / 8.0).transpose(0, 2, 1, 3).reshape(B, S, H * D)
    tq = dev(torch, qkv) if dt == "f32" else _bf16(torch, qkv)
    out = torch.empty((B, S, H * D), dtype=tq.dtype, device="cuda")
    code = L.F32 if dt == "f32" else L.BF16
    fp = L.FlashParams(B, S, H, D, 1.0 / 8.0, 1)
    L.launch(L.K_FLASH_ATTN, [L.make_tensor(tq.data_ptr(), code, (B, S, 3, H, D))],
             [L.make_tensor(out.data_ptr(), code, (B, S, H * D))], fp, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    got = out.float().cpu().numpy()
    assert rel(got, ref) < (RTOL if dt == "f32" else 2e-2)


@pytest.mark.parametrize("n,cout,act", [(3, 64, 1), (2, 32, 0), (1, 16, 1)])
def test_stem_conv_direct(torch_cuda, n, cout, act):
    """Direct small-Cin conv (NCHW f32 -> NHWC bf16) against the oracle conv."""
    import torch
    from hackathon_b200 import _lib as L
    x, w, b = randn(n, 3, 32, 32), randn(cout, 3, 3, 3) * 0.3, randn(cout)
    ref = O.conv2d(x, w, b, strides=[1, 1], pads=[1, 1, 1, 1])
    if act:
        ref = np.maximum(ref, 0)
    wk = np.ascontiguousarray(w.reshape(cout, -1).T)
    tx, tw, tb = dev(torch, x), dev(torch, wk), dev(torch, b)
    out = torch.empty((n * 1024, cout), dtype=torch.bfloat16, device="cuda")
    sp = L.StemParams()
    sp.n, sp.c, sp.h, sp.w, sp.ho, sp.wo, sp.kpad = n, 3, 32, 32, 32, 32, 0
    sp.g = L.ConvGeom(3, 3, 1, 1, 1, 1, 1, 1, 1, 1)
    L.launch(L.K_STEM_CONV, [L.make_tensor(tx.data_ptr(), L.F32, x.shape), L.make_tensor(tw.data_ptr(), L.F32, wk.shape),
                             L.make_tensor(tb.data_ptr(), L.F32, b.shape)],
             [L.make_tensor(out.data_ptr(), L.BF16, (n * 1024, cout))], L.StemConvParams(sp, cout, act),
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy().reshape(n, 32, 32, cout).transpose(0, 3, 1, 2)
    assert rel(got, ref) < 8e-3


@pytest.mark.parametrize("n,c,h", [(300, 3, 32), (7, 1, 32), (5, 2, 16), (149, 3, 32)])
def test_stem_conv_images(torch_cuda, n, c, h):
    """The whole-image stem (3x3 / stride 1 / pad 1, 32-pixel-wide images
    staged in shared memory by TMA): several images per CTA through the ring
    of image slots, fewer channels, 16-row images (4 tiles per image)."""
    import torch
    from hackathon_b200 import _lib as L
    cout = 64
    x, w, b = randn(n, c, h, 32), randn(cout, c, 3, 3) * 0.3, randn(cout)
    ref = np.maximum(O.conv2d(x, w, b, strides=[1, 1], pads=[1, 1, 1, 1]), 0)
    wk = np.ascontiguousarray(w.reshape(cout, -1).T)
    tx, tw, tb = dev(torch, x), dev(torch, wk), dev(torch, b)
    M = n * h * 32
    out = torch.empty((M, cout), dtype=torch.bfloat16, device="cuda")
    sp = L.StemParams()
    sp.n, sp.c, sp.h, sp.w, sp.ho, sp.wo, sp.kpad = n, c, h, 32, h, 32, 0
    sp.g = L.ConvGeom(3, 3, 1, 1, 1, 1, 1, 1, 1, 1)
    L.launch(L.K_STEM_CONV, [L.make_tensor(tx.data_ptr(), L.F32, x.shape), L.make_tensor(tw.data_ptr(), L.F32, wk.shape),
                             L.make_tensor(tb.data_ptr(), L.F32, b.shape)],
             [L.make_tensor(out.data_ptr(), L.BF16, (M, cout))], L.StemConvParams(sp, cout, 1),
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    got = out.float().cpu().numpy().reshape(n, h, 32, cout).transpose(0, 3, 1, 2)
    assert rel(got, ref) < 8e-3


@pytest.mark.parametrize("n,hw,c,classes,h16,bias", [(4096, 16, 512, 10, 0, 1), (37, 16, 256, 32, 1, 0),
                                                     (300, 4, 1024, 7, 0, 1)])
def test_gap_classifier(torch_cuda, n, hw, c, classes, h16, bias):
    """C3B_K_GAP_NHWC with the classifier: mean over the pixels of NHWC 16-bit
    rows, then y = mean w^T + b in fp32, in one launch."""
    import torch
    from hackathon_b200 import _lib as L
    x = randn(n, hw, c)
    x = _round_f16(x) if h16 else round_bf16(x)
    w, b = randn(classes, c) * 0.05, randn(classes)
    tx = _f16(torch, x) if h16 else _bf16(torch, x)
    tw, tb = dev(torch, w), dev(torch, b)
    out = torch.empty((n, classes), dtype=torch.float32, device="cuda")
    ins = [L.make_tensor(tx.data_ptr(), L.F16 if h16 else L.BF16, (n, hw, c)),
           L.make_tensor(tw.data_ptr(), L.F32, (classes, c))]
    if bias:
        ins.append(L.make_tensor(tb.data_ptr(), L.F32, (classes,)))
    L.launch(L.K_GAP_NHWC, ins, [L.make_tensor(out.data_ptr(), L.F32, (n, classes))], L.GapParams(n, hw, c),
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    ref = x.astype(np.float64).mean(1) @ w.astype(np.float64).T + (b if bias else 0)
    assert rel(host(out), ref) < 1e-5


def test_skinny_gemm(torch_cuda):
    """N <= 32 GEMMs take the warp-per-row path."""
    t = torch_cuda
    a, w, b = randn(300, 512), randn(10, 512), randn(10)
    outs = call("fused_gemm_epilogue_f32", [dev(t, a), dev(t, w), dev(t, b)], [arena(t, 3000)],
                {"transB": 1, "_activation": "Relu"})
    assert rel(host(outs[0]), O.gemm_epilogue(a, w, b, transB=1, relu=True)) < RTOL
    w2 = randn(512, 7)
    outs = call("fused_gemm_epilogue_f32", [dev(t, a), dev(t, w2)], [arena(t, 2100)], {"alpha": 0.5})
    assert rel(host(outs[0]), O.gemm_epilogue(a, w2, None, alpha=0.5)) < RTOL


# ------------------------------------------------------------- fp8 precision path

@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("M,K", [(37, 64), (300, 1024), (5, 4096), (129, 16)])
def test_quant_e4m3_bit_exact(torch_cuda, dt, M, K):
    """CUDA rowwise E4M3 quantiser == the oracle's restatement, byte for byte."""
    import torch
    from hackathon_b200 import _lib as L
    from oracle import fp8 as F
    x = randn(M, K) * np.float32(10.0) ** RNG.integers(-4, 3, size=(M, 1)).astype(np.float32)
    x[0] = 0.0  # an all-zero row
    if dt == "bf16":
        x = round_bf16(x)
        xd = _bf16(torch, x)
    else:
        xd = dev(torch, x)
    q = torch.empty((M, K), dtype=torch.uint8, device="cuda")
    s = torch.empty((M,), dtype=torch.float32, device="cuda")
    L.launch(L.K_QUANT_E4M3, [L.make_tensor(xd.data_ptr(), L.F32 if dt == "f32" else L.BF16, (M, K))],
             [L.make_tensor(q.data_ptr(), L.U8, (M, K)), L.make_tensor(s.data_ptr(), L.F32, (M,))],
             L.QuantParams(M, K), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    qr, sr = F.quant_rows(x)
    assert np.array_equal(host(s), sr)
    assert np.array_equal(host(q), qr)


@pytest.mark.parametrize("M,N,K,act,res,odt", [(128, 64, 64, 0, 0, "f32"), (300, 128, 192, 1, 0, "bf16"),
                                               (1000, 256, 512, 2, 1, "f32"), (257, 96, 80, 0, 1, "bf16"),
                                               (2048, 512, 1024, 1, 1, "f32")])
def test_gemm_fp8(torch_cuda, M, N, K, act, res, odt):
    """tcgen05 kind::f8f6f4 GEMM against the oracle on the same E4M3 bytes and
    scales: the products of two E4M3 values are exact in fp32, so the only
    difference is fp32 accumulation order (f32 output) or bf16 output rounding."""
    import torch
    from hackathon_b200 import _lib as L
    from oracle import fp8 as F
    a = randn(M, K)
    w = randn(N, K) * np.float32(0.05)
    qa, sa = F.quant_rows(a)
    qb, sb = F.quant_rows(w)
    bias = randn(N)
    r = randn(M, N) if res else None
    ref = F.gemm_fp8(qa, sa, qb, sb, bias)
    if res:
        ref = ref + (round_bf16(r) if odt == "bf16" else r)
    if act == 1:
        ref = np.maximum(ref, 0)
    elif act == 2:
        ref = O.gelu_erf(ref.astype(np.float32))
    g = L.GemmTcParams()
    g.M, g.N, g.K, g.bias_mode, g.act, g.has_residual, g.block_n = M, N, K, L.BIAS_COL, act, res, 0
    tq, tqb, tsa, tsb, tb = dev(torch, qa), dev(torch, qb), dev(torch, sa), dev(torch, sb), dev(torch, bias)
    ins = [L.make_tensor(tq.data_ptr(), L.U8, (M, K)), L.make_tensor(tqb.data_ptr(), L.U8, (N, K)),
           L.make_tensor(tsa.data_ptr(), L.F32, (M,)), L.make_tensor(tsb.data_ptr(), L.F32, (N,)),
           L.make_tensor(tb.data_ptr(), L.F32, (N,))]
    if res:
        tr = _bf16(torch, round_bf16(r)) if odt == "bf16" else dev(torch, r)
        ins.append(L.make_tensor(tr.data_ptr(), L.BF16 if odt == "bf16" else L.F32, (M, N)))
    out = torch.empty((M, N), dtype=torch.bfloat16 if odt == "bf16" else torch.float32, device="cuda")
    L.launch(L.K_GEMM_FP8, ins, [L.make_tensor(out.data_ptr(), L.BF16 if odt == "bf16" else L.F32, (M, N))], g,
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    got = out.float().cpu().numpy()
    assert rel(got, ref) < (8e-3 if odt == "bf16" else 2e-5)


def test_matmul_f8_registry_name(torch_cuda):
    """The reference name "matmul_f8" (which the reference's lookup cannot
    resolve) runs the fp8 path through the registry: f32 operands are
    quantised rowwise on the device and multiplied on tcgen05."""
    import torch
    from hackathon_b200.kernel_registry import lookup
    from oracle import fp8 as F
    M, K, N = 96, 128, 64
    a, b = randn(M, K), randn(K, N)
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    outs = [out]
    lookup("matmul_f8")([dev(torch, a), dev(torch, b)], outs, {"transA": 0, "transB": 0}, None)
    torch.cuda.synchronize()
    qa, sa = F.quant_rows(a)
    qb, sb = F.quant_rows(np.ascontiguousarray(b.T))
    ref = F.gemm_fp8(qa, sa, qb, sb)
    assert rel(host(outs[0]).reshape(M, N), ref) < 2e-5


# ------------------------------------------------------------- W4A16 (fp4) path

@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("N,K", [(32, 64), (200, 512), (7, 1024)])
def test_quant_fp4_bit_exact(torch_cuda, dt, N, K):
    """CUDA FP4 group quantiser == the oracle's restatement, byte for byte."""
    import torch
    from hackathon_b200 import _lib as L
    from oracle import fp4 as F
    w = randn(N, K) * np.float32(10.0) ** RNG.integers(-3, 2, size=(N, 1)).astype(np.float32)
    w[0, :16] = 0.0  # an all-zero group
    if dt == "bf16":
        w = round_bf16(w)
        wd = _bf16(torch, w)
    else:
        wd = dev(torch, w)
    q = torch.empty((N, K // 2), dtype=torch.uint8, device="cuda")
    s = torch.empty((K // 64, N, 4), dtype=torch.float32, device="cuda")
    L.launch(L.K_QUANT_FP4, [L.make_tensor(wd.data_ptr(), L.F32 if dt == "f32" else L.BF16, (N, K))],
             [L.make_tensor(q.data_ptr(), L.U8, (N, K // 2)), L.make_tensor(s.data_ptr(), L.F32, (K // 64, N, 4))],
             L.QuantParams(N, K), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    qr, sr = F.quant_groups(w)
    assert np.array_equal(host(s), sr)
    assert np.array_equal(host(q), qr)


@pytest.mark.parametrize("M,N,K,act,res,odt", [(128, 64, 64, 0, 0, "f32"), (300, 128, 192, 1, 0, "bf16"),
                                               (1000, 256, 512, 2, 1, "f32"), (257, 96, 128, 0, 1, "bf16"),
                                               (2048, 512, 1024, 1, 1, "f32")])
def test_gemm_w4a16(torch_cuda, M, N, K, act, res, odt):
    """W4A16 tcgen05 GEMM against the oracle on the same FP4 codes and scales:
    the expanded weights are exact bf16 values, so only fp32 accumulation order
    (f32 output) or bf16 output rounding separates the two."""
    import torch
    from hackathon_b200 import _lib as L
    from oracle import fp4 as F
    a = round_bf16(randn(M, K))
    w = randn(N, K) * np.float32(0.05)
    qp, qs = F.quant_groups(w)
    bias = randn(N)
    r = randn(M, N) if res else None
    ref = F.gemm_w4a16(a, qp, qs, bias)
    if res:
        ref = ref + (round_bf16(r) if odt == "bf16" else r)
    if act == 1:
        ref = np.maximum(ref, 0)
    elif act == 2:
        ref = O.gelu_erf(ref.astype(np.float32))
    g = L.GemmTcParams()
    g.M, g.N, g.K, g.bias_mode, g.act, g.has_residual, g.block_n = M, N, K, L.BIAS_COL, act, res, 0
    ta, tq, tsc, tb = _bf16(torch, a), dev(torch, qp), dev(torch, qs), dev(torch, bias)
    ins = [L.make_tensor(ta.data_ptr(), L.BF16, (M, K)), L.make_tensor(tq.data_ptr(), L.U8, (N, K // 2)),
           L.make_tensor(tsc.data_ptr(), L.F32, (K // 64, N, 4)), L.make_tensor(tb.data_ptr(), L.F32, (N,))]
    if res:
        tr = _bf16(torch, round_bf16(r)) if odt == "bf16" else dev(torch, r)
        ins.append(L.make_tensor(tr.data_ptr(), L.BF16 if odt == "bf16" else L.F32, (M, N)))
    out = torch.empty((M, N), dtype=torch.bfloat16 if odt == "bf16" else torch.float32, device="cuda")
    L.launch(L.K_GEMM_W4A16, ins, [L.make_tensor(out.data_ptr(), L.BF16 if odt == "bf16" else L.F32, (M, N))], g,
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    assert rel(out.float().cpu().numpy(), ref) < (8e-3 if odt == "bf16" else 2e-5)


def test_matmul_f4_registry_name(torch_cuda):
    """The reference name "matmul_f4" runs W4A16 through the registry: the
    weight operand is quantised on the device, activations cast to bf16."""
    import torch
    from hackathon_b200.kernel_registry import lookup
    from oracle import fp4 as F
    M, K, N = 96, 128, 64
    a, b = randn(M, K), randn(K, N)
    outs = [torch.empty((M, N), dtype=torch.float32, device="cuda")]
    lookup("matmul_f4")([dev(torch, a), dev(torch, b)], outs, {"transA": 0, "transB": 0}, None)
    torch.cuda.synchronize()
    qp, qs = F.quant_groups(np.ascontiguousarray(b.T))
    ref = F.gemm_w4a16(round_bf16(a), qp, qs)
    assert rel(host(outs[0]).reshape(M, N), ref) < 2e-5


@pytest.mark.parametrize("N,K", [(32, 64), (300, 1024)])
def test_dequant_fp4_bit_exact(torch_cuda, N, K):
    """The once-per-pass FP4 expansion gives the oracle's effective bf16 weights
    (and therefore the fused W4A16 kernel's), bit for bit."""
    import torch
    from hackathon_b200 import _lib as L
    from oracle import fp4 as F
    from oracle.bf16 import round_bf16 as rb
    w = randn(N, K) * np.float32(0.05)
    qp, qs = F.quant_groups(w)
    tq, ts = dev(torch, qp), dev(torch, qs)
    out = torch.empty((N, K), dtype=torch.bfloat16, device="cuda")
    L.launch(L.K_DEQUANT_FP4, [L.make_tensor(tq.data_ptr(), L.U8, (N, K // 2)),
                               L.make_tensor(ts.data_ptr(), L.F32, (K // 64, N, 4))],
             [L.make_tensor(out.data_ptr(), L.BF16, (N, K))], L.QuantParams(N, K),
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(out.float().cpu().numpy(), rb(F.dequant(qp, qs)))


@pytest.mark.parametrize("n,c,hw,k,stride,pad", [(3, 1, 30, 5, 2, 2), (2, 3, 31, 3, 2, 1), (5, 2, 20, 3, 1, 1)])
def test_stem_conv_geometries(torch_cuda, n, c, hw, k, stride, pad):
    """The tcgen05 stem on other geometries: 5x5 stride 2 with one channel
    (K offsets from the table), 3x3 stride 2 on odd sizes, two channels; pixel
    counts that leave a partial last 128-pixel tile."""
    import torch
    from hackathon_b200 import _lib as L
    cout = 64
    x, w, b = randn(n, c, hw, hw), randn(cout, c, k, k) * 0.3, randn(cout)
    ref = np.maximum(O.conv2d(x, w, b, strides=[stride, stride], pads=[pad] * 4), 0)
    ho = ref.shape[2]
    wk = np.ascontiguousarray(w.reshape(cout, -1).T)
    tx, tw, tb = dev(torch, x), dev(torch, wk), dev(torch, b)
    M = n * ho * ho
    out = torch.empty((M, cout), dtype=torch.bfloat16, device="cuda")
    sp = L.StemParams()
    sp.n, sp.c, sp.h, sp.w, sp.ho, sp.wo, sp.kpad = n, c, hw, hw, ho, ho, 0
    sp.g = L.ConvGeom(k, k, stride, stride, pad, pad, pad, pad, 1, 1)
    L.launch(L.K_STEM_CONV, [L.make_tensor(tx.data_ptr(), L.F32, x.shape), L.make_tensor(tw.data_ptr(), L.F32, wk.shape),
                             L.make_tensor(tb.data_ptr(), L.F32, b.shape)],
             [L.make_tensor(out.data_ptr(), L.BF16, (M, cout))], L.StemConvParams(sp, cout, 1),
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    got = out.float().cpu().numpy().reshape(n, ho, ho, cout).transpose(0, 3, 1, 2)
    assert rel(got, ref) < 8e-3


@pytest.mark.parametrize("dt,cols", [("f32", 1024), ("bf16", 256), ("f32", 2048)])
def test_layernorm_e4m3(torch_cuda, dt, cols):
    """LayerNorm writing E4M3 bytes and row scales (fp8 path) against the
    oracle LayerNorm followed by the oracle's rowwise E4M3 scheme: scales to
    fp32 rounding, values to E4M3 precision (3 mantissa bits; below 2^-6 of the
    scale, the subnormal spacing 2^-9)."""
    import torch
    from hackathon_b200 import _lib as L
    from oracle import fp8 as F
    rows = 300
    x = randn(rows, cols) * np.float32(3.0) + np.float32(0.5)
    if dt == "bf16":
        x = round_bf16(x)
    g, b = randn(cols), randn(cols) * np.float32(0.1)
    ref = O.layer_norm(x, g, b, epsilon=1e-5).astype(np.float32)
    _, sref = F.quant_rows(ref)
    xd = _bf16(torch, x) if dt == "bf16" else dev(torch, x)
    tg, tb = dev(torch, g), dev(torch, b)
    q = torch.empty((rows, cols), dtype=torch.uint8, device="cuda")
    s = torch.empty((rows,), dtype=torch.float32, device="cuda")
    L.launch(L.K_LAYERNORM, [L.make_tensor(xd.data_ptr(), L.BF16 if dt == "bf16" else L.F32, (rows, cols)),
                             L.make_tensor(tg.data_ptr(), L.F32, (cols,)), L.make_tensor(tb.data_ptr(), L.F32, (cols,))],
             [L.make_tensor(q.data_ptr(), L.U8, (rows, cols)), L.make_tensor(s.data_ptr(), L.F32, (rows,))],
             L.LayerNormParams(rows, cols, 1e-5, 0, 1, 0), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    sg = host(s)
    assert np.allclose(sg, sref, rtol=1e-5, atol=0)
    deq = F.e4m3_decode(host(q)) * sg[:, None]
    err = np.abs(deq - ref)
    assert np.all(err <= np.abs(ref) * 2.0 ** -4 + sg[:, None] * 2.0 ** -9 * 1.01)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("growth,qscale", [(1.0 / 64.0, 1.5), (1.0 / 16.0, 3.0), (1.0 / 4.0, 6.0)])
def test_flash_attention_growing_scores(torch_cuda, dt, growth, qscale):
    """Scores whose row maxima keep growing along the keys.

    Key j is scaled by 1 + growth*j, so the running maximum of a row rises tile
    after tile: the online softmax must rescale O and the row sum many times
    (the bf16 kernel rescales only when a maximum grows by more than 8 in log2
    units, so small N(0,1) scores never reach that branch after the first tile).
    With the larger setting most early keys also fall more than 126 (log2) below
    the row maximum, exercising the exponent's underflow clamp.
    """
    import torch
    from hackathon_b200 import _lib as L
    B, S, H, D = 2, 512, 2, 64
    qkv = randn(B, S, 3, H, D)
    qkv[:, :, 0] *= np.float32(qscale)
    qkv[:, :, 1] *= (np.float32(1.0) + np.float32(growth) * np.arange(S, dtype=np.float32))[None, :, None, None]
    if dt == "bf16":
        qkv = round_bf16(qkv)
    q, k, v = (qkv[:, :, i].transpose(0, 2, 1, 3) for i in range(3))
    ref = O.causal_attention(q, k, v, 1.0 / 8.0).transpose(0, 2, 1, 3).reshape(B, S, H * D)
    tq = dev(torch, qkv) if dt == "f32" else _bf16(torch, qkv)
    out = torch.empty((B, S, H * D), dtype=tq.dtype, device="cuda")
    code = L.F32 if dt == "f32" else L.BF16
    fp = L.FlashParams(B, S, H, D, 1.0 / 8.0, 1)
    L.launch(L.K_FLASH_ATTN, [L.make_tensor(tq.data_ptr(), code, (B, S, 3, H, D))],
             [L.make_tensor(out.data_ptr(), code, (B, S, H * D))], fp, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    # An fp32 score of magnitude |s| carries about eps32*|s| of absolute rounding
    # that depends on summation order, and exp() turns it into the same relative
    # error in P; at these magnitudes (up to ~1400) that exceeds RTOL, so the fp32
    # bound grows with the largest score.  bf16 keeps its 2e-2 gate.
    smax = float(np.abs(np.matmul(q, k.transpose(0, 1, 3, 2))).max()) / 8.0
    tol = max(RTOL, 4.0 * float(np.finfo(np.float32).eps) * smax)
    assert rel(got, ref) < (tol if dt == "f32" else 2e-2)


# ------------------------------------------------------------------ fp16 profile

def _f16(t, a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda().to(torch.float16)


def _round_f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("M,N,K,act,res,odt", [(128, 64, 64, 0, 0, "f32"), (300, 128, 192, 1, 1, "f16"),
                                               (1000, 256, 512, 2, 1, "f32"), (257, 96, 72, 0, 1, "f16")])
def test_gemm_tc_fp16(torch_cuda, M, N, K, act, res, odt):
    """tcgen05 kind::f16 with fp16 operands (format code 0): fp16 A and B, fp32
    accumulation, fp32 or fp16 output, fp16 residual with an fp16 output."""
    import torch
    from hackathon_b200 import _lib as L
    a, w, b = _round_f16(randn(M, K)), _round_f16(randn(N, K) * 0.1), randn(N)
    r = _round_f16(randn(M, N))
    code = L.F32 if odt == "f32" else L.F16
    out = torch.empty((M, N), dtype=torch.float32 if odt == "f32" else torch.float16, device="cuda")
    g = L.GemmTcParams()
    g.M, g.N, g.K, g.bias_mode, g.act, g.has_residual, g.block_n = M, N, K, L.BIAS_COL, act, res, 0
    ta, tw, tb = _f16(torch, a), _f16(torch, w), dev(torch, b)
    tr = _f16(torch, r) if odt == "f16" else dev(torch, r)
    ins = [L.make_tensor(ta.data_ptr(), L.F16, (M, K)), L.make_tensor(tw.data_ptr(), L.F16, (N, K)),
           L.make_tensor(tb.data_ptr(), L.F32, (N,))]
    if res:
        ins.append(L.make_tensor(tr.data_ptr(), L.F16 if odt == "f16" else L.F32, (M, N)))
    L.launch(L.K_GEMM_TC, ins, [L.make_tensor(out.data_ptr(), code, (M, N))], g,
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    ref = a.astype(np.float64) @ w.astype(np.float64).T + b
    if res:
        ref = ref + r
    if act == 1:
        ref = np.maximum(ref, 0)
    elif act == 2:
        ref = O.gelu_erf(ref.astype(np.float32))
    # fp32 output: accumulation order only; fp16 output: half an fp16 ulp
    assert rel(host(out), ref) < (2e-5 if odt == "f32" else 1e-3)


@pytest.mark.parametrize("M,N,K,odt,res,act", [(384, 256, 64, "bf16", 0, 0), (2176, 768, 1024, "bf16", 1, 2),
                                              (1000, 512, 256, "f32", 1, 1), (256, 256, 4096, "bf16", 0, 1),
                                              (640, 256, 192, "f16", 1, 0), (768, 128, 320, "bf16", 1, 0),
                                              (1280, 384, 128, "f32", 0, 1)])
def test_gemm_tc_pairs(torch_cuda, M, N, K, odt, res, act):
    """128- and 256-column tiles run on CTA pairs (tcgen05.mma.cta_group::2, M = 256 per
    pair): odd 128-row tile counts leave the second CTA of the last pair past
    M, ragged M clips inside a CTA, every output / residual format."""
    import torch
    from hackathon_b200 import _lib as L
    f16 = odt == "f16"
    rnd = _round_f16 if f16 else round_bf16
    conv = _f16 if f16 else _bf16
    code = {"bf16": L.BF16, "f16": L.F16, "f32": L.F32}[odt]
    ocode = L.F16 if f16 else L.BF16
    a, w, b = rnd(randn(M, K)), rnd(randn(N, K) * 0.1), randn(N)
    r = rnd(randn(M, N))
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[odt]
    out = torch.empty((M, N), dtype=tdt, device="cuda")
    g = L.GemmTcParams()
    g.M, g.N, g.K, g.bias_mode, g.act, g.has_residual, g.block_n = M, N, K, L.BIAS_COL, act, res, 0
    ta, tw, tb = conv(torch, a), conv(torch, w), dev(torch, b)
    tr = dev(torch, r) if odt == "f32" else conv(torch, r)
    ins = [L.make_tensor(ta.data_ptr(), ocode, (M, K)), L.make_tensor(tw.data_ptr(), ocode, (N, K)),
           L.make_tensor(tb.data_ptr(), L.F32, (N,))]
    if res:
        ins.append(L.make_tensor(tr.data_ptr(), L.F32 if odt == "f32" else ocode, (M, N)))
    L.launch(L.K_GEMM_TC, ins, [L.make_tensor(out.data_ptr(), code, (M, N))], g,
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    ref = a.astype(np.float64) @ w.astype(np.float64).T + b
    if res:
        ref = ref + r
    if act == 1:
        ref = np.maximum(ref, 0)
    elif act == 2:
        ref = O.gelu_erf(ref.astype(np.float32))
    got = out.float().cpu().numpy()
    # fp32 output: accumulation order only; 16-bit output: half an ulp of the format
    assert rel(got, ref) < {"f32": 2e-5, "f16": 1e-3, "bf16": 8e-3}[odt]


def test_gemm_tc_rejects_mixed_16bit_operands(torch_cuda):
    import torch
    from hackathon_b200 import _lib as L
    a = torch.zeros((128, 64), dtype=torch.float16, device="cuda")
    w = torch.zeros((64, 64), dtype=torch.bfloat16, device="cuda")
    out = torch.empty((128, 64), dtype=torch.float32, device="cuda")
    g = L.GemmTcParams()
    g.M, g.N, g.K = 128, 64, 64
    with pytest.raises(RuntimeError, match="both bf16 or both fp16"):
        L.launch(L.K_GEMM_TC, [L.make_tensor(a.data_ptr(), L.F16, (128, 64)), L.make_tensor(w.data_ptr(), L.BF16, (64, 64))],
                 [L.make_tensor(out.data_ptr(), L.F32, (128, 64))], g, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("n,h,cin,cout,k,stride,res", [(2, 32, 64, 64, 3, 1, 0), (3, 16, 64, 128, 3, 2, 0),
                                                       (4, 16, 128, 128, 3, 1, 1), (8, 8, 128, 256, 1, 2, 0),
                                                       (9, 32, 64, 64, 3, 1, 1)])
def test_conv_tc_fp16(torch_cuda, n, h, cin, cout, k, stride, res, mode):
    """The convolution variants (row ring, halo, per-tap windows) with fp16
    activations, weights, residual and output."""
    import torch
    from hackathon_b200 import _lib as L
    pad = k // 2
    x = _round_f16(randn(n, cin, h, h))
    w = _round_f16(randn(cout, cin, k, k) * 0.05)
    b = randn(cout)
    ref = O.conv2d(x, w, b, strides=[stride, stride], pads=[pad] * 4)
    ho = ref.shape[2]
    r = _round_f16(randn(n, cout, ho, ho)) if res else None
    if res:
        ref = np.maximum(ref + r, 0)
    xn = _f16(torch, x.transpose(0, 2, 3, 1))
    wn = _f16(torch, w.transpose(0, 2, 3, 1))
    tb = dev(torch, b)
    out = torch.empty((n, ho, ho, cout), dtype=torch.float16, device="cuda")
    cp = L.ConvTcParams()
    cp.n, cp.h, cp.w, cp.cin, cp.cout, cp.ho, cp.wo, cp.k, cp.stride, cp.pad = n, h, h, cin, cout, ho, ho, k, stride, pad
    cp.has_residual, cp.act, cp.block_n, cp.mode = res, 1 if res else 0, 0, mode
    ins = [L.make_tensor(xn.data_ptr(), L.F16, (n, h, h, cin)), L.make_tensor(wn.data_ptr(), L.F16, (cout, k, k, cin)),
           L.make_tensor(tb.data_ptr(), L.F32, (cout,))]
    if res:
        rn = _f16(torch, r.transpose(0, 2, 3, 1))
        ins.append(L.make_tensor(rn.data_ptr(), L.F16, (n, ho, ho, cout)))
    L.launch(L.K_CONV_TC, ins, [L.make_tensor(out.data_ptr(), L.F16, (n, ho, ho, cout))], cp,
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    got = out.float().cpu().numpy().transpose(0, 3, 1, 2)
    assert rel(got, ref) < 1e-3  # fp16 output rounding: half an ulp is 2^-11


@pytest.mark.parametrize("B,S,H", [(2, 128, 4), (2, 512, 3)])
def test_flash_attention_fp16(torch_cuda, B, S, H):
    import torch
    from hackathon_b200 import _lib as L
    D = 64
    qkv = _round_f16(randn(B, S, 3, H, D))
    q, k, v = (qkv[:, :, i].transpose(0, 2, 1, 3) for i in range(3))
    ref = O.causal_attention(q, k, v, 1.0 / 8.0).transpose(0, 2, 1, 3).reshape(B, S, H * D)
    tq = _f16(torch, qkv)
    out = torch.empty((B, S, H * D), dtype=torch.float16, device="cuda")
    L.launch(L.K_FLASH_ATTN, [L.make_tensor(tq.data_ptr(), L.F16, (B, S, 3, H, D))],
             [L.make_tensor(out.data_ptr(), L.F16, (B, S, H * D))], L.FlashParams(B, S, H, D, 1.0 / 8.0, 1),
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    # P is rounded to fp16 (2^-11) before P.V; the output to fp16
    assert rel(out.float().cpu().numpy(), ref) < 4e-3


@pytest.mark.parametrize("M,N,K,act,res", [(128, 64, 64, 0, 0), (300, 128, 200, 1, 1), (1000, 256, 1024, 2, 1)])
def test_gemm_tf32(torch_cuda, M, N, K, act, res):
    """kind::tf32 on fp32 operands: the inputs lose their low 13 mantissa bits,
    so the error is bounded by ~2^-10 of the dot products' magnitude."""
    import torch
    from hackathon_b200 import _lib as L
    a, w, b, r = randn(M, K), randn(N, K) * 0.1, randn(N), randn(M, N)
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    g = L.GemmTcParams()
    g.M, g.N, g.K, g.bias_mode, g.act, g.has_residual, g.block_n = M, N, K, L.BIAS_COL, act, res, 0
    ta, tw, tb, tr = dev(torch, a), dev(torch, w), dev(torch, b), dev(torch, r)
    ins = [L.make_tensor(ta.data_ptr(), L.F32, (M, K)), L.make_tensor(tw.data_ptr(), L.F32, (N, K)),
           L.make_tensor(tb.data_ptr(), L.F32, (N,))]
    if res:
        ins.append(L.make_tensor(tr.data_ptr(), L.F32, (M, N)))
    L.launch(L.K_GEMM_TF32, ins, [L.make_tensor(out.data_ptr(), L.F32, (M, N))], g,
             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    ref = a.astype(np.float64) @ w.astype(np.float64).T + b
    if res:
        ref = ref + r
    if act == 1:
        ref = np.maximum(ref, 0)
    elif act == 2:
        ref = O.gelu_erf(ref.astype(np.float32))
    err = rel(host(out), ref)
    assert 0 < err < 2e-3  # tf32, not fp32: some error must show
