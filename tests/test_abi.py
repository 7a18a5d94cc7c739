"""The C-ABI library: loads without a GPU, exports every declared entry point,
resolves kernel names with the reference's alias rules, and its parameter
structs have the layout the ctypes mirror assumes."""

import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from hackathon_b200 import _lib as L
from hackathon_b200 import kernels as K

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "c3b200.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(c3b_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    decl = declared_functions()
    assert len(decl) >= 20
    for name in decl:
        assert hasattr(lib, name), f"{name} declared in c3b200.h but not exported"
    assert set(L.EXPORTS) <= set(decl)
    assert lib.c3b_version() == 1


REFERENCE_NAMES = [
    "add", "add_f32", "mul", "mul_f32", "div", "div_f32", "sub", "sub_f32", "relu_f32", "erf_f32", "exp",
    "exp_f32", "sqrt", "sqrt_f32", "reciprocal", "reciprocal_f32", "reduce_max", "reduce_max_f32", "reduce_sum",
    "reduce_sum_f32", "reduce_mean", "reduce_mean_f32", "matmul_f32", "conv_reshape_f32", "add_bias_f32",
    "im2col_f32", "winograd_forward_f32", "batchnorm_f32", "fused_matmul_bias_f32", "fused_ew_f32",
    "fused_softmax_f32", "fused_residual_norm_f32", "fused_gemm_epilogue_f32", "fused_attention_scores_f32",
    "fused_layer_norm_f32", "fused_transpose_reshape_f32", "fused_residual_relu_f32", "reshape", "transpose",
    "flatten", "split", "gather", "constant",
]


def test_every_reference_kernel_name_resolves():
    """c32/kernel_registry.py:200-759 names, through both the C and Python registries."""
    from hackathon_b200 import kernel_registry as R
    for n in REFERENCE_NAMES:
        assert L.kernel_id(n) >= 0
        assert R.is_registered(n)
        K.resolve(n)
    # alias rules of c32/kernel_registry.py:42-67
    assert L.kernel_id("relu") == L.kernel_id("relu_f32")
    assert L.kernel_id("matmul_fp32") == L.K_GEMM
    assert L.kernel_id("add_fp32") == L.K_EW
    assert R.lookup("relu") is R.lookup("relu_f32")
    assert R.lookup("im2col_fp32") is R.lookup("im2col_f32")


def test_unknown_kernel_fails_closed():
    from hackathon_b200 import kernel_registry as R
    with pytest.raises(RuntimeError, match="Unknown kernel"):
        L.kernel_id("sigmoid_f32")
    with pytest.raises(RuntimeError, match="Unknown kernel"):
        R.lookup("sigmoid_f32")
    with pytest.raises(RuntimeError, match="Unknown kernel"):
        K.resolve("softplus")


STRUCTS = {
    "c3b_tensor": L.Tensor, "c3b_ew_params": L.EwParams, "c3b_copy_params": L.CopyParams,
    "c3b_conv_geom": L.ConvGeom, "c3b_reduce_params": L.ReduceParams, "c3b_gemm_params": L.GemmParams,
    "c3b_layernorm_params": L.LayerNormParams, "c3b_softmax_params": L.SoftmaxParams,
    "c3b_attn_scores_params": L.AttnScoresParams, "c3b_gather_params": L.GatherParams,
    "c3b_conv_params": L.ConvParams, "c3b_gemm_tc_params": L.GemmTcParams, "c3b_conv_tc_params": L.ConvTcParams,
    "c3b_flash_params": L.FlashParams, "c3b_embed_params": L.EmbedParams, "c3b_stem_params": L.StemParams,
    "c3b_gap_params": L.GapParams, "c3b_stem_conv_params": L.StemConvParams,
    "c3b_quant_params": L.QuantParams, "c3b_wait_probe_params": L.WaitProbeParams,
}


def test_struct_layout_matches_header():
    src = "#include <stdio.h>\n#include <stddef.h>\n#include \"c3b200.h\"\nint main(void){\n"
    for n in STRUCTS:
        src += f'printf("{n} %zu\\n", sizeof({n}));\n'
    src += 'printf("c3b_tensor.flags %zu\\n", offsetof(c3b_tensor, flags));\n'
    src += 'printf("c3b_gemm_params.alpha %zu\\n", offsetof(c3b_gemm_params, alpha));\n'
    src += 'printf("c3b_conv_params.g %zu\\n", offsetof(c3b_conv_params, g));\n'
    src += "return 0;}\n"
    with tempfile.TemporaryDirectory() as d:
        c, exe = os.path.join(d, "s.c"), os.path.join(d, "s")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    got = dict(line.split() for line in out.strip().splitlines())
    for n, cls in STRUCTS.items():
        assert int(got[n]) == ctypes.sizeof(cls), n
    assert int(got["c3b_tensor.flags"]) == L.Tensor.flags.offset
    assert int(got["c3b_gemm_params.alpha"]) == L.GemmParams.alpha.offset
    assert int(got["c3b_conv_params.g"]) == L.ConvParams.g.offset


def test_invalid_launch_reports_error_without_gpu_work():
    """Argument validation happens before any CUDA call: a bad parameter block
    size returns C3B_E_INVALID with a message."""
    with pytest.raises(RuntimeError, match="parameter block size"):
        L.launch(L.K_EW, [L.make_tensor(1, L.F32, (4,))], [L.make_tensor(1, L.F32, (4,))], L.CopyParams())


@pytest.mark.parametrize("change,match", [
    ({"has_residual": 1}, "takes no residual"),
    ({"stride": 1, "ho": 32, "wo": 32}, "stride 2, pad k/2"),
    ({"cout": 256}, "Cout 64 or 128"),
    ({"ws_shape": (128, 32)}, r"ws \[Cout, Cin\]"),
])
def test_fused_shortcut_arguments_checked_without_gpu_work(change, match):
    """C3B_K_CONV_TC with has_shortcut: the shortcut's conditions (stride 2, no
    residual, one column block of Cout 64 or 128, ws [Cout, Cin]) are checked
    before any CUDA call; the pointers are never dereferenced."""
    c = {"n": 2, "h": 32, "cin": 64, "cout": 128, "stride": 2, "ho": 16, "wo": 16, "has_residual": 0,
         "ws_shape": None}
    c.update(change)
    n, h, cin, cout, ho = c["n"], c["h"], c["cin"], c["cout"], c["ho"]
    cp = L.ConvTcParams()
    cp.n, cp.h, cp.w, cp.cin, cp.cout, cp.ho, cp.wo = n, h, h, cin, cout, ho, c["wo"]
    cp.k, cp.stride, cp.pad = 3, c["stride"], 1
    cp.has_residual, cp.act, cp.block_n, cp.mode, cp.has_shortcut = c["has_residual"], 1, 0, 0, 1
    ptr = iter(range(1 << 20, 64 << 20, 1 << 20))  # 16-byte aligned, never dereferenced
    t = lambda dt, shape: L.make_tensor(next(ptr), dt, shape)  # noqa: E731
    ins = [t(L.BF16, (n, h, h, cin)), t(L.BF16, (cout, 3, 3, cin)), t(L.F32, (cout,))]
    if c["has_residual"]:
        ins.append(t(L.BF16, (n, ho, ho, cout)))
    ins += [t(L.BF16, c["ws_shape"] or (cout, cin)), t(L.F32, (cout,))]
    outs = [t(L.BF16, (n, ho, ho, cout)), t(L.BF16, (n, ho, ho, cout))]
    with pytest.raises(RuntimeError, match=match):
        L.launch(L.K_CONV_TC, ins, outs, cp)
