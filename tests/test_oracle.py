"""The CPU oracle against the reference's own outputs (golden fixtures).

tests/golden/engine_*.npz hold logits the reference's engine ops produced on
the seeded workloads (tests/golden/make_golden.py); registry_kat.npz holds the
reference registry's im2col / conv_contract / conv_reshape / add_bias / erf
outputs on fixed inputs.
"""

import json
import os

import numpy as np
import pytest

from hackathon_b200.workloads import BUILDERS, make_inputs
from oracle import ops as O
from oracle.evaluate import run_graph

HERE = os.path.dirname(os.path.abspath(__file__))


def _gold(name):
    return np.load(os.path.join(HERE, "golden", name))


@pytest.mark.parametrize("model", ["mlp", "resnet18", "tx_small", "tx_large"])
def test_oracle_matches_reference_engine(model):
    z = _gold(f"engine_{model}.npz")
    g = BUILDERS[model]()
    feeds = make_inputs(g, int(z["batch"]))
    for k, v in feeds.items():
        assert np.array_equal(v, z[k]), "seeded inputs drifted from the fixture"
    out = run_graph(g, feeds)["logits"]
    ref = z["logits"]
    assert out.shape == ref.shape
    assert np.abs(out - ref).max() / np.abs(ref).max() < 1e-5


def test_registry_known_answers():
    z = _gold("registry_kat.npz")
    p = json.loads(str(z["params"]))
    col = O.im2col(z["x"], p["kernel_shape"], p["strides"], p["pads"], p["dilations"])
    assert np.array_equal(col, z["im2col"])
    contract = col @ z["w"].reshape(z["w"].shape[0], -1).T
    assert np.abs(contract - z["contract"]).max() < 1e-5
    conv = O.conv2d(z["x"], z["w"], z["b"], strides=p["strides"], pads=p["pads"], dilations=p["dilations"])
    assert np.abs(conv - z["biased"]).max() < 1e-5
    assert np.abs(O.erf_as(z["x"]) - z["erf_as"]).max() < 1e-7


def test_oracle_fused_restatements_agree_with_unfused():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 5, 16), dtype=np.float32)
    r = rng.standard_normal((3, 5, 16), dtype=np.float32)
    g, b = rng.standard_normal(16, dtype=np.float32), rng.standard_normal(16, dtype=np.float32)
    assert np.allclose(O.residual_layer_norm(x, r, g, b), O.layer_norm(x + r, g, b), atol=1e-6)
    q = rng.standard_normal((2, 2, 9, 8), dtype=np.float32)
    k = rng.standard_normal((2, 2, 9, 8), dtype=np.float32)
    v = rng.standard_normal((2, 2, 9, 8), dtype=np.float32)
    mask = np.triu(np.full((9, 9), -1e9, np.float32), 1)[None, None]
    p = O.attention_scores(q, k.transpose(0, 1, 3, 2), np.array([np.sqrt(8)], np.float32), mask)
    assert np.allclose(p @ v, O.causal_attention(q, k, v, 1 / np.sqrt(8)), atol=1e-5)
    a = rng.standard_normal((7, 5), dtype=np.float32)
    w = rng.standard_normal((4, 5), dtype=np.float32)
    assert np.allclose(O.gemm_epilogue(a, w, np.ones(4, np.float32), transB=1, relu=True),
                       np.maximum(a @ w.T + 1, 0), atol=1e-5)
    wf, bf = O.fold_conv_bn(np.ones((2, 1, 1, 1), np.float32), np.array([2., 2.], np.float32),
                            np.array([1., 0.], np.float32), np.array([0.5, 0.], np.float32),
                            np.array([3., 3.], np.float32), epsilon=1.0)
    assert np.allclose(wf.reshape(-1), [1.0, 1.0]) and np.allclose(bf, [0.5, 0.0])


def test_erf_approximation_error_bound():
    x = np.linspace(-4, 4, 4001, dtype=np.float32)
    assert np.abs(O.erf_as(x) - O.erf_exact(x)).max() < 2e-6  # A&S 7.1.26 bound 1.5e-7 + fp32 rounding


def test_e4m3_encoder_pinned():
    """The fp8 oracle's E4M3 encoder against the OCP E4M3 code points and against
    torch's float8_e4m3fn conversion (round to nearest even), exact ties included."""
    import torch
    from oracle import fp8 as F
    points = {0.0: 0x00, 1.0: 0x38, 2.0: 0x40, 448.0: 0x7E, 2.0 ** -6: 0x08, 2.0 ** -9: 0x01, -2.0: 0xC0,
              0.5: 0x30, 1.125: 0x39, 240.0: 0x77, 7 * 2.0 ** -9: 0x07, 1000.0: 0x7E, -1e6: 0xFE}
    for v, b in points.items():
        assert int(F.e4m3_encode(np.float32(v))) == b, v
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-3, 0.05, 1.0, 30.0, 200.0)])
    vals = F.e4m3_decode(np.arange(256, dtype=np.uint8))
    vals = np.unique(vals[np.isfinite(vals)])
    mids = ((vals[1:] + vals[:-1]) / 2).astype(np.float32)  # exact ties
    x = np.clip(np.concatenate([x, mids, -mids]), -448, 448).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(F.e4m3_encode(x), ref)
    # decode(encode(v)) == v for every finite code
    codes = np.arange(256, dtype=np.uint8)
    fin = np.isfinite(F.e4m3_decode(codes))
    assert np.array_equal(F.e4m3_encode(F.e4m3_decode(codes[fin]).astype(np.float32)), codes[fin])


def test_fp8_rowwise_scheme():
    from oracle import fp8 as F
    rng = np.random.default_rng(1)
    x = rng.standard_normal((7, 64)).astype(np.float32) * np.array([1e-4, 1, 10, 100, 0, 3, 1e3], np.float32)[:, None]
    q, s = F.quant_rows(x)
    assert s[4] == 1.0 and not F.e4m3_decode(q[4]).any()  # all-zero row (signed zeros keep their sign bit)
    d = F.e4m3_decode(q) * s[:, None]
    rows = [i for i in range(7) if i != 4]
    # E4M3 keeps 3 mantissa bits: relative error <= 2^-4 for normal values
    big = np.abs(x) > np.max(np.abs(x), axis=1, keepdims=True) * 2.0 ** -6 * 1.01
    assert np.all(np.abs(d - x)[rows][big[rows]] <= np.abs(x)[rows][big[rows]] * 2.0 ** -4 + 1e-30)
    assert np.max(np.abs(q[rows].astype(np.int64) & 0x7F)) == 0x7E  # the row maximum maps to 448


def test_e2m1_encoder_pinned():
    """The fp4 oracle's E2M1 encoder against the OCP E2M1 code points (every
    magnitude, every tie between neighbours, saturation, sign) and the
    package's host quantiser against the oracle's scheme, byte for byte."""
    from oracle import fp4 as F
    from hackathon_b200.fp4 import quant_groups_fp4
    points = {0.0: 0, 0.5: 1, 1.0: 2, 1.5: 3, 2.0: 4, 3.0: 5, 4.0: 6, 6.0: 7,
              0.25: 0, 0.75: 2, 1.25: 2, 1.75: 4, 2.5: 4, 3.5: 6, 5.0: 6,  # ties -> even code
              0.26: 1, 5.01: 7, 7.0: 7, 1e9: 7, -1.0: 10, -6.0: 15, -0.6: 9}
    for v, c in points.items():
        assert int(F.e2m1_encode(np.float32(v))) == c, v
    codes = np.arange(16, dtype=np.uint8)
    assert np.array_equal(F.e2m1_encode(F.e2m1_decode(codes).astype(np.float32))[1:], codes[1:])
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((64, 320)) * rng.choice([1e-3, 1.0, 40.0], (64, 1))).astype(np.float32)[:, :256]
    w[5, 16:32] = 0.0
    p1, s1 = F.quant_groups(w)
    p2, s2 = quant_groups_fp4(w)
    assert np.array_equal(p1, p2) and np.array_equal(s1, s2)
    d = F.dequant(p1, s1)
    # E2M1 spacing is at most 2 (between 4 and 6) of a scale of group-max / 6
    gmax = np.max(np.abs(w.reshape(64, 16, 16)), axis=2).repeat(16, axis=1)
    assert np.all(np.abs(d - w) <= gmax / 6.0 + np.abs(w) * 2.0 ** -8 + 1e-30)
