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


@pytest.mark.parametrize("model", ["mlp", "resnet18", "tx_small"])
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
