"""Seeded synthetic workloads: the five graphs the C3.5 path is measured on.

Each builder returns a :class:`ModelGraph` holding the *unfused* ONNX op
sequence with opset-17 attributes, exactly as C3.1 would import it
(c31/import_onnx.py:59-240), plus seeded weights.  All randomness comes from
``numpy.random.default_rng(seed)``: weights first, in graph order, then the
inputs (``make_inputs``).  The reference publishes no asset for these
configurations, so the shapes and value distributions below are the whole
specification:

* ``mlp``      seed 0: Gemm 784->512, Relu, Gemm 512->256, Relu, Gemm 256->10.
* ``resnet18`` seed 1: CIFAR ResNet-18 with explicit BatchNormalization.
* ``tx_small`` seed 2: 4-block pre-LN decoder, d 256, 4 heads, FFN 1024,
  vocab 4096, causal seq 128.
* ``tx_large`` seed 3: 12 blocks, d 1024, 16 heads, FFN 4096, vocab 32000,
  causal seq 512.

Scalar constants are stored with shape [1] (the C3.4 scheduler gives
rank-0 initializers no arena slot).  The transformer graphs use the op forms the reference fusion passes match
(c33/fusion.py:1223-1314 for MatMul->Div->Add(mask)->Softmax,
c33/fusion.py:1317-1383 for Transpose->Reshape, the 5-op exact-erf GELU
chain of c33/fusion.py:530-560).
"""

from __future__ import annotations

import math
from typing import Dict, Tuple

import numpy as np

from .graph import ModelGraph, ValueInfo

F32 = np.float32


def _kaiming(rng: np.random.Generator, shape: Tuple[int, ...], fan_in: int) -> np.ndarray:
    return (rng.standard_normal(shape, dtype=F32) * F32(math.sqrt(2.0 / fan_in))).astype(F32)


# ---------------------------------------------------------------- MLP (C0)

def build_mlp(seed: int = 0) -> ModelGraph:
    rng = np.random.default_rng(seed)
    g = ModelGraph("mlp_seed0")
    g.inputs.append(ValueInfo("input", "float32", ["batch", 784]))
    x = "input"
    dims = [784, 512, 256, 10]
    for i in range(3):
        fin, fout = dims[i], dims[i + 1]
        w = g.init(f"fc{i}.weight", _kaiming(rng, (fout, fin), fin))
        b = g.init(f"fc{i}.bias", rng.uniform(-0.01, 0.01, (fout,)).astype(F32))
        last = i == 2
        x = g.add("Gemm", [x, w, b], out_names=["logits"] if last else None,
                  alpha=1.0, beta=1.0, transA=0, transB=1)
        if not last:
            x = g.add("Relu", [x])
    g.outputs.append(ValueInfo("logits", "float32", ["batch", 10]))
    g.meta.update(kind="mlp", in_shape=(784,), classes=10)
    return g


# ---------------------------------------------------------- ResNet-18 (C1/C3)

def _conv_bn(g: ModelGraph, rng: np.random.Generator, x: str, cin: int, cout: int,
             k: int, stride: int, tag: str) -> str:
    w = g.init(f"{tag}.conv.weight", _kaiming(rng, (cout, cin, k, k), cin * k * k))
    gamma = g.init(f"{tag}.bn.weight", rng.uniform(0.8, 1.2, (cout,)).astype(F32))
    beta = g.init(f"{tag}.bn.bias", (rng.standard_normal((cout,), dtype=F32) * F32(0.05)).astype(F32))
    mean = g.init(f"{tag}.bn.running_mean", (rng.standard_normal((cout,), dtype=F32) * F32(0.1)).astype(F32))
    var = g.init(f"{tag}.bn.running_var", rng.uniform(0.5, 1.5, (cout,)).astype(F32))
    pad = k // 2
    y = g.add("Conv", [x, w], kernel_shape=[k, k], pads=[pad, pad, pad, pad],
              strides=[stride, stride], dilations=[1, 1], group=1)
    return g.add("BatchNormalization", [y, gamma, beta, mean, var], epsilon=1e-5)


def build_resnet18(seed: int = 1) -> ModelGraph:
    rng = np.random.default_rng(seed)
    g = ModelGraph(f"resnet18_seed{seed}")
    g.inputs.append(ValueInfo("input", "float32", ["batch", 3, 32, 32]))
    x = _conv_bn(g, rng, "input", 3, 64, 3, 1, "stem")
    x = g.add("Relu", [x])
    cin = 64
    for stage, width in enumerate([64, 128, 256, 512]):
        for blk in range(2):
            stride = 2 if (stage > 0 and blk == 0) else 1
            tag = f"layer{stage + 1}.{blk}"
            y = _conv_bn(g, rng, x, cin, width, 3, stride, tag + ".a")
            y = g.add("Relu", [y])
            y = _conv_bn(g, rng, y, width, width, 3, 1, tag + ".b")
            if stride != 1 or cin != width:
                sc = _conv_bn(g, rng, x, cin, width, 1, stride, tag + ".down")
            else:
                sc = x
            y = g.add("Add", [y, sc])
            x = g.add("Relu", [y])
            cin = width
    x = g.add("GlobalAveragePool", [x])
    x = g.add("Flatten", [x], axis=1)
    w = g.init("fc.weight", _kaiming(rng, (10, 512), 512))
    b = g.init("fc.bias", rng.uniform(-0.01, 0.01, (10,)).astype(F32))
    g.add("Gemm", [x, w, b], out_names=["logits"], alpha=1.0, beta=1.0, transA=0, transB=1)
    g.outputs.append(ValueInfo("logits", "float32", ["batch", 10]))
    g.meta.update(kind="resnet18", in_shape=(3, 32, 32), classes=10)
    return g


# ------------------------------------------------------- Transformer (C2/C4)

TX_SMALL = dict(seed=2, d_model=256, layers=4, heads=4, ffn=1024, vocab=4096, seq=128)
TX_LARGE = dict(seed=3, d_model=1024, layers=12, heads=16, ffn=4096, vocab=32000, seq=512)


def build_transformer(seed: int, d_model: int, layers: int, heads: int, ffn: int,
                      vocab: int, seq: int, name: str | None = None) -> ModelGraph:
    rng = np.random.default_rng(seed)
    d, hd = d_model, d_model // heads
    g = ModelGraph(name or f"transformer_d{d}_l{layers}_seed{seed}")
    g.inputs.append(ValueInfo("input_ids", "int64", ["batch", seq]))

    def normal(shape):
        return (rng.standard_normal(shape, dtype=F32) * F32(0.02)).astype(F32)

    tok = g.init("tok_emb", normal((vocab, d)))
    pos = g.init("pos_emb", normal((seq, d)))
    mask = np.triu(np.full((seq, seq), -1e9, dtype=F32), k=1).reshape(1, 1, seq, seq)
    g.init("causal_mask", mask)
    g.init("attn_divisor", np.array([math.sqrt(hd)], dtype=F32))
    g.init("qkv_split", np.array([d, d, d], dtype=np.int64))
    g.init("heads_shape", np.array([0, 0, heads, hd], dtype=np.int64))
    g.init("merge_shape", np.array([0, 0, d], dtype=np.int64))
    g.init("gelu_sqrt2", np.array([math.sqrt(2.0)], dtype=F32))
    g.init("gelu_one", np.array([1.0], dtype=F32))
    g.init("gelu_half", np.array([0.5], dtype=F32))
    g.init("last_index", np.array([seq - 1], dtype=np.int64))

    x = g.add("Gather", [tok, "input_ids"], axis=0)
    x = g.add("Add", [x, pos])
    for layer in range(layers):
        p = f"h{layer}"
        ln1_g = g.init(f"{p}.ln1.weight", np.ones((d,), F32))
        ln1_b = g.init(f"{p}.ln1.bias", np.zeros((d,), F32))
        wqkv = g.init(f"{p}.attn.qkv.weight", normal((d, 3 * d)))
        bqkv = g.init(f"{p}.attn.qkv.bias", normal((3 * d,)))
        wo = g.init(f"{p}.attn.out.weight", normal((d, d)))
        bo = g.init(f"{p}.attn.out.bias", normal((d,)))
        ln2_g = g.init(f"{p}.ln2.weight", np.ones((d,), F32))
        ln2_b = g.init(f"{p}.ln2.bias", np.zeros((d,), F32))
        w1 = g.init(f"{p}.ffn.fc1.weight", normal((d, ffn)))
        b1 = g.init(f"{p}.ffn.fc1.bias", normal((ffn,)))
        w2 = g.init(f"{p}.ffn.fc2.weight", normal((ffn, d)))
        b2 = g.init(f"{p}.ffn.fc2.bias", normal((d,)))

        h = g.add("LayerNormalization", [x, ln1_g, ln1_b], axis=-1, epsilon=1e-5)
        qkv = g.add("MatMul", [h, wqkv])
        qkv = g.add("Add", [qkv, bqkv])
        q, k, v = g.add("Split", [qkv, "qkv_split"], n_out=3, axis=-1)
        q = g.add("Transpose", [g.add("Reshape", [q, "heads_shape"])], perm=[0, 2, 1, 3])
        k = g.add("Transpose", [g.add("Reshape", [k, "heads_shape"])], perm=[0, 2, 3, 1])
        v = g.add("Transpose", [g.add("Reshape", [v, "heads_shape"])], perm=[0, 2, 1, 3])
        s = g.add("MatMul", [q, k])
        s = g.add("Div", [s, "attn_divisor"])
        s = g.add("Add", [s, "causal_mask"])
        s = g.add("Softmax", [s], axis=-1)
        o = g.add("MatMul", [s, v])
        o = g.add("Transpose", [o], perm=[0, 2, 1, 3])
        o = g.add("Reshape", [o, "merge_shape"])
        a = g.add("MatMul", [o, wo])
        a = g.add("Add", [a, bo])
        x = g.add("Add", [x, a])
        h = g.add("LayerNormalization", [x, ln2_g, ln2_b], axis=-1, epsilon=1e-5)
        f = g.add("MatMul", [h, w1])
        f = g.add("Add", [f, b1])
        t = g.add("Div", [f, "gelu_sqrt2"])
        t = g.add("Erf", [t])
        t = g.add("Add", [t, "gelu_one"])
        t = g.add("Mul", [f, t])
        t = g.add("Mul", [t, "gelu_half"])
        f = g.add("MatMul", [t, w2])
        f = g.add("Add", [f, b2])
        x = g.add("Add", [x, f])
    lnf_g = g.init("ln_f.weight", np.ones((d,), F32))
    lnf_b = g.init("ln_f.bias", np.zeros((d,), F32))
    x = g.add("LayerNormalization", [x, lnf_g, lnf_b], axis=-1, epsilon=1e-5)
    last = g.add("Gather", [x, "last_index"], axis=1)   # [B,1,d]
    last = g.add("Flatten", [last], axis=1)              # [B,d]
    wl = g.init("lm_head.weight", normal((d, vocab)))
    bl = g.init("lm_head.bias", normal((vocab,)))
    y = g.add("MatMul", [last, wl])
    g.add("Add", [y, bl], out_names=["logits"])
    g.outputs.append(ValueInfo("logits", "float32", ["batch", vocab]))
    g.meta.update(kind="transformer", d_model=d, layers=layers, heads=heads,
                  head_dim=hd, ffn=ffn, vocab=vocab, seq=seq)
    return g


def build_tx_small() -> ModelGraph:
    return build_transformer(name="tx_small_seed2", **TX_SMALL)


def build_tx_large() -> ModelGraph:
    return build_transformer(name="tx_large_seed3", **TX_LARGE)


BUILDERS = {
    "mlp": build_mlp,
    "resnet18": build_resnet18,
    "tx_small": build_tx_small,
    "tx_large": build_tx_large,
}


def make_inputs(graph: ModelGraph, batch: int, seed: int | None = None) -> Dict[str, np.ndarray]:
    """Seeded inputs (``seed`` defaults to the model's seed)."""
    if seed is None:
        seed = {"mlp": 0, "resnet18": 1}.get(graph.meta["kind"], None)
        if seed is None:
            seed = 2 if graph.meta.get("d_model") == 256 else 3
    # Inputs use their own stream derived from the seed, so a batch shard is
    # always a slice of the same global input whatever the batch size.
    rng = np.random.default_rng([seed, 0x1A2B])
    feeds: Dict[str, np.ndarray] = {}
    for vi in graph.inputs:
        shape = tuple(batch if isinstance(d, str) else d for d in vi.shape)
        if vi.dtype == "int64":
            feeds[vi.name] = rng.integers(0, graph.meta["vocab"], size=shape, dtype=np.int64)
        else:
            feeds[vi.name] = rng.standard_normal(shape, dtype=F32)
    return feeds
