"""The backend's extra C3.3 passes (hackathon_b200.c33_passes), on CPU.

The passes run on the reference IR in the container that builds the plan
fixtures; here they run on a minimal stand-in with the same interface, on
small graphs shaped like the reference pipeline's output (FusedConv2dBatchNorm
with bn_folded, FusedEWChain, FusedMatMulBias, FusedAttentionScores, ...,
c33/pipeline.py:108-119).  The committed b200 plans are checked structurally
and walked by the plan runner with a recorder (no GPU).
"""

import json
import os
from dataclasses import dataclass, field
from typing import Any, Dict, List

import numpy as np
import pytest

from hackathon_b200 import _lib as L
from hackathon_b200.c33_passes import run_b200_passes

HERE = os.path.dirname(os.path.abspath(__file__))


@dataclass
class Node:
    id: str
    name: str
    op_type: str
    inputs: List[str] = field(default_factory=list)
    outputs: List[str] = field(default_factory=list)
    attributes: Dict[str, Any] = field(default_factory=dict)
    domain: str = ""


@dataclass
class T:
    name: str


class MiniGraph:
    """The slice of the reference Graph interface the passes use."""

    def __init__(self, inputs, outputs, initializers):
        self.nodes, self.node_order = {}, []
        self.tensor_producer, self.tensor_consumers = {}, {}
        self.inputs = [T(n) for n in inputs]
        self.outputs = [T(n) for n in outputs]
        self.initializers = {n: None for n in initializers}

    def add(self, nid, op, ins, outs, **attrs):
        n = Node(nid, nid, op, list(ins), list(outs), dict(attrs))
        self.add_node(n)
        for o in outs:
            self.set_producer(o, nid)
        self.node_order.append(nid)

    def add_node(self, node):
        self.nodes[node.id] = node
        for t in node.inputs:
            if t:
                self.tensor_consumers.setdefault(t, [])
                if node.id not in self.tensor_consumers[t]:
                    self.tensor_consumers[t].append(node.id)

    def set_producer(self, t, nid):
        self.tensor_producer[t] = nid

    def remove_node(self, nid):
        n = self.nodes.pop(nid)
        for t in n.inputs:
            if t in self.tensor_consumers and nid in self.tensor_consumers[t]:
                self.tensor_consumers[t].remove(nid)
        for o in n.outputs:
            if self.tensor_producer.get(o) == nid:
                del self.tensor_producer[o]
        if nid in self.node_order:
            self.node_order.remove(nid)

    def topological_sort(self):
        done, order = set(self.initializers) | {t.name for t in self.inputs}, []
        pending = list(self.node_order)
        while pending:
            for nid in pending:
                if all(not t or t in done for t in self.nodes[nid].inputs):
                    order.append(nid)
                    done.update(self.nodes[nid].outputs)
                    pending.remove(nid)
                    break
            else:
                raise RuntimeError("cycle or missing producer")
        self.node_order = order
        return order


def _conv(g, nid, x, out, stride=1, k=3):
    g.add(nid, "FusedConv2dBatchNorm", [x, f"{nid}_w", f"{nid}_b"], [out], kernel_shape=[k, k],
          pads=[k // 2] * 4, strides=[stride, stride], dilations=[1, 1], group=1, bn_folded=True)
    g.initializers[f"{nid}_w"] = g.initializers[f"{nid}_b"] = None


def test_conv_passes_fuse_relu_and_residual_into_the_later_conv():
    g = MiniGraph(["x"], ["y"], [])
    _conv(g, "c0", "x", "a0")
    g.add("r0", "Relu", ["a0"], ["h0"])
    _conv(g, "c1", "h0", "a1")                 # block main conv (no act)
    _conv(g, "c2", "x", "a2", stride=1, k=1)   # shortcut conv, later in the order
    g.add("ew", "FusedEWChain", ["a1", "a2"], ["y"], chain_ops=["Add", "Relu"])
    res = run_b200_passes(g)
    assert res["counts"]["B200ConvBiasAct"] == 3
    ops = [g.nodes[n] for n in g.node_order]
    assert [n.op_type for n in ops] == ["B200ConvBiasAct"] * 3
    first, main, short = ops
    assert first.attributes["_activation"] == "Relu" and first.outputs == ["h0"]
    assert "_activation" not in main.attributes and main.outputs == ["a1"]
    # the residual goes into the conv that runs later (its other input is ready)
    assert short.inputs == ["x", "c2_w", "c2_b", "a1"] and short.attributes["_residual_input_index"] == 3
    assert short.outputs == ["y"] and short.attributes["kernel_shape"] == [1, 1]


def test_unfolded_batchnorm_is_left_alone():
    g = MiniGraph(["x"], ["y"], ["w", "b", "s", "t", "m", "v"])
    g.add("c", "FusedConv2dBatchNorm", ["x", "w", "b", "s", "t", "m", "v"], ["y"], kernel_shape=[3, 3])
    assert run_b200_passes(g)["counts"]["B200ConvBiasAct"] == 0


def test_linear_pass_fuses_gelu_and_residual():
    g = MiniGraph(["x"], ["z"], ["w1", "b1", "w2", "b2", "c1", "c2", "c3"])
    g.add("m1", "FusedMatMulBias", ["x", "w1", "b1"], ["h"])
    g.add("gelu", "FusedEWChain", ["h", "c1", "c2", "c3"], ["g"], chain_ops=["Div", "Erf", "Add", "Mul", "Mul"])
    g.add("m2", "FusedMatMulBias", ["g", "w2", "b2"], ["o"])
    g.add("add", "Add", ["x", "o"], ["z"])
    res = run_b200_passes(g)
    assert res["counts"]["B200LinearEpilogue"] == 2
    a, b = (g.nodes[n] for n in g.node_order)
    assert a.attributes == {"_activation": "Gelu", "_gelu_constants": ["c1", "c2", "c3"]} and a.outputs == ["g"]
    assert b.inputs == ["g", "w2", "b2", "x"] and b.attributes["_residual_input_index"] == 3 and b.outputs == ["z"]


def _attention_graph():
    g = MiniGraph(["qkv"], ["y"], ["split", "hs", "div", "mask", "ms"])
    g.add("sp", "Split", ["qkv", "split"], ["s0", "s1", "s2"], axis=-1)
    for i, perm in ((0, [0, 2, 1, 3]), (1, [0, 2, 3, 1]), (2, [0, 2, 1, 3])):
        g.add(f"r{i}", "Reshape", [f"s{i}", "hs"], [f"h{i}"])
        g.add(f"t{i}", "Transpose", [f"h{i}"], [f"p{i}"], perm=perm)
    g.add("sc", "FusedAttentionScores", ["p0", "p1", "div", "mask"], ["pr"], axis=-1)
    g.add("pv", "MatMul", ["pr", "p2"], ["o"])
    g.add("mg", "FusedTransposeReshape", ["o", "ms"], ["y"], perm=[0, 2, 1, 3])
    return g


def test_attention_pass_collapses_ten_nodes():
    g = _attention_graph()
    res = run_b200_passes(g)
    assert res["counts"]["B200FlashAttention"] == 1
    (n,) = [g.nodes[i] for i in g.node_order]
    assert n.op_type == "B200FlashAttention"
    assert n.inputs == ["qkv", "hs", "div", "mask", "ms"] and n.outputs == ["y"]
    assert n.attributes["_qkv_order"] == [0, 1, 2]


def test_attention_pass_needs_single_use_intermediates():
    g = _attention_graph()
    g.add("leak", "Relu", ["pr"], ["leak_out"])  # the score tensor is used elsewhere
    g.outputs.append(T("leak_out"))
    assert run_b200_passes(g)["counts"]["B200FlashAttention"] == 0


class _Recorder:
    def __init__(self):
        self.actions = []

    def upload(self, *a):
        pass

    def add_input_slot(self, n):
        return 0

    def add_output_slot(self, n):
        return 0

    def h2d(self, *a):
        pass

    def d2h(self, *a):
        pass

    def record(self, *a):
        pass

    def wait(self, *a):
        pass

    def kernel(self, s, ln, label=""):
        self.actions.append((label, ln))


@pytest.mark.parametrize("model,batch,profile,want", [
    ("resnet18", 4, "bf16", {L.K_CONV_TC: 19, L.K_STEM_CONV: 1, L.K_GAP_NHWC: 1, L.K_GEMM: 1}),
    ("resnet18", 4096, "bf16", {L.K_CONV_TC: 19, L.K_STEM_CONV: 1, L.K_GAP_NHWC: 1, L.K_GEMM: 1}),
    ("tx_small", 4, "bf16", {L.K_GEMM_TC: 17, L.K_FLASH_ATTN: 4, L.K_LAYERNORM: 9}),
    ("resnet18", 4, "fp16", {L.K_CONV_TC: 19, L.K_STEM_CONV: 1, L.K_GAP_NHWC: 1, L.K_GEMM: 1}),
    ("tx_small", 4, "fp16", {L.K_GEMM_TC: 17, L.K_FLASH_ATTN: 4, L.K_LAYERNORM: 9}),
])
def test_b200_plans_walk_onto_tensor_core_kernels(model, batch, profile, want):
    from hackathon_b200.c34_plan import C34PlanRunner
    from hackathon_b200.workloads import BUILDERS, make_inputs
    plan = json.load(open(os.path.join(HERE, "golden", f"plan_{model}_b{batch}_b200_{profile}.json")))
    steps = plan["kernel_steps"]
    assert all(k["precision_profile"]["compute_dtype"] == profile for k in steps if k["kernel_name"].startswith("b200"))
    g = BUILDERS[model]()
    feeds = make_inputs(g, batch)
    rec = _Recorder()
    r = C34PlanRunner(plan, g.initializers, {k: (v.shape, v.dtype) for k, v in feeds.items()}, target=rec)
    got = {}
    for _, ln in rec.actions:
        got[ln.kid] = got.get(ln.kid, 0) + 1
    for kid, n in want.items():
        assert got.get(kid, 0) == n, (L.KERNEL_NAMES[kid], got)
    t16 = L.F16 if profile == "fp16" else L.BF16
    tc_outs = [int(ln.outs[0].dtype) for _, ln in rec.actions if ln.kid in (L.K_CONV_TC, L.K_FLASH_ATTN)]
    assert tc_outs and all(d == t16 for d in tc_outs)
    # every tensor a launch touches lies inside the arena (plan arena + conversion slots)
    for _, ln in rec.actions:
        for t in list(ln.ins) + list(ln.outs):
            n = int(np.prod([t.shape[i] for i in range(t.ndim)])) if t.ndim else 1
            assert t.flags & L.TENSOR_ARENA
            assert (t.ptr or 0) + n * L.DTYPE_SIZE[t.dtype] <= r._extra_top
    # the same plan replayed in fp32 uses no tensor-core kernel
    rec32 = _Recorder()
    C34PlanRunner(plan, g.initializers, {k: (v.shape, v.dtype) for k, v in feeds.items()}, profile="fp32",
                  target=rec32)
    assert not {ln.kid for _, ln in rec32.actions} & {L.K_CONV_TC, L.K_GEMM_TC, L.K_STEM_CONV}
