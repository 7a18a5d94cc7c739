"""Host logic: the backend lowering, the arena planner and the reference-plan
adapter, exercised without a GPU (launch records are built but not run)."""

import json
import os

import numpy as np
import pytest

from hackathon_b200 import _lib as L
from hackathon_b200.c34_plan import C34PlanRunner, _DryPlan, fold_weights
from hackathon_b200.lowering import bf16_bits, bf16_to_f32, lower
from hackathon_b200.workloads import BUILDERS, make_inputs
from oracle.bf16 import round_bf16

HERE = os.path.dirname(os.path.abspath(__file__))


def _launches(prog):
    d = {n: prog.desc(n) for n in prog.tensors}
    return [ln for s in prog.steps for ln in s.build(d)]


def _check_arena(prog):
    """No two tensors whose lifetimes overlap share arena bytes."""
    first, last = {}, {}
    for n in prog.inputs:
        first[n] = -1
    for i, s in enumerate(prog.steps):
        for t in s.inputs + s.outputs:
            first.setdefault(t, i)
            last[t] = i
    for n in prog.outputs + prog.inputs:
        last[n] = len(prog.steps)
    acts = [t for t in prog.tensors.values() if t.kind != "weight"]
    for t in prog.tensors.values():
        assert t.offset >= 0 and t.offset % 256 == 0
        assert t.offset + t.nbytes <= prog.arena_bytes
    for i, a in enumerate(acts):
        for b in acts[i + 1:]:
            live = not (last[a.name] < first[b.name] or last[b.name] < first[a.name])
            if live:
                assert a.offset + a.nbytes <= b.offset or b.offset + b.nbytes <= a.offset, (a.name, b.name)
    for w in prog.tensors.values():
        if w.kind == "weight":
            assert w.offset + w.nbytes <= prog.weight_bytes


@pytest.mark.parametrize("model,batch,profile,kinds", [
    ("mlp", 256, "fp32", {L.K_GEMM: 3}),
    ("resnet18", 64, "fp32", {L.K_CONV: 20, L.K_REDUCE: 1, L.K_GEMM: 1}),
    # GAP + classifier fused; the stage-2 downsampling shortcut rides in its 3x3 stride-2 conv
    ("resnet18", 64, "bf16", {L.K_STEM_CONV: 1, L.K_CONV_TC: 18, L.K_GAP_NHWC: 1}),
    ("tx_small", 8, "fp32", {L.K_EMBED: 1, L.K_LAYERNORM: 9, L.K_GEMM: 17, L.K_FLASH_ATTN: 4, L.K_COPY: 1}),
    ("tx_small", 8, "bf16", {L.K_EMBED: 1, L.K_LAYERNORM: 9, L.K_GEMM_TC: 16, L.K_GEMM_TF32: 1, L.K_FLASH_ATTN: 4,
                             L.K_COPY: 1}),
])
def test_lowering_fuses_to_expected_kernels(model, batch, profile, kinds):
    g = BUILDERS[model]()
    prog = lower(g, batch, profile)
    got = {}
    for ln in _launches(prog):
        got[ln.kid] = got.get(ln.kid, 0) + 1
    assert got == kinds
    _check_arena(prog)
    assert prog.outputs == ["logits"]
    assert prog.tensors["logits"].dtype == L.F32


def test_shortcut_fused_into_stride2_conv():
    """The 64->128 stride-2 stage entry launches once with both outputs; the
    128- and 256-channel entries (CTA pairs) keep their own shortcut launch."""
    prog = lower(BUILDERS["resnet18"](), 8, "bf16")
    fused = [ln for ln in _launches(prog) if ln.kid == L.K_CONV_TC and ln.params.has_shortcut]
    assert len(fused) == 1
    (ln,) = fused
    assert ln.params.stride == 2 and ln.params.k == 3 and ln.params.cout == 128
    assert len(ln.ins) == 5 and len(ln.outs) == 2
    assert [ln.ins[3].shape[i] for i in range(2)] == [128, 64]


def test_shortcut_fusion_switch(monkeypatch):
    """C3B200_CONV_SHORTCUT=0 keeps the 64->128 shortcut as its own launch:
    19 tcgen05 conv launches, none with a second output, the same FLOPs."""
    fused = lower(BUILDERS["resnet18"](), 8, "bf16")
    monkeypatch.setenv("C3B200_CONV_SHORTCUT", "0")
    prog = lower(BUILDERS["resnet18"](), 8, "bf16")
    lns = [ln for ln in _launches(prog) if ln.kid == L.K_CONV_TC]
    assert len(lns) == 19 and not any(ln.params.has_shortcut for ln in lns)
    assert all(len(ln.outs) == 1 for ln in lns)
    assert abs(sum(s.flops for s in prog.steps) - sum(s.flops for s in fused.steps)) < 1.0
    _check_arena(prog)


def test_flop_accounting_per_image():
    """ResNet-18 conv GEMMs: 1.1108 GFLOP per image (the figure roofline.achieved uses)."""
    p = lower(BUILDERS["resnet18"](), 16, "bf16")
    conv = sum(s.flops for s in p.steps if s.label.startswith("conv") or s.label == "stem_conv")
    assert abs(conv / 16 - 1.1108e9) / 1.1108e9 < 1e-3


def test_bf16_rounding_helpers():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.14159, 65504.0, 1e-30], np.float32)
    assert np.array_equal(bf16_to_f32(bf16_bits(x)), round_bf16(x))
    assert bf16_bits(np.array([1.0], np.float32))[0] == 0x3F80


def test_lowering_rejects_unknown_patterns():
    from hackathon_b200.graph import ModelGraph, ValueInfo
    g = ModelGraph("bad")
    g.inputs.append(ValueInfo("x", "float32", ["batch", 4]))
    g.add("Softmax", ["x"], out_names=["logits"], axis=0)
    g.outputs.append(ValueInfo("logits", "float32", ["batch", 4]))
    g.meta["kind"] = "bad"
    with pytest.raises(NotImplementedError):
        lower(g, 2, "fp32")


class _Recorder(_DryPlan):
    def __init__(self):
        self.actions = []

    def kernel(self, s, ln, label=""):
        self.actions.append(("K", s, label, ln))

    def record(self, s, e):
        self.actions.append(("R", s, e))

    def wait(self, s, e):
        self.actions.append(("W", s, e))


def _dry_runner(model, batch, suffix="", profile=None):
    plan = json.load(open(os.path.join(HERE, "golden", f"plan_{model}_b{batch}{suffix}.json")))
    g = BUILDERS[model]()
    gold = np.load(os.path.join(HERE, "golden", f"engine_{model}.npz"))
    specs = {vi.name: (gold[vi.name][:batch].shape, gold[vi.name].dtype) for vi in g.inputs}
    rec = _Recorder()
    r = C34PlanRunner(plan, g.initializers, specs, profile=profile, target=rec)
    return r, rec, plan


@pytest.mark.parametrize("model,batch", [("mlp", 16), ("resnet18", 4), ("tx_small", 4)])
def test_reference_plan_adapter_walks_fixture(model, batch):
    r, rec, plan = _dry_runner(model, batch)
    kernels = [a for a in rec.actions if a[0] == "K"]
    names = [k["kernel_name"] for k in plan["kernel_steps"] if k["kernel_name"] != "constant"]
    assert len({a[2] for a in kernels}) == len(set(names))
    assert r.output_slots["logits"][1] == (batch, 10 if model != "tx_small" else 4096)
    recorded = set()
    for a in rec.actions:
        if a[0] == "R":
            recorded.add(a[2])
        if a[0] == "W":
            assert a[2] in recorded
    limit = r._extra_top
    for _, _, _, ln in kernels:
        for t in list(ln.ins) + list(ln.outs):
            n = int(np.prod([t.shape[i] for i in range(t.ndim)])) if t.ndim else 1
            assert t.flags & L.TENSOR_ARENA
            assert (t.ptr or 0) + n * L.DTYPE_SIZE[t.dtype] <= limit


def test_winograd_output_spills_past_the_plan():
    r, _, plan = _dry_runner("resnet18", 4)
    assert len(r.spills) >= 1
    for off, size in r.spills.values():
        assert off >= plan["arena_bytes"] and size >= 4 * 64 * 4 * 4 * 4


def test_bn_fold_formula():
    host = {"w": np.ones((2, 3, 1, 1), np.float32), "g": np.array([2.0, 4.0], np.float32),
            "b": np.array([0.5, -0.5], np.float32), "m": np.array([1.0, 2.0], np.float32),
            "v": np.array([3.0, 15.0], np.float32)}
    f = fold_weights({"W": {"weight": "w", "conv_bias": "", "bn": ["g", "b", "m", "v"], "epsilon": 1.0,
                            "bias_name": "B"}}, host)
    assert np.allclose(f["W"][:, 0, 0, 0], [1.0, 1.0])
    assert np.allclose(f["B"], [(0 - 1) * 1 + 0.5, (0 - 2) * 1 - 0.5])


def test_inputs_are_seeded():
    g = BUILDERS["resnet18"]()
    assert np.array_equal(make_inputs(g, 64)["input"], make_inputs(g, 64)["input"])
    ids = make_inputs(BUILDERS["tx_small"](), 4)["input_ids"]
    assert ids.dtype == np.int64 and ids.min() >= 0 and ids.max() < 4096
