"""Generate the committed golden fixtures from the reference itself.

Run in a container that has the reference tree (``--reference PATH``); the
outputs are small files under ``tests/golden/`` that travel with the repo, so
nothing at test time needs the reference.  What it produces:

1. ``engine_<model>.npz`` — logits of each seeded workload (small batch) computed
   by the reference's own unfused engine ops (``c35/engine.py`` OP_DISPATCH)
   with NumPy standing in for CuPy, the substitution the reference's own
   c32/test_kernel_registry.py:14-25 uses.  Also per-op known answers for the
   registry kernels that run under that substitution (im2col/contract/reshape/
   bias, c32/kernel_registry.py:318-453).
   The large decoder (configs[4] shapes) gets an engine golden at one
   sequence: ``--models tx_large --no-kat``.
3. ``plan_<model>_b<N>_b200_<bf16|fp16>.json`` -- the same graphs through the
   reference pipeline, the executor's fold rewrite, the backend's extra C3.3
   passes (``hackathon_b200.c33_passes``) and the reference scheduler with the
   bf16 or fp16 precision profile (``hackathon_b200.c34_precision``):
   ``--b200-plans``.
2. ``plan_<model>_b<N>.json`` — the reference's C3.3 fusion + C3.4 plan
   (``GraphPassPipeline().run``, ``ExecutionScheduler(graph, N).build()``) for the
   same graph, with the Conv+BN fold rewrite of c35/executor.py:359-442 applied
   first.  The backend's plan adapter replays this plan with its own kernels.

Usage: python tests/golden/make_golden.py --reference /path/to/reference
"""

from __future__ import annotations

import argparse
import copy
import json
import os
import sys
import types
from pathlib import Path
from unittest import mock

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from hackathon_b200.workloads import BUILDERS, make_inputs  # noqa: E402

# Small batches keep the fixtures a few hundred KB.
GOLDEN_BATCH = {"mlp": 16, "resnet18": 4, "tx_small": 4, "tx_large": 1}
PLAN_BATCH = {"mlp": 16, "resnet18": 4, "tx_small": 4}
# Plans through the B200 C3.3 passes and the bf16 C3.2/C3.4 profile
# (hackathon_b200.c33_passes, hackathon_b200.c34_precision): the test batches,
# plus the headline ResNet batch and its 2/4/8-GPU shards that bench.py replays.
B200_PLANS = [("mlp", 16, "bf16"), ("resnet18", 4, "bf16"), ("tx_small", 4, "bf16"), ("resnet18", 4096, "bf16"),
              ("resnet18", 2048, "bf16"), ("resnet18", 1024, "bf16"), ("resnet18", 512, "bf16"),
              ("resnet18", 4, "fp16"), ("tx_small", 4, "fp16"), ("resnet18", 4096, "fp16")]


def numpy_cupy_shim() -> types.ModuleType:
    shim = types.ModuleType("cupy")
    for k in dir(np):
        if not k.startswith("__"):
            setattr(shim, k, getattr(np, k))
    shim.asnumpy = np.asarray
    shim.ndarray = np.ndarray
    return shim


def load_reference(ref: str):
    sys.path.insert(0, ref)
    shim = numpy_cupy_shim()
    with mock.patch.dict(sys.modules, {"cupy": shim}):
        import c35.engine as engine  # noqa
        import c32.kernel_registry as registry  # noqa
    return engine, registry


def engine_run(engine, graph, feeds):
    """Unfused graph through engine.OP_DISPATCH (c35/engine.py:1448-1466)."""
    vals = dict(graph.initializers)
    vals.update(feeds)
    for n in graph.nodes:
        op = n.op_type
        xs = [vals[t] for t in n.inputs]
        attrs = dict(n.attrs)
        if op == "BatchNormalization":
            x, s, b, m, v = xs
            sh = [1, -1, 1, 1]
            r = ((x - m.reshape(sh)) / np.sqrt(v.reshape(sh) + np.float32(attrs["epsilon"]))
                 * s.reshape(sh) + b.reshape(sh)).astype(np.float32)
        elif op == "Split":
            r = engine.execute_op(op, xs, {**attrs, "_num_outputs": len(n.outputs)})
        else:
            r = engine.execute_op(op, xs, attrs)
        if isinstance(r, list):
            for name, val in zip(n.outputs, r):
                vals[name] = np.asarray(val)
        else:
            vals[n.outputs[0]] = np.asarray(r)
    return {o.name: vals[o.name] for o in graph.outputs}


def infer_shapes(graph):
    """Symbolic-batch tensor shapes, from two oracle-free engine runs (b=2, b=3)."""
    from oracle.evaluate import run_graph
    v2 = run_graph(graph, make_inputs(graph, 2), keep=True)
    v3 = run_graph(graph, make_inputs(graph, 3), keep=True)
    shapes = {}
    for k in v2:
        if k in graph.initializers:
            continue
        a, b = np.shape(v2[k]), np.shape(v3[k])
        shapes[k] = ["batch" if x != y else int(x) for x, y in zip(a, b)]
        shapes[k + "::dtype"] = str(np.asarray(v2[k]).dtype)
    return shapes


def to_reference_ir(ref_ir, graph, shapes):
    Graph, Node, ONNSType = ref_ir.Graph, ref_ir.Node, ref_ir.ONNSType
    g = Graph()
    g.name = graph.name
    g.opsets = {"ai.onnx": 17}
    dt = {"float32": ONNSType.FLOAT, "int64": ONNSType.INT64}
    for name, val in graph.initializers.items():
        t = g.register_tensor(name, dtype=dt[str(val.dtype)], shape=list(val.shape), is_initializer=True)
        g.initializers[name] = t
        g.tensor_producer[name] = "INITIALIZER"
    for vi in graph.inputs:
        t = g.register_tensor(vi.name, dtype=dt[vi.dtype], shape=list(vi.shape))
        g.inputs.append(t)
        g.tensor_producer[vi.name] = "INPUT"
    for vi in graph.outputs:
        t = g.register_tensor(vi.name, dtype=dt[vi.dtype], shape=list(vi.shape))
        g.outputs.append(t)
    for idx, n in enumerate(graph.nodes):
        nid = ref_ir.generate_node_id(n.name, n.op_type, idx)
        node = Node(id=nid, name=n.name, op_type=n.op_type, inputs=list(n.inputs),
                    outputs=list(n.outputs), attributes=copy.deepcopy(n.attrs))
        g.add_node(node)
        for o in n.outputs:
            g.register_tensor(o, dtype=dt[shapes[o + "::dtype"]], shape=list(shapes[o]))
            g.set_producer(o, nid)
    g.validate()
    return g


def fold_bn_rewrite(g):
    """c35/executor.py:359-442 graph rewrite (values are folded by the adapter)."""
    folds = {}
    for nid in list(g.node_order):
        node = g.nodes.get(nid)
        if node is None or node.op_type != "FusedConv2dBatchNorm" or node.attributes.get("bn_folded"):
            continue
        off = int(node.attributes.get("bn_parameter_offset", len(node.inputs)))
        conv_in = list(node.inputs[:off])
        bn_in = list(node.inputs[off:off + 4])
        wname = f"__c3_folded_{nid}_weight__"
        bname = f"__c3_folded_{nid}_bias__"
        wt = g.tensors[conv_in[1]]
        from c3common.ir.graph import ONNSType
        for name, shape in ((wname, list(wt.shape)), (bname, [int(wt.shape[0])])):
            t = g.register_tensor(name, dtype=ONNSType.FLOAT, shape=shape, is_initializer=True)
            g.initializers[name] = t
            g.tensor_producer[name] = "INITIALIZER"
        g.replace_node_inputs(nid, list(node.inputs), [conv_in[0], wname, bname])
        node.attributes["bn_folded"] = True
        node.attributes["bn_parameter_offset"] = 3
        node.attributes["folded_weight"] = wname
        node.attributes["folded_bias"] = bname
        folds[wname] = {"weight": conv_in[1], "conv_bias": conv_in[2] if len(conv_in) > 2 else "",
                        "bn": bn_in, "epsilon": float(node.attributes.get("bn_epsilon", 1e-5)),
                        "bias_name": bname}
    g.validate()
    return folds


def _jsonable(v):
    if isinstance(v, dict):
        return {str(k): _jsonable(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [_jsonable(x) for x in v]
    if isinstance(v, (np.integer,)):
        return int(v)
    if isinstance(v, (np.floating,)):
        return float(v)
    if isinstance(v, np.ndarray):
        return v.tolist()
    if isinstance(v, (str, int, float, bool)) or v is None:
        return v
    return str(v)


def plan_to_json(plan, g, folds, graph):
    return {
        "model": graph.name,
        "batch_size": plan.batch_size,
        "arena_bytes": int(plan.pool_stats.peak_reserved_bytes),
        "copy_stream_id": plan.copy_stream_id,
        "allocations": [dict(alloc_id=a.alloc_id, tensor_name=a.tensor_name, size_bytes=a.size_bytes,
                             offset_bytes=a.offset_bytes, capacity_bytes=a.capacity_bytes,
                             is_weight=a.is_weight, is_output=a.is_output) for a in plan.allocations],
        "transfers": [dict(kind=t.kind, tensor_name=t.tensor_name, alloc_id=t.alloc_id,
                           size_bytes=t.size_bytes, stream_id=t.stream_id) for t in plan.transfers],
        "kernel_steps": [dict(step_index=k.step_index, kernel_name=k.kernel_name, node_id=k.node_id,
                              logical_inputs=list(k.logical_inputs), logical_outputs=list(k.logical_outputs),
                              inputs=dict(k.inputs), outputs=dict(k.outputs), stream_id=k.stream_id,
                              tuning_params=_jsonable(k.tuning_params),
                              operator_params=_jsonable(k.operator_params),
                              precision_profile=_jsonable(k.precision_profile or {})) for k in plan.kernel_steps],
        "events": [e.event_id for e in plan.events],
        "timeline": [dict(kind=s.kind, stream_id=s.stream_id, ref_index=s.ref_index,
                          event_id=s.event_id, tensor_name=s.tensor_name) for s in plan.timeline],
        "weight_slots": dict(plan.weight_slots),
        "tensor_shapes": {name: _jsonable(t.shape) for name, t in g.tensors.items()},
        "graph_inputs": [t.name for t in g.inputs],
        "graph_outputs": [t.name for t in g.outputs],
        "folds": folds,
    }


def b200_plans(ref: str) -> None:
    load_reference(ref)
    sys.path.insert(0, ref)
    import c3common.ir.graph as ref_ir
    from c33.pipeline import GraphPassPipeline
    from hackathon_b200.c33_passes import run_b200_passes
    from hackathon_b200.c34_precision import build_plan
    for model, batch, profile in B200_PLANS:
        graph = BUILDERS[model]()
        g = to_reference_ir(ref_ir, graph, infer_shapes(graph))
        res = GraphPassPipeline().run(g)
        assert res["Fusion"]["stats"]["validation_passed"]
        folds = fold_bn_rewrite(g)
        counts = run_b200_passes(g)["counts"]
        plan = build_plan(g, batch, profile)
        js = plan_to_json(plan, g, folds, graph)
        js["b200_passes"] = counts
        with open(HERE / f"plan_{model}_b{batch}_b200_{profile}.json", "w") as f:
            json.dump(js, f, separators=(",", ":"))
        names = [k["kernel_name"] for k in js["kernel_steps"]]
        print(model, batch, profile, "b200 plan kernels", len(names), sorted(set(names)), counts)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--models", default=",".join(GOLDEN_BATCH),
                    help="comma-separated subset of the workloads to (re)generate")
    ap.add_argument("--no-kat", action="store_true", help="skip the registry known answers")
    ap.add_argument("--b200-plans", action="store_true",
                    help="only (re)generate the plans with the backend's passes and bf16 profile")
    args = ap.parse_args()
    wanted = [m for m in args.models.split(",") if m]
    if args.b200_plans:
        b200_plans(args.reference)
        return
    engine, registry = load_reference(args.reference)
    sys.path.insert(0, args.reference)
    import c3common.ir.graph as ref_ir
    from c33.pipeline import GraphPassPipeline
    from c34.scheduler import ExecutionScheduler

    for model in wanted:
        batch = GOLDEN_BATCH[model]
        graph = BUILDERS[model]()
        feeds = make_inputs(graph, batch)
        out = engine_run(engine, graph, feeds)
        np.savez_compressed(HERE / f"engine_{model}.npz", batch=batch, **feeds, **out)
        print(model, "engine logits", out["logits"].shape)
        if model not in PLAN_BATCH:
            continue  # engine golden only (the large config's plan is not a fixture)

        shapes = infer_shapes(graph)
        g = to_reference_ir(ref_ir, graph, shapes)
        res = GraphPassPipeline().run(g)
        assert res["Fusion"]["stats"]["validation_passed"]
        folds = fold_bn_rewrite(g)
        pb = PLAN_BATCH[model]
        plan = ExecutionScheduler(g, batch_size=pb).build()
        issues = plan.validate()
        assert not issues, issues[:5]
        js = plan_to_json(plan, g, folds, graph)
        with open(HERE / f"plan_{model}_b{pb}.json", "w") as f:
            json.dump(js, f, separators=(",", ":"))
        names = [k["kernel_name"] for k in js["kernel_steps"]]
        print(model, "plan kernels", len(names), sorted(set(names)))

    if args.no_kat:
        return
    # Registry known answers (c32/test_kernel_registry.py:52-105 style).
    rng = np.random.default_rng(7)
    x = rng.standard_normal((2, 3, 7, 6), dtype=np.float32)
    w = rng.standard_normal((5, 3, 3, 2), dtype=np.float32)
    b = rng.standard_normal((5,), dtype=np.float32)
    params = {"kernel_shape": [3, 2], "strides": [2, 1], "pads": [1, 0, 1, 1],
              "dilations": [1, 2], "_batch_size": 2}
    n, c, h, wd = x.shape
    ho = (h + 2 - 3) // 2 + 1
    wo = (wd + 1 - (2 * 1 + 1)) // 1 + 1
    col = np.zeros((n * ho * wo, c * 3 * 2), np.float32)
    outs = [col]
    registry.kernel_im2col([x], outs, params, None)
    col = outs[0]
    mm = [np.zeros((n * ho * wo, 5), np.float32)]
    registry.kernel_matmul([col, w], mm, {**params, "lowering_kind": "conv_contract"}, None)
    rs = [np.zeros((n, 5, ho, wo), np.float32)]
    registry.kernel_conv_reshape([mm[0]], rs, {**params, "_output_spatial": [ho, wo]}, None)
    ob = [np.zeros_like(rs[0])]
    registry.kernel_add_bias([rs[0], b], ob, {"bias_axis": 1}, None)
    sc = [np.zeros((2, 3, 7, 6), np.float32)]
    registry.kernel_erf([x], sc, {}, None)
    np.savez_compressed(HERE / "registry_kat.npz", x=x, w=w, b=b, im2col=col, contract=mm[0],
                        nchw=rs[0], biased=ob[0], erf_as=sc[0],
                        params=json.dumps(params))
    print("registry KAT written")


if __name__ == "__main__":
    main()
