"""ONNX file -> ModelGraph, for ``deploy --onnx`` (the job of C3.1's
``import_onnx``, c31/import_onnx.py:59-240: initializers, graph inputs that are
not initializers, outputs, nodes with their attributes, in file order).

Needs the ``onnx`` package; without it this raises ImportError with a clear
message (the built-in seeded workloads need no ONNX).
"""

from __future__ import annotations

from .graph import ModelGraph, Node, ValueInfo

_ELEM = {1: "float32", 7: "int64", 6: "int32"}


def import_onnx(path: str) -> ModelGraph:
    try:
        import onnx
        from onnx import numpy_helper
    except ImportError as e:  # pragma: no cover - depends on the environment
        raise ImportError("deploy --onnx needs the 'onnx' package; use --model for the built-in workloads") from e
    model = onnx.load(path)
    onnx.checker.check_model(model)
    gp = model.graph
    g = ModelGraph(gp.name or path)
    inits = set()
    for t in gp.initializer:
        g.initializers[t.name] = numpy_helper.to_array(t).copy()
        inits.add(t.name)

    def vinfo(v):
        tt = v.type.tensor_type
        dims = [d.dim_param if d.dim_param else int(d.dim_value) for d in tt.shape.dim]
        dims = ["batch" if isinstance(d, str) or d == 0 else d for d in dims]
        return ValueInfo(v.name, _ELEM.get(tt.elem_type, "float32"), dims)

    for v in gp.input:
        if v.name not in inits:
            g.inputs.append(vinfo(v))
    for v in gp.output:
        g.outputs.append(vinfo(v))
    for i, n in enumerate(gp.node):
        if n.op_type == "Constant":
            for a in n.attribute:
                if a.name == "value":
                    g.initializers[n.output[0]] = numpy_helper.to_array(a.t).copy()
            continue
        attrs = {a.name: onnx.helper.get_attribute_value(a) for a in n.attribute}
        attrs = {k: (v.decode() if isinstance(v, bytes) else v) for k, v in attrs.items()}
        attrs = {k: (list(v) if isinstance(v, (list, tuple)) else v) for k, v in attrs.items()}
        g.nodes.append(Node(n.op_type, list(n.input), list(n.output), attrs, n.name or f"{n.op_type}_{i}"))
    g.meta["kind"] = "onnx"
    return g
