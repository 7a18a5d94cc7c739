"""CPU oracle: run an unfused workload graph op by op in float32 NumPy.

TEST INFRASTRUCTURE ONLY (see ``oracle/ops.py``).  This restates the
reference's unfused ``GraphExecutor`` (c35/executor.py:240-321), which walks the
graph in topological order and dispatches each ONNX op through
``engine.OP_DISPATCH`` (c35/engine.py:696-716).
"""

from __future__ import annotations

from typing import Dict

import numpy as np

from . import ops

F32 = np.float32


def _run_node(n, vals: Dict[str, np.ndarray]):
    a = n.attrs
    x = [vals[t] if t else None for t in n.inputs]
    op = n.op_type
    if op == "Gemm":
        return ops.gemm(x[0], x[1], x[2] if len(x) > 2 else None, a.get("alpha", 1.0),
                        a.get("beta", 1.0), a.get("transA", 0), a.get("transB", 0))
    if op == "Relu":
        return np.maximum(x[0], F32(0))
    if op == "Conv":
        return ops.conv2d(x[0], x[1], x[2] if len(x) > 2 else None, **a)
    if op == "BatchNormalization":
        return ops.batchnorm(x[0], x[1], x[2], x[3], x[4], a.get("epsilon", 1e-5))
    if op == "Add":
        return (x[0] + x[1]).astype(F32)
    if op == "Sub":
        return (x[0] - x[1]).astype(F32)
    if op == "Mul":
        return (x[0] * x[1]).astype(F32)
    if op == "Div":
        return (x[0] / x[1]).astype(F32)
    if op == "Erf":
        return ops.erf_as(x[0])
    if op == "GlobalAveragePool":
        return ops.global_average_pool(x[0])
    if op == "Flatten":
        ax = int(a.get("axis", 1)) % (x[0].ndim + 1)
        return x[0].reshape(int(np.prod(x[0].shape[:ax])), -1)
    if op == "Gather":
        return ops.gather(x[0], x[1], a.get("axis", 0)).astype(x[0].dtype)
    if op == "LayerNormalization":
        return ops.layer_norm(x[0], x[1], x[2] if len(x) > 2 else None,
                              a.get("axis", -1), a.get("epsilon", 1e-5))
    if op == "MatMul":
        return np.matmul(x[0], x[1]).astype(F32)
    if op == "Split":
        return ops.split(x[0], x[1].tolist(), a.get("axis", 0))
    if op == "Reshape":
        return x[0].reshape(ops.resolve_reshape(x[0].shape, x[1].tolist(), a.get("allowzero", 0)))
    if op == "Transpose":
        return np.ascontiguousarray(np.transpose(x[0], a["perm"]))
    if op == "Softmax":
        return ops.softmax(x[0], a.get("axis", -1))
    raise ValueError(f"oracle: unsupported op {op}")


def run_graph(graph, feeds: Dict[str, np.ndarray], keep: bool = False) -> Dict[str, np.ndarray]:
    """Execute ``graph`` (hackathon_b200.graph.ModelGraph) on host arrays."""
    vals: Dict[str, np.ndarray] = dict(graph.initializers)
    vals.update(feeds)
    for n in graph.nodes:
        r = _run_node(n, vals)
        if isinstance(r, list):
            for name, v in zip(n.outputs, r):
                vals[name] = v
        else:
            vals[n.outputs[0]] = r
    if keep:
        return vals
    return {o.name: vals[o.name] for o in graph.outputs}
