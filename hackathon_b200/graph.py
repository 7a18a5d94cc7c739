"""Minimal ONNX-shaped graph container used by the workload builders.

The reference imports ONNX files into ``c3common.ir.graph.Graph``
(c3common/ir/graph.py:117-480) through C3.1 (c31/import_onnx.py:59-240).
Neither ``onnx`` nor the reference tree is available where this backend runs,
so the seeded workloads are built directly as this small container: ordered
ONNX nodes (op type, input/output tensor names, opset-17 attributes),
initializers as host arrays, and the public inputs/outputs with their shapes.
It carries exactly what the lowering and the oracle need and nothing more.
A symbolic batch dimension is written as the string ``"batch"`` as in the
reference's IR.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Sequence, Tuple, Union

import numpy as np

Dim = Union[int, str]


@dataclass
class Node:
    op_type: str
    inputs: List[str]
    outputs: List[str]
    attrs: Dict[str, Any] = field(default_factory=dict)
    name: str = ""


@dataclass
class ValueInfo:
    name: str
    dtype: str  # numpy dtype name: "float32" or "int64"
    shape: List[Dim]


@dataclass
class ModelGraph:
    name: str
    nodes: List[Node] = field(default_factory=list)
    initializers: Dict[str, np.ndarray] = field(default_factory=dict)
    inputs: List[ValueInfo] = field(default_factory=list)
    outputs: List[ValueInfo] = field(default_factory=list)
    # Metadata for builders (e.g. transformer dims) — not used by execution.
    meta: Dict[str, Any] = field(default_factory=dict)

    _counter: int = 0

    def fresh(self, stem: str) -> str:
        self._counter += 1
        return f"{stem}_{self._counter}"

    def add(self, op_type: str, inputs: Sequence[str], n_out: int = 1,
            out_names: Sequence[str] | None = None, **attrs: Any) -> Union[str, List[str]]:
        if out_names is None:
            out_names = [self.fresh(op_type.lower()) for _ in range(n_out)]
        node = Node(op_type, list(inputs), list(out_names), dict(attrs),
                    name=f"{op_type}_{len(self.nodes)}")
        self.nodes.append(node)
        return out_names[0] if len(out_names) == 1 else list(out_names)

    def init(self, name: str, value: np.ndarray) -> str:
        if name in self.initializers:
            raise ValueError(f"duplicate initializer {name!r}")
        self.initializers[name] = value
        return name

    def param_count(self) -> int:
        return int(sum(v.size for v in self.initializers.values()))

    def consumers(self) -> Dict[str, List[int]]:
        out: Dict[str, List[int]] = {}
        for i, n in enumerate(self.nodes):
            for t in n.inputs:
                if t:
                    out.setdefault(t, []).append(i)
        return out

    def producer(self) -> Dict[str, int]:
        out: Dict[str, int] = {}
        for i, n in enumerate(self.nodes):
            for t in n.outputs:
                out[t] = i
        return out


def concrete_shape(shape: Sequence[Dim], batch: int) -> Tuple[int, ...]:
    return tuple(batch if isinstance(d, str) else int(d) for d in shape)
