"""Run the reference's own C3.4 ``ExecutionPlan`` on the native executor.

This is the drop-in for ``PlannedGraphExecutor`` (c35/executor.py:324-903):
given the plan C3.4 built (``ExecutionScheduler(graph, batch).build()``) and
the model's host initializers, it

* folds Conv+BN initializers on the host with the executor's formula
  (c35/executor.py:400-411) for every fold the plan references;
* binds every plan allocation at the plan's own arena offset
  (``Allocation.offset_bytes``) inside one arena of
  ``pool_stats.peak_reserved_bytes`` (executor.py:757-765);
* uploads model tensors once (they stay resident, executor.py:805-839);
* turns each timeline action into a native action: H2D of graph inputs from
  pinned slots, KERNEL steps through the same per-name launch builders the
  eager registry uses (``kernels.prepare``), EVENT_RECORD / EVENT_WAIT on real
  events, D2H of graph outputs into pinned slots;
* ALLOC / FREE are bookkeeping only, as in the reference (executor.py:791-796).

Plans are accepted as the live reference object (duck-typed) or as the JSON
dict ``plan_to_dict`` produces (the committed fixtures use that form).
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import numpy as np

from . import _lib as L
from .kernels import Desc, prepare
from .runtime import NativePlan

_NP_DTYPE = {np.dtype(np.float32): L.F32, np.dtype(np.int64): L.I64, np.dtype(np.int32): L.I32}


def plan_to_dict(plan: Any, graph: Any, folds: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    """Flatten a reference ``ExecutionPlan`` (c34/execution_plan.py:17-189)."""
    return {
        "model": getattr(graph, "name", ""),
        "batch_size": plan.batch_size,
        "arena_bytes": int(plan.pool_stats.peak_reserved_bytes),
        "allocations": [dict(alloc_id=a.alloc_id, tensor_name=a.tensor_name, size_bytes=a.size_bytes,
                             offset_bytes=a.offset_bytes, capacity_bytes=a.capacity_bytes,
                             is_weight=a.is_weight, is_output=a.is_output) for a in plan.allocations],
        "transfers": [dict(kind=t.kind, tensor_name=t.tensor_name, alloc_id=t.alloc_id, size_bytes=t.size_bytes,
                           stream_id=t.stream_id) for t in plan.transfers],
        "kernel_steps": [dict(step_index=k.step_index, kernel_name=k.kernel_name, node_id=k.node_id,
                              logical_inputs=list(k.logical_inputs), logical_outputs=list(k.logical_outputs),
                              inputs=dict(k.inputs), outputs=dict(k.outputs), stream_id=k.stream_id,
                              tuning_params=k.tuning_params, operator_params=dict(k.operator_params))
                         for k in plan.kernel_steps],
        "events": [e.event_id for e in plan.events],
        "timeline": [dict(kind=s.kind, stream_id=s.stream_id, ref_index=s.ref_index, event_id=s.event_id,
                          tensor_name=s.tensor_name) for s in plan.timeline],
        "weight_slots": dict(plan.weight_slots),
        "graph_inputs": [t.name for t in graph.inputs],
        "graph_outputs": [t.name for t in graph.outputs],
        "folds": folds or {},
    }


def fold_weights(folds: Dict[str, Any], host: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    """c35/executor.py:400-411: w' = w*g/sqrt(v+eps); b' = (b - mu)*g/sqrt(v+eps) + beta."""
    out: Dict[str, np.ndarray] = {}
    for wname, f in folds.items():
        w = np.asarray(host[f["weight"]], np.float32)
        scale, beta, mean, var = (np.asarray(host[n], np.float32).reshape(-1) for n in f["bn"])
        cb = np.asarray(host[f["conv_bias"]], np.float32).reshape(-1) if f.get("conv_bias") else np.zeros_like(mean)
        factor = (scale / np.sqrt(var + np.float32(f.get("epsilon", 1e-5)))).astype(np.float32)
        out[wname] = np.ascontiguousarray(w * factor.reshape((-1,) + (1,) * (w.ndim - 1)), np.float32)
        out[f["bias_name"]] = np.ascontiguousarray((cb - mean) * factor + beta, np.float32)
    return out


class _DryPlan:
    """Records nothing; lets the adapter walk a plan once to size spill slots."""

    def upload(self, *a):
        pass

    def add_input_slot(self, nbytes):
        return 0

    def add_output_slot(self, nbytes):
        return 0

    def h2d(self, *a):
        pass

    def d2h(self, *a):
        pass

    def record(self, *a):
        pass

    def wait(self, *a):
        pass

    def kernel(self, *a, **k):
        pass


class C34PlanRunner:
    """Native replay of one reference plan for one batch size.

    A kernel whose correctly sized output exceeds the slot C3.4 planned for it
    gets a dedicated slot past the plan's arena ("spill").  This happens for
    ``winograd_forward_f32``: the reference sizes its output for the
    unpadded F(2,3) tiling and the kernel itself raises before writing
    (c32/kernel_registry.py:521,534), so the reference never noticed.
    """

    def __init__(self, plan: Dict[str, Any], host_weights: Dict[str, np.ndarray],
                 input_specs: Dict[str, Tuple[Tuple[int, ...], Any]], use_graph: bool = True):
        self.plan = plan
        weights = dict(host_weights)
        weights.update(fold_weights(plan.get("folds", {}), host_weights))
        self._weights = weights
        self._specs = input_specs
        stream_ids = sorted({s["stream_id"] for s in plan["timeline"] if s["kind"] not in ("ALLOC", "FREE")})
        self.stream_index = {sid: i for i, sid in enumerate(stream_ids)}
        self.event_index = {eid: i for i, eid in enumerate(plan["events"])}
        base = max(256, int(plan["arena_bytes"]))
        self.spills: Dict[str, Tuple[int, int]] = {}
        self._walk(_DryPlan(), base)
        total = base + sum(sz for _, sz in self.spills.values())
        self.native = NativePlan(total, len(stream_ids), len(plan["events"]))
        self._walk(self.native, base)
        self.native.finalize(use_graph)

    def _walk(self, np_, base: int) -> None:
        plan, weights, input_specs = self.plan, self._weights, self._specs
        allocs = {a["alloc_id"]: a for a in plan["allocations"]}
        values: Dict[str, Desc] = {}
        self.input_slots: Dict[str, Tuple[int, Tuple[int, ...], Any]] = {}
        self.output_slots: Dict[str, Tuple[int, Tuple[int, ...], Any]] = {}
        for step in plan["timeline"]:
            kind = step["kind"]
            if kind in ("ALLOC", "FREE"):
                continue
            s = self.stream_index[step["stream_id"]]
            if kind == "EVENT_RECORD":
                np_.record(s, self.event_index[step["event_id"]])
            elif kind == "EVENT_WAIT":
                np_.wait(s, self.event_index[step["event_id"]])
            elif kind == "H2D":
                tr = plan["transfers"][step["ref_index"]]
                name = tr["tensor_name"]
                a = allocs[tr["alloc_id"]]
                cap = a["capacity_bytes"] or a["size_bytes"]
                if name in input_specs:
                    shape, dt = input_specs[name]
                    nbytes = int(np.prod(shape)) * np.dtype(dt).itemsize
                    if nbytes > cap:
                        raise ValueError(f"input {name!r} needs {nbytes} bytes, planned capacity is {cap}")
                    slot = np_.add_input_slot(nbytes)
                    self.input_slots[name] = (slot, tuple(shape), np.dtype(dt))
                    np_.h2d(s, slot, 0, a["offset_bytes"], nbytes)
                    values[name] = Desc(a["offset_bytes"], _NP_DTYPE[np.dtype(dt)], tuple(shape), True)
                else:
                    if name not in weights:
                        raise KeyError(f"No H2D source for '{name}'")
                    host = np.ascontiguousarray(weights[name])
                    if host.dtype not in _NP_DTYPE:
                        host = host.astype(np.float32)
                    if host.nbytes > cap:
                        raise ValueError(f"'{name}' requires {host.nbytes} bytes, planned capacity is {cap}")
                    # Model tensors are uploaded once and stay resident (executor.py:805-839).
                    np_.upload(a["offset_bytes"], host)
                    values[name] = Desc(a["offset_bytes"], _NP_DTYPE[host.dtype], tuple(host.shape), True,
                                        host=host if host.size <= 64 else None)
            elif kind == "KERNEL":
                ks = plan["kernel_steps"][step["ref_index"]]
                ins: List[Optional[Desc]] = []
                for nm in ks["logical_inputs"]:
                    if not nm:
                        ins.append(None)
                    elif nm not in values:
                        raise KeyError(f"Kernel '{ks['kernel_name']}' (node '{ks['node_id']}') requires "
                                       f"unavailable input '{nm}'")
                    else:
                        ins.append(values[nm])
                onames = [n for n in ks["logical_outputs"] if n]

                def out_descs():
                    res = []
                    for nm in onames:
                        if nm in self.spills:
                            off, sz = self.spills[nm]
                            res.append(Desc(off, L.F32, (sz // 4,), True))
                        else:
                            a = allocs[ks["outputs"][nm]]
                            cap = a["capacity_bytes"] or a["size_bytes"]
                            res.append(Desc(a["offset_bytes"], L.F32, (cap // 4,), True))
                    return res
                outs = out_descs()
                params = ks.get("operator_params") or {}
                try:
                    prep = prepare(ks["kernel_name"], ins, outs, params)
                except ValueError as e:
                    if "Output arena too small" not in str(e) or not isinstance(np_, _DryPlan):
                        raise
                    big = [Desc(0, L.F32, (1 << 40,), True) for _ in onames]
                    prep = prepare(ks["kernel_name"], ins, big, params)
                    top = base + sum(sz for _, sz in self.spills.values())
                    for nm, shp in zip(onames, prep.out_shapes):
                        need = (int(np.prod(shp)) * 4 + 255) // 256 * 256
                        self.spills[nm] = (top, need)
                        top += need
                    outs = out_descs()
                    prep = prepare(ks["kernel_name"], ins, outs, params)
                for ln in prep.launches:
                    np_.kernel(s, ln, ks["kernel_name"])
                k = 0
                for ln in prep.launches:
                    for t in ln.outs:
                        if k < len(onames):
                            values[onames[k]] = Desc(outs[k].ptr, int(t.dtype), tuple(prep.out_shapes[k]), True)
                        k += 1
            elif kind == "D2H":
                tr = plan["transfers"][step["ref_index"]]
                name = tr["tensor_name"]
                if name not in values:
                    raise KeyError(f"D2H source '{name}' is unavailable")
                d = values[name]
                nbytes = d.numel * L.DTYPE_SIZE[d.dtype]
                slot = np_.add_output_slot(nbytes)
                np_dt = {L.F32: np.float32, L.I64: np.int64, L.I32: np.int32}[d.dtype]
                self.output_slots[name] = (slot, d.shape, np.dtype(np_dt))
                np_.d2h(s, slot, 0, d.ptr, nbytes)
            else:
                raise ValueError(f"Unsupported timeline action: {kind}")
        self.values = values

    def run(self, feeds: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
        for name, (slot, shape, dt) in self.input_slots.items():
            arr = np.asarray(feeds[name])
            if tuple(arr.shape) != shape:
                raise ValueError(f"input {name!r} shape {arr.shape} != planned {shape}")
            self.native.slot_array(False, slot, dt, shape)[...] = arr
        self.native.run()
        return {name: self.native.slot_array(True, slot, dt, shape).copy()
                for name, (slot, shape, dt) in self.output_slots.items()}
