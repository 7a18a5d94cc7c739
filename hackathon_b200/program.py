"""Backend program: fused kernel steps, arena planning and native execution.

A :class:`Program` is what the backend's own lowering (``lowering.py``)
produces from a workload graph: tensors (inputs, resident weights,
activations, outputs) and an ordered list of fused kernel steps.  ``plan()``
assigns arena offsets with lifetime-based best-fit reuse (the job of C3.4's
``_allocate_intermediates`` / memory_pool, c34/scheduler.py:529-597,
c34/memory_pool.py:66-126; here 256-byte aligned so every tensor can be a TMA
base), and ``Executor`` turns the result into a native plan: H2D of inputs on a
copy stream, the kernels on a compute stream, D2H of outputs, captured as one
CUDA graph.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib as L
from .kernels import Desc, Launch
from .runtime import NativePlan

ALIGN = 256
NP_OF = {L.F32: np.float32, L.I64: np.int64, L.I32: np.int32, L.F16: np.float16, L.BF16: np.uint16, L.U8: np.uint8}


def _align(x: int) -> int:
    return (x + ALIGN - 1) // ALIGN * ALIGN


@dataclass
class TensorInfo:
    name: str
    shape: Tuple[int, ...]
    dtype: int
    kind: str  # "input" | "weight" | "act"
    host: Optional[np.ndarray] = None  # weights: the (already converted) host values
    offset: int = -1
    # weights quantised on the device at set-up (fp8 profile): fp32 source and
    # the name of the row-scale tensor the quantiser also writes
    quant_src: Optional[np.ndarray] = None
    quant_scale: Optional[str] = None

    @property
    def nbytes(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64)) * L.DTYPE_SIZE[self.dtype]


@dataclass
class Step:
    label: str
    inputs: List[str]
    outputs: List[str]
    build: Callable[[Dict[str, Desc]], List[Launch]]
    flops: float = 0.0
    bytes: float = 0.0


@dataclass
class Program:
    name: str
    tensors: Dict[str, TensorInfo] = field(default_factory=dict)
    steps: List[Step] = field(default_factory=list)
    inputs: List[str] = field(default_factory=list)
    outputs: List[str] = field(default_factory=list)
    arena_bytes: int = 0
    weight_bytes: int = 0

    def add_tensor(self, name: str, shape, dtype: int, kind: str = "act", host=None) -> str:
        if name in self.tensors:
            raise ValueError(f"duplicate tensor {name}")
        self.tensors[name] = TensorInfo(name, tuple(int(d) for d in shape), dtype, kind, host)
        return name

    def add_step(self, label, inputs, outputs, build, flops=0.0, nbytes=0.0) -> None:
        for t in list(inputs) + list(outputs):
            if t not in self.tensors:
                raise KeyError(f"step {label}: unknown tensor {t}")
        self.steps.append(Step(label, list(inputs), list(outputs), build, flops, nbytes))

    # ---------------------------------------------------------------- planning
    def plan(self) -> int:
        """Assign arena offsets; returns the arena size in bytes."""
        off = 0
        for t in self.tensors.values():
            if t.kind == "weight":
                t.offset = off
                off = _align(off + t.nbytes)
        self.weight_bytes = off
        first: Dict[str, int] = {}
        last: Dict[str, int] = {}
        for name in self.inputs:
            first[name] = -1
        for i, s in enumerate(self.steps):
            for t in s.outputs:
                first.setdefault(t, i)
                last[t] = max(last.get(t, i), i)
            for t in s.inputs:
                last[t] = max(last.get(t, i), i)
                first.setdefault(t, i)
        # Outputs and inputs live for the whole pass: inputs may be uploaded once
        # and replayed (kernels-only executor), so their bytes are never reused.
        for name in list(self.outputs) + list(self.inputs):
            last[name] = len(self.steps)
        acts = [t for t in self.tensors.values() if t.kind in ("act", "input") and t.name in first]
        # best-fit free list over [base, ...)
        base = off
        free: List[Tuple[int, int]] = []  # (offset, size)
        top = base
        events = []
        for t in acts:
            events.append((first[t.name], 1, t.name))
            events.append((last.get(t.name, first[t.name]) + 0.5, 0, t.name))
        events.sort(key=lambda e: (e[0], e[1]))
        for _, is_alloc, name in events:
            t = self.tensors[name]
            size = _align(max(1, t.nbytes))
            if is_alloc:
                best = None
                for i, (fo, fs) in enumerate(free):
                    if fs >= size and (best is None or fs < free[best][1]):
                        best = i
                if best is not None:
                    fo, fs = free.pop(best)
                    t.offset = fo
                    if fs > size:
                        free.append((fo + size, fs - size))
                else:
                    t.offset = top
                    top += size
            else:
                free.append((t.offset, size))
                free.sort()
                merged: List[Tuple[int, int]] = []
                for fo, fs in free:
                    if merged and merged[-1][0] + merged[-1][1] == fo:
                        merged[-1] = (merged[-1][0], merged[-1][1] + fs)
                    else:
                        merged.append((fo, fs))
                free = merged
        self.arena_bytes = max(top, base, 256)
        return self.arena_bytes

    def desc(self, name: str) -> Desc:
        t = self.tensors[name]
        return Desc(t.offset, t.dtype, t.shape, True)


def _quantize_weights_on_device(prog: Program) -> None:
    """Rowwise E4M3 weights (the fp8 profile) computed once on the GPU by the
    same kernel that quantises activations (C3B_K_QUANT_E4M3: per row
    scale = max|w| / 448, bytes = E4M3(w / scale), nearest even, saturating),
    through a one-off native plan; the bytes and scales become the weights'
    host values, uploaded like every other weight."""
    todo = [t for t in prog.tensors.values() if t.quant_src is not None and t.host is None]
    if not todo:
        return
    offs, top = [], 0
    for t in todo:
        n, k = t.shape
        src, q, sc = top, top + _align(n * k * 4), 0
        sc = q + _align(n * k)
        top = sc + _align(n * 4)
        offs.append((src, q, sc))
    plan = NativePlan(top, n_streams=1)
    try:
        for t, (src, q, sc) in zip(todo, offs):
            n, k = t.shape
            plan.upload(src, np.ascontiguousarray(t.quant_src, np.float32))
            plan.kernel(0, Launch(L.K_QUANT_E4M3, [L.make_tensor(src, L.F32, (n, k), True)],
                                  [L.make_tensor(q, L.U8, (n, k), True), L.make_tensor(sc, L.F32, (n,), True)],
                                  L.QuantParams(n, k)), "quant_weights_e4m3")
        plan.finalize(use_graph=False)  # finalize runs the pass once
        plan.sync()
        for t, (src, q, sc) in zip(todo, offs):
            n, k = t.shape
            t.host = plan.download(q, np.empty((n, k), np.uint8))
            prog.tensors[t.quant_scale].host = plan.download(sc, np.empty((n,), np.float32))
    finally:
        plan.close()


class Executor:
    """A planned program bound to a native plan with pinned input/output slots."""

    COPY, COMPUTE = 0, 1

    def __init__(self, prog: Program, use_graph: bool = True, copies: bool = True):
        """``copies=False`` builds a kernels-only pass over inputs that stay
        resident in the arena (``upload_inputs`` / ``read_outputs``)."""
        if prog.arena_bytes == 0:
            prog.plan()
        self.prog = prog
        self.copies = copies
        _quantize_weights_on_device(prog)
        p = NativePlan(prog.arena_bytes, n_streams=2, n_events=2)
        self.native = p
        for t in prog.tensors.values():
            if t.kind == "weight":
                p.upload(t.offset, t.host)
        self.in_slots: Dict[str, int] = {}
        self.out_slots: Dict[str, int] = {}
        if copies:
            for name in prog.inputs:
                t = prog.tensors[name]
                s = p.add_input_slot(t.nbytes)
                self.in_slots[name] = s
                p.h2d(self.COPY, s, 0, t.offset, t.nbytes)
            p.record(self.COPY, 0)
            p.wait(self.COMPUTE, 0)
        descs = {n: prog.desc(n) for n in prog.tensors}
        self.step_of_kernel: List[int] = []
        for i, st in enumerate(prog.steps):
            for ln in st.build(descs):
                p.kernel(self.COMPUTE, ln, st.label)
                self.step_of_kernel.append(i)
        if copies:
            p.record(self.COMPUTE, 1)
            p.wait(self.COPY, 1)
            for name in prog.outputs:
                t = prog.tensors[name]
                s = p.add_output_slot(t.nbytes)
                self.out_slots[name] = s
                p.d2h(self.COPY, s, 0, t.offset, t.nbytes)
        p.finalize(use_graph)

    def upload_inputs(self, feeds: Dict[str, np.ndarray]) -> None:
        for name in self.prog.inputs:
            t = self.prog.tensors[name]
            a = np.ascontiguousarray(feeds[name], NP_OF[t.dtype])
            if a.shape != t.shape:
                raise ValueError(f"input {name!r} shape {a.shape} != planned {t.shape}")
            self.native.upload(t.offset, a)

    def read_outputs(self) -> Dict[str, np.ndarray]:
        out = {}
        for name in self.prog.outputs:
            t = self.prog.tensors[name]
            out[name] = self.native.download(t.offset, np.empty(t.shape, NP_OF[t.dtype]))
        return out

    def input_view(self, name: str) -> np.ndarray:
        t = self.prog.tensors[name]
        return self.native.slot_array(False, self.in_slots[name], NP_OF[t.dtype], t.shape)

    def output_view(self, name: str) -> np.ndarray:
        t = self.prog.tensors[name]
        return self.native.slot_array(True, self.out_slots[name], NP_OF[t.dtype], t.shape)

    @property
    def h2d_bytes(self) -> int:
        return sum(self.prog.tensors[n].nbytes for n in self.prog.inputs)

    @property
    def d2h_bytes(self) -> int:
        return sum(self.prog.tensors[n].nbytes for n in self.prog.outputs)

    def run(self, feeds: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
        if not self.copies:
            self.upload_inputs(feeds)
            self.native.run()
            return self.read_outputs()
        for name in self.prog.inputs:
            self.input_view(name)[...] = feeds[name]
        self.native.run()
        return {n: self.output_view(n).copy() for n in self.prog.outputs}

    def stream(self, batches: Sequence[Dict[str, np.ndarray]]) -> Tuple[List[Dict[str, np.ndarray]], float]:
        """Run one pass per batch, back to back, with each batch's host->device
        copy overlapped with the previous pass (``c3b_plan_stream``).  Batches
        are staged in pinned buffers first; returns the outputs of every pass
        and the device time of the stream in ms."""
        if not self.copies:
            raise RuntimeError("stream() needs an executor built with copies=True")
        import torch
        pins: List[List] = []
        for feeds in batches:
            row = []
            for name in self.prog.inputs:
                t = self.prog.tensors[name]
                a = np.ascontiguousarray(feeds[name], NP_OF[t.dtype])
                if a.shape != t.shape:
                    raise ValueError(f"input {name!r} shape {a.shape} != planned {t.shape}")
                h = torch.from_numpy(a).pin_memory()
                row.append(h)
            pins.append(row)
        outs = [{n: torch.from_numpy(np.empty(self.prog.tensors[n].shape, NP_OF[self.prog.tensors[n].dtype])).pin_memory()
                 for n in self.prog.outputs} for _ in pins]
        ms = self.native.stream([[h.data_ptr() for h in row] for row in pins],
                                [[o[n].data_ptr() for n in self.prog.outputs] for o in outs])
        return [{n: o[n].numpy().copy() for n in self.prog.outputs} for o in outs], ms

    def stream_slots(self, n_steps: int) -> float:
        """``n_steps`` overlapped passes that all read this executor's pinned
        input slots and write its output slots (the benchmark's e2e stream)."""
        ins = [self.native.slot_ptr(False, self.in_slots[n]) for n in self.prog.inputs]
        outs = [self.native.slot_ptr(True, self.out_slots[n]) for n in self.prog.outputs]
        return self.native.stream([ins] * n_steps, [outs] * n_steps)

    def kernel_times(self) -> List[Tuple[str, float]]:
        ms = self.native.run_timed()
        return list(zip(self.native.kernel_labels, ms.tolist()))
