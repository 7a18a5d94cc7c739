"""Python handle over the native plan executor (``c3b_plan_*``).

A :class:`NativePlan` owns one device arena, a set of CUDA streams and events,
pinned input/output staging and an ordered action list — the runtime half of
the reference's ``PlannedGraphExecutor.run_planned`` (c35/executor.py:723-903),
executed natively (and, once finalized, optionally as one CUDA graph).
"""

from __future__ import annotations

import ctypes as C
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib as L
from .kernels import Launch

_NP_OF = {L.F32: np.float32, L.I64: np.int64, L.I32: np.int32, L.F16: np.float16, L.U8: np.uint8,
          L.BF16: np.uint16}


class NativePlan:
    def __init__(self, arena_bytes: int, n_streams: int = 1, n_events: int = 0):
        self._L = L.lib()
        h = C.c_void_p()
        L.check(self._L.c3b_plan_create(C.byref(h), int(arena_bytes), int(n_streams), int(n_events)), "plan_create")
        self.h = h
        self.arena_bytes = int(arena_bytes)
        self.n_streams = n_streams
        self.kernel_ids: List[int] = []
        self.kernel_labels: List[str] = []
        self._in_slots: List[Tuple[int, int]] = []   # (bytes, dtype)
        self._out_slots: List[Tuple[int, int]] = []
        self.finalized = False

    # -------------------------------------------------------------- build
    def upload(self, offset: int, host: np.ndarray) -> None:
        a = np.ascontiguousarray(host)
        L.check(self._L.c3b_plan_upload(self.h, int(offset), a.ctypes.data_as(C.c_void_p), a.nbytes), "plan_upload")

    def download(self, offset: int, out: np.ndarray) -> np.ndarray:
        assert out.flags["C_CONTIGUOUS"]
        L.check(self._L.c3b_plan_download(self.h, int(offset), out.ctypes.data_as(C.c_void_p), out.nbytes),
                "plan_download")
        return out

    def add_input_slot(self, nbytes: int) -> int:
        s = L.check(self._L.c3b_plan_add_input_slot(self.h, int(nbytes)), "add_input_slot")
        self._in_slots.append((int(nbytes), 0))
        return s

    def add_output_slot(self, nbytes: int) -> int:
        s = L.check(self._L.c3b_plan_add_output_slot(self.h, int(nbytes)), "add_output_slot")
        self._out_slots.append((int(nbytes), 0))
        return s

    def h2d(self, stream: int, slot: int, slot_off: int, arena_off: int, nbytes: int) -> None:
        L.check(self._L.c3b_plan_add_h2d(self.h, stream, slot, int(slot_off), int(arena_off), int(nbytes)), "add_h2d")

    def d2h(self, stream: int, slot: int, slot_off: int, arena_off: int, nbytes: int) -> None:
        L.check(self._L.c3b_plan_add_d2h(self.h, stream, slot, int(slot_off), int(arena_off), int(nbytes)), "add_d2h")

    def record(self, stream: int, event: int) -> None:
        L.check(self._L.c3b_plan_add_record(self.h, stream, event), "add_record")

    def wait(self, stream: int, event: int) -> None:
        L.check(self._L.c3b_plan_add_wait(self.h, stream, event), "add_wait")

    def kernel(self, stream: int, ln: Launch, label: str = "") -> None:
        ia, oa = L.tensor_array(ln.ins), L.tensor_array(ln.outs)
        pp = C.byref(ln.params) if ln.params is not None else None
        plen = C.sizeof(ln.params) if ln.params is not None else 0
        L.check(self._L.c3b_plan_add_kernel(self.h, stream, ln.kid, ia, len(ln.ins), oa, len(ln.outs), pp, plen),
                f"add_kernel {label or L.KERNEL_NAMES.get(ln.kid)}")
        self.kernel_ids.append(ln.kid)
        self.kernel_labels.append(label or L.KERNEL_NAMES.get(ln.kid, str(ln.kid)))

    def finalize(self, use_graph: bool = True) -> None:
        L.check(self._L.c3b_plan_finalize(self.h, int(bool(use_graph))), "plan_finalize")
        self.finalized = True

    # -------------------------------------------------------------- run
    def slot_array(self, is_output: bool, slot: int, dtype, shape) -> np.ndarray:
        """NumPy view over a pinned staging slot (no copy)."""
        ptr = self._L.c3b_plan_slot_ptr(self.h, int(is_output), slot)
        if not ptr:
            raise RuntimeError("invalid staging slot")
        dt = np.dtype(dtype)
        n = int(np.prod(shape, dtype=np.int64)) if len(shape) else 1
        buf = (C.c_char * (n * dt.itemsize)).from_address(ptr)
        return np.frombuffer(buf, dtype=dt, count=n).reshape(shape)

    def launch(self) -> None:
        L.check(self._L.c3b_plan_launch(self.h), "plan_launch")

    def sync(self, timeout_s: float = 600.0) -> None:
        L.check(self._L.c3b_plan_sync(self.h, float(timeout_s)), "plan_sync")

    def run(self) -> None:
        L.check(self._L.c3b_plan_run(self.h), "plan_run")

    def run_timed(self) -> np.ndarray:
        n = len(self.kernel_ids)
        arr = (C.c_float * max(1, n))()
        L.check(self._L.c3b_plan_run_timed(self.h, arr, n), "plan_run_timed")
        return np.array(arr[:n], dtype=np.float64)

    def stream(self, in_ptrs: Sequence[Sequence[int]], out_ptrs: Sequence[Sequence[int]]) -> float:
        """Run ``len(in_ptrs)`` passes back to back with host copies overlapped
        (``c3b_plan_stream``).  ``in_ptrs[k][i]`` is pass k's host source for
        input slot i, ``out_ptrs[k][j]`` its host destination for output slot j.
        Returns the device time of the whole stream in ms."""
        n = len(in_ptrs)
        if len(out_ptrs) != n:
            raise ValueError("in_ptrs and out_ptrs need one entry per pass")
        flat_in = [int(p) for row in in_ptrs for p in row]
        flat_out = [int(p) for row in out_ptrs for p in row]
        ia = (C.c_void_p * max(1, len(flat_in)))(*flat_in)
        oa = (C.c_void_p * max(1, len(flat_out)))(*flat_out)
        ms = C.c_float(0.0)
        L.check(self._L.c3b_plan_stream(self.h, n, ia, oa, C.byref(ms)), "plan_stream")
        return float(ms.value)

    def slot_ptr(self, is_output: bool, slot: int) -> int:
        return int(self._L.c3b_plan_slot_ptr(self.h, int(is_output), slot) or 0)

    @property
    def origin_stream(self) -> int:
        return int(self._L.c3b_plan_origin_stream(self.h) or 0)

    @property
    def arena_ptr(self) -> int:
        return int(self._L.c3b_plan_arena(self.h) or 0)

    def close(self) -> None:
        if self.h:
            self._L.c3b_plan_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
