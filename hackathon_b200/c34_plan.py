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

Precision.  Each ``KernelStep`` carries the ``precision_profile`` C3.2 chose
for its node (c34/scheduler.py:173-192, c34/execution_plan.py:65).  Steps
whose profile computes in bf16 or fp16 (one of them per plan) and whose kernel is one of the fused nodes of
``c33_passes`` (or ``fused_gemm_epilogue``, when aligned) run on the tcgen05
kernels: convolutions read and write channels-last 16-bit activations,
linear layers 16-bit rows with an fp32 output where a residual stream or a
graph output needs it, attention reads the packed 16-bit QKV rows.  Weights
of those steps are uploaded in the layout their kernel reads.  Every other
step runs its fp32 kernel; where it consumes a 16-bit or channels-last
tensor, the runner inserts one conversion launch into a slot past the plan's
arena (and global average pooling reads channels-last directly).
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import numpy as np

from . import _lib as L
from .kernels import Desc, Launch, conv_geometry, flash_params_from_node, prepare
from .runtime import NativePlan

_NP_DTYPE = {np.dtype(np.float32): L.F32, np.dtype(np.int64): L.I64, np.dtype(np.int32): L.I32,
             np.dtype(np.uint16): L.BF16}

# kernels of the fused nodes that run on tensor cores in a 16-bit profile
_TC_BASES = ("b200convbiasact", "b200linearepilogue", "b200flashattention", "fused_gemm_epilogue")
_LINEAR_BASES = ("b200linearepilogue", "fused_gemm_epilogue")


def _base(kernel_name: str) -> str:
    for suf in ("_f32", "_fp32", "_bf16", "_fp16"):
        if kernel_name.endswith(suf):
            return kernel_name[: -len(suf)]
    return kernel_name


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


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
                              tuning_params=k.tuning_params, operator_params=dict(k.operator_params),
                              precision_profile=dict(k.precision_profile or {}))
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

    def finalize(self, *a, **k):
        pass


class C34PlanRunner:
    """Native replay of one reference plan for one batch size.

    A kernel whose correctly sized output exceeds the slot C3.4 planned for it
    gets a dedicated slot past the plan's arena ("spill").  This happens for
    ``winograd_forward_f32``: the reference sizes its output for the
    unpadded F(2,3) tiling and the kernel itself raises before writing
    (c32/kernel_registry.py:521,534), so the reference never noticed.

    ``profile`` overrides every step's ``precision_profile`` compute dtype
    ("fp32" replays a 16-bit plan in fp32); by default each step's own
    profile decides.  ``target`` (tests) replaces the native plan with a
    recorder that receives the same actions.
    """

    def __init__(self, plan: Dict[str, Any], host_weights: Dict[str, np.ndarray],
                 input_specs: Dict[str, Tuple[Tuple[int, ...], Any]], use_graph: bool = True,
                 profile: Optional[str] = None, target: Any = None):
        self.plan = plan
        weights = dict(host_weights)
        weights.update(fold_weights(plan.get("folds", {}), host_weights))
        self._weights = weights
        self._specs = input_specs
        self._profile = profile
        stream_ids = sorted({s["stream_id"] for s in plan["timeline"] if s["kind"] not in ("ALLOC", "FREE")})
        self.stream_index = {sid: i for i, sid in enumerate(stream_ids)}
        self.event_index = {eid: i for i, eid in enumerate(plan["events"])}
        self.base = max(256, int(plan["arena_bytes"]))
        self._extra: Dict[str, Tuple[int, int]] = {}
        self._extra_top = self.base
        self.spills: Dict[str, Tuple[int, int]] = {}
        self._analyze()
        self._walk(_DryPlan(), self.base)
        if target is not None:
            self.native = target
            self._walk(target, self.base)
            return
        self.native = NativePlan(self._extra_top, len(stream_ids), len(plan["events"]))
        self._walk(self.native, self.base)
        self.native.finalize(use_graph)

    # ---------------------------------------------------------- analysis
    def _dtype_of(self, ks) -> str:
        if self._profile is not None:
            return self._profile
        pp = ks.get("precision_profile") or {}
        return str(pp.get("compute_dtype") or "fp32")

    def _analyze(self) -> None:
        """Decide, before walking, which steps run on tensor cores, the dtype
        of every output they write, and the layout each weight is uploaded in."""
        steps = self.plan["kernel_steps"]
        outputs = set(self.plan.get("graph_outputs", []))
        cons: Dict[str, List[int]] = {}
        for i, ks in enumerate(steps):
            for nm in ks["logical_inputs"]:
                if nm:
                    cons.setdefault(nm, []).append(i)
        self._tc: Dict[int, bool] = {}
        self._wfmt: Dict[str, str] = {}
        dts = set()
        for i, ks in enumerate(steps):
            base = _base(ks["kernel_name"])
            dt = self._dtype_of(ks)
            tc = base in _TC_BASES and dt in ("bf16", "fp16")
            if tc:
                dts.add(dt)
            ins = ks["logical_inputs"]
            if tc and base == "fused_gemm_epilogue":
                p = ks.get("operator_params") or {}
                w = self._weights.get(ins[1])
                if w is None or w.ndim != 2 or int(p.get("transA", 0)) or float(p.get("alpha", 1.0)) != 1.0 \
                        or float(p.get("beta", 1.0)) != 1.0:
                    tc = False
                else:
                    N, K = (w.shape if int(p.get("transB", 0)) else w.shape[::-1])
                    tc = N % 32 == 0 and K % 64 == 0
                if tc:
                    self._wfmt[ins[1]] = "nk16" if not int(p.get("transB", 0)) else "nk16_t"
            elif tc and base == "b200linearepilogue":
                self._wfmt[ins[1]] = "nk16"
                w = self._weights.get(ins[1])
                if w is None or w.ndim != 2 or w.shape[1] % 32 or w.shape[0] % 64:
                    raise ValueError(f"linear step {ks['node_id']}: weight must be [K, N] with K % 64 == 0, "
                                     f"N % 32 == 0 for the tensor-core path")
            elif tc and base == "b200convbiasact":
                w = self._weights[ins[1]]
                O, C, kh, kw = w.shape
                stem = (ins[0] in self.plan.get("graph_inputs", []) and C % 64 != 0 and C * kh * kw <= 64
                        and O in (16, 32, 64) and (ks.get("operator_params") or {}).get("_residual_input_index")
                        is None)
                self._wfmt[ins[1]] = "stem" if stem else "ohwc16"
                if not stem and C % 64 != 0:
                    raise ValueError(f"conv step {ks['node_id']}: Cin {C} is not a multiple of 64")
            self._tc[i] = tc
        if len(dts) > 1:
            raise ValueError("plan replay: bf16 and fp16 steps in one plan")
        # 16-bit format of the plan's tensor-core steps (bf16 or fp16 profile)
        self.t16 = L.F16 if dts == {"fp16"} else L.BF16
        # output dtypes of the 16-bit steps and of LayerNorms feeding them
        self._out16: Dict[str, bool] = {}

        def feeds_only_tc(name, bases):
            users = cons.get(name, [])
            return bool(users) and name not in outputs and all(
                self._tc[u] and _base(steps[u]["kernel_name"]) in bases
                and steps[u]["logical_inputs"][0] == name for u in users)
        for i, ks in enumerate(steps):
            base = _base(ks["kernel_name"])
            outs = [n for n in ks["logical_outputs"] if n]
            if not outs:
                continue
            o = outs[0]
            p = ks.get("operator_params") or {}
            if self._tc[i] and base in _LINEAR_BASES:
                self._out16[o] = (p.get("_residual_input_index") is None and
                                  feeds_only_tc(o, _LINEAR_BASES + ("b200flashattention",)))
            elif base in ("fused_layer_norm", "fused_residual_norm"):
                self._out16[o] = feeds_only_tc(o, _LINEAR_BASES)

    # ---------------------------------------------------------- helpers
    def _k(self, np_, s: int, ln: Launch, label: str, flops: float = 0.0) -> None:
        np_.kernel(s, ln, label)
        self.launch_flops.append(float(flops))

    def _extra_alloc(self, key: str, nbytes: int) -> int:
        """A slot past the plan's arena (spills and conversions), stable
        across the sizing walk and the real walk."""
        if key not in self._extra:
            need = (int(nbytes) + 255) // 256 * 256
            self._extra[key] = (self._extra_top, need)
            self._extra_top += need
        return self._extra[key][0]

    def _to_f32(self, np_, s, name: str, d: Desc, label: str) -> Desc:
        """The fp32 plain-layout copy of a 16-bit or channels-last tensor."""
        if d.dtype not in (L.BF16, L.F16) and d.layout == "plain":
            return d
        off = self._extra_alloc(f"f32:{name}", d.numel * 4)
        dst = L.make_tensor(off, L.F32, d.shape, True)
        if d.layout == "nhwc":
            N, C, H, W = d.shape
            strides = [H * W * C, 1, W * C, C]  # NCHW coordinates into NHWC storage
        else:
            strides = list(_contig(d.shape))
        cp = L.CopyParams()
        for k, v in enumerate(strides):
            cp.in_stride[k] = int(v)
        src = L.make_tensor(d.ptr, d.dtype, (d.numel,), True)
        self._k(np_, s, Launch(L.K_COPY, [src], [dst], cp), f"{label}:to_f32")
        return Desc(off, L.F32, d.shape, True)

    def _to_16(self, np_, s, name: str, d: Desc, nhwc: bool, label: str) -> Desc:
        """The 16-bit copy of a tensor (the plan's format), channels-last when ``nhwc``."""
        want = "nhwc" if nhwc else "plain"
        if d.dtype == self.t16 and d.layout == want:
            return d
        src = self._to_f32(np_, s, name, d, label) if d.layout != "plain" else d
        off = self._extra_alloc(f"bf16{want}:{name}", d.numel * 2)
        cp = L.CopyParams()
        if nhwc:
            N, C, H, W = d.shape
            oshape = (N, H, W, C)
            strides = [C * H * W, W, 1, H * W]  # NHWC coordinates into NCHW storage
        else:
            oshape = d.shape
            strides = list(_contig(d.shape))
        for k, v in enumerate(strides):
            cp.in_stride[k] = int(v)
        self._k(np_, s, Launch(L.K_COPY, [L.make_tensor(src.ptr, src.dtype, (d.numel,), True)],
                             [L.make_tensor(off, self.t16, oshape, True)], cp), f"{label}:to_16")
        return Desc(off, self.t16, d.shape, True, layout=want)

    def _out_slot(self, allocs, ks, name: str, nbytes: int) -> int:
        a = allocs[ks["outputs"][name]]
        cap = a["capacity_bytes"] or a["size_bytes"]
        if nbytes > cap:
            raise ValueError(f"output '{name}' needs {nbytes} bytes, planned capacity is {cap}")
        return a["offset_bytes"]

    def _bits16(self, x: np.ndarray) -> np.ndarray:
        if self.t16 == L.F16:
            return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)
        return _bf16_bits(x)

    def _weight_host(self, name: str, host: np.ndarray) -> np.ndarray:
        fmt = self._wfmt.get(name)
        if fmt is None:
            return host
        w = np.asarray(host, np.float32)
        if fmt == "ohwc16":
            return self._bits16(np.ascontiguousarray(w.transpose(0, 2, 3, 1)))
        if fmt == "stem":
            return np.ascontiguousarray(w.reshape(w.shape[0], -1).T, np.float32)
        if fmt == "nk16":      # [K, N] (MatMul / Gemm transB=0) -> [N, K]
            return self._bits16(np.ascontiguousarray(w.T))
        if fmt == "nk16_t":    # already [N, K] (Gemm transB=1)
            return self._bits16(np.ascontiguousarray(w))
        raise ValueError(fmt)

    # ---------------------------------------------------------- tensor-core steps
    def _tc_step(self, np_, s, ks, ins: List[Optional[Desc]], allocs, values) -> None:
        base = _base(ks["kernel_name"])
        p = ks.get("operator_params") or {}
        label = ks["kernel_name"]
        out = [n for n in ks["logical_outputs"] if n][0]
        if base == "b200convbiasact":
            x, w, b = ins[0], ins[1], ins[2]
            ri = p.get("_residual_input_index")
            res = ins[int(ri)] if ri is not None else None
            O, C, kh, kw = self._weights[ks["logical_inputs"][1]].shape
            N, Cx, H, W = x.shape
            if Cx != C or int(p.get("group", 1)) != 1:
                raise ValueError(f"conv step {ks['node_id']}: channel mismatch or grouped conv")
            geo, Ho, Wo = conv_geometry(p, H, W, kh, kw)
            act = L.ACT_RELU if p.get("_activation") == "Relu" else L.ACT_NONE
            M = N * Ho * Wo
            off = self._out_slot(allocs, ks, out, M * O * 2)
            if self._wfmt[ks["logical_inputs"][1]] == "stem":
                x = self._to_f32(np_, s, ks["logical_inputs"][0], x, label)
                sp = L.StemParams()
                sp.n, sp.c, sp.h, sp.w, sp.ho, sp.wo, sp.kpad = N, C, H, W, Ho, Wo, 0
                sp.g = geo
                self._k(np_, s, Launch(L.K_STEM_CONV, [x.t(), w.t(), b.t((O,))],
                                       [L.make_tensor(off, self.t16, (M, O), True)], L.StemConvParams(sp, O, act)),
                        label + ":stem", 2.0 * M * O * C * kh * kw)
            else:
                if kh != kw or geo.ph0 != geo.ph1 or geo.pw0 != geo.ph0 or geo.sh != geo.sw or geo.dh != 1:
                    raise NotImplementedError("tc conv: square kernels, symmetric padding, equal strides")
                x = self._to_16(np_, s, ks["logical_inputs"][0], x, True, label)
                tin = [x.t((N * H * W, C)), w.t(), b.t((O,))]
                if res is not None:
                    res = self._to_16(np_, s, ks["logical_inputs"][int(ri)], res, True, label)
                    tin.append(res.t((M, O)))
                cp = L.ConvTcParams()
                cp.n, cp.h, cp.w, cp.cin, cp.cout, cp.ho, cp.wo = N, H, W, C, O, Ho, Wo
                cp.k, cp.stride, cp.pad = kh, geo.sh, geo.ph0
                cp.has_residual, cp.act, cp.block_n, cp.mode = int(res is not None), act, 0, 0
                self._k(np_, s, Launch(L.K_CONV_TC, tin, [L.make_tensor(off, self.t16, (M, O), True)], cp), label,
                        2.0 * M * O * C * kh * kw)
            values[out] = Desc(off, self.t16, (N, O, Ho, Wo), True, layout="nhwc")
            return
        if base in _LINEAR_BASES:
            x, w = ins[0], ins[1]
            bias = ins[2] if len(ins) > 2 and ins[2] is not None else None
            ri = p.get("_residual_input_index")
            res = ins[int(ri)] if ri is not None else None
            if base == "fused_gemm_epilogue":
                fa = p.get("_flatten_axis")
                shp = x.shape
                if fa is not None:
                    ax = int(fa) % len(shp) if int(fa) < 0 else int(fa)
                    shp = (int(np.prod(shp[:ax], dtype=np.int64)), int(np.prod(shp[ax:], dtype=np.int64)))
                lead, K = tuple(shp[:-1]), shp[-1]
            else:
                lead, K = tuple(x.shape[:-1]), x.shape[-1]
            N = w.shape[0]
            M = int(np.prod(lead, dtype=np.int64))
            act = {"Relu": L.ACT_RELU, "Gelu": L.ACT_GELU}.get(p.get("_activation"), L.ACT_NONE)
            if act == L.ACT_GELU:
                vals = [float(np.asarray(self._weights[c]).reshape(-1)[0]) for c in p.get("_gelu_constants", [])]
                if len(vals) != 3 or abs(vals[0] - 2 ** 0.5) > 1e-6 or vals[1] != 1.0 or vals[2] != 0.5:
                    raise ValueError(f"linear step {ks['node_id']}: the GELU chain's constants are not "
                                     f"(sqrt 2, 1, 0.5): {vals}")
            x = self._to_16(np_, s, ks["logical_inputs"][0], Desc(x.ptr, x.dtype, (M, K), True, layout=x.layout)
                            if x.layout == "plain" else x, False, label)
            odt = self.t16 if self._out16.get(out) else L.F32
            off = self._out_slot(allocs, ks, out, M * N * L.DTYPE_SIZE[odt])
            g = L.GemmTcParams()
            g.M, g.N, g.K = M, N, K
            g.bias_mode = L.BIAS_COL if bias is not None else L.BIAS_NONE
            g.act, g.has_residual, g.block_n = act, int(res is not None), 0
            tin = [x.t((M, K)), w.t()] + ([bias.t((N,))] if bias is not None else [])
            if res is not None:
                if res.layout != "plain":
                    res = self._to_f32(np_, s, ks["logical_inputs"][int(ri)], res, label)
                tin.append(res.t((M, N)))
            self._k(np_, s, Launch(L.K_GEMM_TC, tin, [L.make_tensor(off, odt, (M, N), True)], g), label,
                    2.0 * M * N * K)
            values[out] = Desc(off, odt, lead + (N,), True)
            return
        if base == "b200flashattention":
            qkv = self._to_16(np_, s, ks["logical_inputs"][0], ins[0], False, label)
            fp = flash_params_from_node(qkv, ins[1], ins[2], ins[3], p)
            shape = (fp.batch, fp.seq, fp.heads * fp.head_dim)
            off = self._out_slot(allocs, ks, out, int(np.prod(shape)) * 2)
            self._k(np_, s, Launch(L.K_FLASH_ATTN, [qkv.t()], [L.make_tensor(off, self.t16, shape, True)], fp), label,
                    4.0 * fp.batch * fp.heads * fp.seq * fp.seq * fp.head_dim * (0.5 if fp.causal else 1.0))
            values[out] = Desc(off, self.t16, shape, True)
            return
        raise NotImplementedError(base)

    # ---------------------------------------------------------- walk
    def _walk(self, np_, base: int) -> None:
        plan, weights, input_specs = self.plan, self._weights, self._specs
        allocs = {a["alloc_id"]: a for a in plan["allocations"]}
        values: Dict[str, Desc] = {}
        self.launch_flops: List[float] = []  # per kernel launch, in launch order (roofline accounting)
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
                    orig = np.ascontiguousarray(weights[name])
                    host = np.ascontiguousarray(self._weight_host(name, orig))
                    if host.dtype not in _NP_DTYPE:
                        host = host.astype(np.float32)
                    if host.nbytes > cap:
                        raise ValueError(f"'{name}' requires {host.nbytes} bytes, planned capacity is {cap}")
                    # Model tensors are uploaded once and stay resident (executor.py:805-839).
                    np_.upload(a["offset_bytes"], host)
                    dt = self.t16 if host.dtype == np.uint16 else _NP_DTYPE[host.dtype]
                    values[name] = Desc(a["offset_bytes"], dt, tuple(host.shape), True, host=orig)
            elif kind == "KERNEL":
                idx = step["ref_index"]
                ks = plan["kernel_steps"][idx]
                ins: List[Optional[Desc]] = []
                for nm in ks["logical_inputs"]:
                    if not nm:
                        ins.append(None)
                    elif nm not in values:
                        raise KeyError(f"Kernel '{ks['kernel_name']}' (node '{ks['node_id']}') requires "
                                       f"unavailable input '{nm}'")
                    else:
                        ins.append(values[nm])
                if self._tc.get(idx):
                    self._tc_step(np_, s, ks, ins, allocs, values)
                    continue
                self._fp32_step(np_, s, ks, ins, allocs, values, base)
            elif kind == "D2H":
                tr = plan["transfers"][step["ref_index"]]
                name = tr["tensor_name"]
                if name not in values:
                    raise KeyError(f"D2H source '{name}' is unavailable")
                d = values[name]
                if d.dtype != L.F32 or d.layout != "plain":
                    d = self._to_f32(np_, s, name, d, "d2h")
                nbytes = d.numel * L.DTYPE_SIZE[d.dtype]
                slot = np_.add_output_slot(nbytes)
                np_dt = {L.F32: np.float32, L.I64: np.int64, L.I32: np.int32}[d.dtype]
                self.output_slots[name] = (slot, d.shape, np.dtype(np_dt))
                np_.d2h(s, slot, 0, d.ptr, nbytes)
            else:
                raise ValueError(f"Unsupported timeline action: {kind}")
        self.values = values

    def _fp32_step(self, np_, s, ks, ins, allocs, values, base) -> None:
        name = ks["kernel_name"]
        if name.endswith(("_bf16", "_fp16")):  # a 16-bit step replayed in fp32
            name = _base(name) + "_f32"
        onames = [n for n in ks["logical_outputs"] if n]
        params = ks.get("operator_params") or {}
        # Global average pooling reads channels-last activations directly.
        if _base(name) in ("reduce_mean",) and ins and ins[0] is not None and ins[0].layout == "nhwc" \
                and sorted(int(a) % 4 for a in (params.get("axes") or [2, 3])) == [2, 3]:
            x = ins[0]
            N, C, H, W = x.shape
            off = self._out_slot(allocs, ks, onames[0], N * C * 4)
            keep = int(params.get("keepdims", 1))
            self._k(np_, s, Launch(L.K_GAP_NHWC, [x.t((N, H * W, C))], [L.make_tensor(off, L.F32, (N, C), True)],
                                 L.GapParams(N, H * W, C)), name)
            values[onames[0]] = Desc(off, L.F32, (N, C, 1, 1) if keep else (N, C), True)
            return
        ins = [None if d is None else self._to_f32(np_, s, nm, d, name)
               for nm, d in zip(ks["logical_inputs"], ins)]

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
        try:
            prep = prepare(name, ins, outs, params)
        except ValueError as e:
            if "Output arena too small" not in str(e) or not isinstance(np_, _DryPlan):
                raise
            big = [Desc(0, L.F32, (1 << 40,), True) for _ in onames]
            prep = prepare(name, ins, big, params)
            for nm, shp in zip(onames, prep.out_shapes):
                need = (int(np.prod(shp)) * 4 + 255) // 256 * 256
                self.spills[nm] = (self._extra_alloc(f"spill:{nm}", need), need)
            outs = out_descs()
            prep = prepare(name, ins, outs, params)
        o16 = len(onames) == 1 and self._out16.get(onames[0]) and len(prep.launches) == 1 and \
            prep.launches[0].kid == L.K_LAYERNORM
        if o16:  # the LayerNorm feeds only tensor-core linears: write bf16 rows
            prep.launches[0].outs[0].dtype = self.t16
        for ln in prep.launches:
            self._k(np_, s, ln, name)
        k = 0
        for ln in prep.launches:
            for t in ln.outs:
                if k < len(onames):
                    values[onames[k]] = Desc(outs[k].ptr, int(t.dtype), tuple(prep.out_shapes[k]), True)
                k += 1

    def run(self, feeds: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
        for name, (slot, shape, dt) in self.input_slots.items():
            arr = np.asarray(feeds[name])
            if tuple(arr.shape) != shape:
                raise ValueError(f"input {name!r} shape {arr.shape} != planned {shape}")
            self.native.slot_array(False, slot, dt, shape)[...] = arr
        self.native.run()
        return {name: self.native.slot_array(True, slot, dt, shape).copy()
                for name, (slot, shape, dt) in self.output_slots.items()}


def _contig(shape):
    st, acc = [], 1
    for d in reversed(shape):
        st.append(acc)
        acc *= int(d)
    return list(reversed(st))
