"""Backend lowering: workload graph -> fused B200 program.

This is the backend's own fusion + lowering, applied after (and in the spirit
of) the reference's C3.3 passes (c33/pipeline.py:108-119), which stop short of
one-launch convolutions and attention (the "next" fusions the reference
leaves open: fuse_conv_epilogues only matches a plain Conv,
c33/fusion.py:1135-1136, and attention keeps the [B,H,S,S] score tensor).
Patterns recognised on the unfused ONNX graph:

* Conv -> BatchNormalization [-> Relu | -> Add(shortcut) -> Relu]: BN folded on
  the host with the executor's formula (c35/executor.py:400-411); bias,
  residual and ReLU run in the conv epilogue.
* Gemm [-> Relu]: one GEMM with bias/ReLU epilogue (fused_gemm_epilogue_f32).
* GlobalAveragePool -> Flatten: one pooling kernel; Flatten is a view.
* Gather(token table, ids) -> Add(position table): one embedding kernel.
* MatMul(W) -> Add(b) [-> exact-erf GELU chain] [-> Add(residual)]: one GEMM.
* Split -> 3x(Reshape -> Transpose) -> MatMul -> Div -> Add(causal mask) ->
  Softmax -> MatMul -> Transpose -> Reshape: one flash-attention kernel reading
  the packed QKV projection.
* LayerNormalization -> Gather(axis=1, const) -> Flatten: the row selection
  moves in front of the (row-wise) LayerNorm.

Precision profiles: ``fp32`` keeps IEEE FP32 math everywhere (SIMT FFMA
contractions); ``tf32`` is ``fp32`` with the linear layers (N % 32 == 0,
K % 4 == 0) on tcgen05 ``kind::tf32`` (fp32 operands read with a 10-bit
mantissa, fp32 accumulation), convolutions and attention still fp32 SIMT;
``fp16`` is ``bf16`` with fp16 in place of bf16 (tcgen05
``kind::f16`` with fp16 operands, fp16 activations, the same fp32
accumulation, residual stream and logits); ``bf16`` runs contractions on tcgen05 with bf16 operands and
fp32 accumulation, NHWC bf16 activations for convolutions, an fp32 residual
stream and fp32 LayerNorm statistics for transformers, fp32 logits (the
classifier head of ``bf16`` / ``fp16`` runs on ``kind::tf32`` from an f32
LayerNorm output, as the ResNet classifier stays fp32); ``fp8``
is ``bf16`` with the linear layers the reference's precision policy marks fp8
(aligned GEMMs with K, N >= 64: c32/strategy.py:147-157) run as rowwise-scaled
E4M3 GEMMs — a quantisation step for the activation rows, E4M3 weights with
per-output-row scales, tcgen05 ``kind::f8f6f4`` with fp32 accumulation and the
two scales applied in the epilogue; ``mixed`` applies the whole GEMM policy
(c32/strategy.py:146-157) for a device that supports fp8 and fp4: constant-weight
GEMMs with K, N >= 128, K and N multiples of 32 and K*N >= 32768 run W4A16
(FP4 E2M1 weights in groups of 16 with fp32 scales, expanded to fp16 in
shared memory next to the MMA), other aligned GEMMs with K, N >= 64 run fp8,
the rest fp16 (its 16-bit activations are fp16 throughout, the policy's
activation format, c32/strategy.py:102-108).
"""

from __future__ import annotations

import math
import os
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import _lib as L
from .graph import ModelGraph
from .kernels import Desc, Launch, conv_geometry
from .program import Program


# W4A16 GEMMs with at least this many rows expand their FP4 weights to bf16
# once per pass (C3B_K_DEQUANT_FP4, ~N*K*2.5 bytes of traffic) and run the bf16
# GEMM; fewer rows use the fused kernel, whose converter warps re-expand the
# weights for every 128-row tile but read only the packed FP4 bytes.  Measured
# on B200: fused Tx-large QKV (M = 131072) 1.58 ms vs bf16 GEMM 0.73 ms, the
# expansion ~3 us; the fused path wins only where weight bandwidth dominates.
W4A16_EXPAND_ROWS = 2048


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (round to nearest even), as uint16."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    return r


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


class _State:
    def __init__(self, graph: ModelGraph, batch: int, profile: str):
        if profile not in ("fp32", "tf32", "bf16", "fp16", "fp8", "mixed"):
            raise ValueError(f"unknown precision profile {profile!r}")
        # 16-bit format of tensor-core operands and 16-bit activations: fp16 for
        # the fp16 profile and for `mixed` (the reference policy's activation
        # format, c32/strategy.py:102-108), bf16 otherwise
        self.t16 = L.F16 if profile in ("fp16", "mixed") else L.BF16
        self.g = graph
        self.batch = batch
        self.profile = profile
        self.prog = Program(f"{graph.name}_{profile}_b{batch}")
        self.cons: Dict[str, List[int]] = graph.consumers()
        self.prod: Dict[str, int] = graph.producer()
        self.init = graph.initializers
        self.done = set()
        self.alias: Dict[str, str] = {}   # logical name -> program tensor
        self.layout: Dict[str, str] = {}  # program tensor -> "nchw" | "nhwc" | "rows"
        self.lshape: Dict[str, Tuple[int, ...]] = {}  # logical (ONNX) shape of a program tensor
        self.ops: List[dict] = []         # fused ops before topological ordering
        self.fused_q: Dict[str, Tuple[str, str]] = {}  # LayerNorm output -> (E4M3 bytes, row scales)
        self.wcount = 0

    def node(self, i):
        return self.g.nodes[i]

    def sole(self, tensor: str) -> Optional[int]:
        c = self.cons.get(tensor, [])
        if len(c) != 1 or any(o.name == tensor for o in self.g.outputs) or c[0] in self.done:
            return None
        return c[0]

    def t(self, logical: str) -> str:
        return self.alias.get(logical, logical)

    def bits16(self, x: np.ndarray) -> np.ndarray:
        """float32 -> this profile's 16-bit weight bits (uint16)."""
        if self.t16 == L.F16:
            return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)
        return bf16_bits(x)

    def weight(self, stem: str, host: Optional[np.ndarray], dtype: int, shape=None) -> str:
        self.wcount += 1
        name = f"w{self.wcount}:{stem}"
        self.prog.add_tensor(name, host.shape if host is not None else shape, dtype, "weight", host)
        return name


# ---------------------------------------------------------------- matching

def _match_conv(st: _State, i: int) -> bool:
    n = st.node(i)
    if n.op_type != "Conv":
        return False
    w = st.init[n.inputs[1]]
    b0 = st.init[n.inputs[2]] if len(n.inputs) > 2 and n.inputs[2] else None
    used = [i]
    out = n.outputs[0]
    wf, bf = w, b0 if b0 is not None else np.zeros((w.shape[0],), np.float32)
    j = st.sole(out)
    if j is not None and st.node(j).op_type == "BatchNormalization":
        bn = st.node(j)
        sc, be, mu, var = (st.init[x] for x in bn.inputs[1:5])
        eps = float(bn.attrs.get("epsilon", 1e-5))
        factor = (sc / np.sqrt(var + np.float32(eps))).astype(np.float32)
        wf = (w * factor.reshape(-1, 1, 1, 1)).astype(np.float32)
        bf = ((bf - mu) * factor + be).astype(np.float32)
        used.append(j)
        out = bn.outputs[0]
    act, res = L.ACT_NONE, None
    j = st.sole(out)
    if j is not None and st.node(j).op_type == "Relu":
        act = L.ACT_RELU
        used.append(j)
        out = st.node(j).outputs[0]
    elif j is not None and st.node(j).op_type == "Add":
        add = st.node(j)
        other = add.inputs[1] if add.inputs[0] == out else add.inputs[0]
        k = st.sole(add.outputs[0])
        if other not in st.init and k is not None and st.node(k).op_type == "Relu":
            res = other
            act = L.ACT_RELU
            used += [j, k]
            out = st.node(k).outputs[0]
    st.done.update(used)
    st.ops.append(dict(kind="conv", x=n.inputs[0], w=wf, b=bf, res=res, act=act, out=out, attrs=n.attrs))
    return True


def _match_gemm(st: _State, i: int) -> bool:
    n = st.node(i)
    if n.op_type != "Gemm":
        return False
    a = n.attrs
    if int(a.get("transA", 0)):
        raise NotImplementedError("Gemm transA=1 is not lowered")
    w = st.init[n.inputs[1]]
    w_nk = w if int(a.get("transB", 0)) else np.ascontiguousarray(w.T)  # [N, K]
    b = st.init.get(n.inputs[2]) if len(n.inputs) > 2 else None
    out, used, act = n.outputs[0], [i], L.ACT_NONE
    j = st.sole(out)
    if j is not None and st.node(j).op_type == "Relu":
        act, out = L.ACT_RELU, st.node(j).outputs[0]
        used.append(j)
    st.done.update(used)
    st.ops.append(dict(kind="linear", x=n.inputs[0], w=w_nk, b=b, alpha=float(a.get("alpha", 1.0)),
                       beta=float(a.get("beta", 1.0)), act=act, res=None, out=out, gemm=True))
    return True


def _match_gap(st: _State, i: int) -> bool:
    n = st.node(i)
    if n.op_type != "GlobalAveragePool":
        return False
    out, used = n.outputs[0], [i]
    j = st.sole(out)
    flat = False
    if j is not None and st.node(j).op_type == "Flatten" and int(st.node(j).attrs.get("axis", 1)) == 1:
        out, flat = st.node(j).outputs[0], True
        used.append(j)
    st.done.update(used)
    st.ops.append(dict(kind="gap", x=n.inputs[0], out=out, flat=flat))
    return True


def _match_embed(st: _State, i: int) -> bool:
    n = st.node(i)
    if n.op_type != "Gather" or int(n.attrs.get("axis", 0)) != 0 or n.inputs[0] not in st.init:
        return False
    j = st.sole(n.outputs[0])
    if j is None or st.node(j).op_type != "Add":
        return False
    add = st.node(j)
    pos = add.inputs[1] if add.inputs[0] == n.outputs[0] else add.inputs[0]
    if pos not in st.init:
        return False
    st.done.update([i, j])
    st.ops.append(dict(kind="embed", ids=n.inputs[1], tok=st.init[n.inputs[0]], pos=st.init[pos],
                       out=add.outputs[0]))
    return True


def _is_gelu_chain(st: _State, f: str) -> Tuple[Optional[str], List[int]]:
    """Div(f, sqrt2) -> Erf -> Add(1) -> Mul(f, .) -> Mul(., 0.5); returns the output."""
    used = []
    j = None
    cons = st.cons.get(f, [])
    if len(cons) != 2:
        return None, []
    div = next((c for c in cons if st.node(c).op_type == "Div"), None)
    mul = next((c for c in cons if st.node(c).op_type == "Mul"), None)
    if div is None or mul is None:
        return None, []
    dn = st.node(div)
    if not np.allclose(st.init.get(dn.inputs[1], np.array([0.0])), math.sqrt(2.0), rtol=1e-6):
        return None, []
    e = st.sole(dn.outputs[0])
    if e is None or st.node(e).op_type != "Erf":
        return None, []
    a = st.sole(st.node(e).outputs[0])
    if a is None or st.node(a).op_type != "Add":
        return None, []
    an = st.node(a)
    one = an.inputs[1] if an.inputs[0] == st.node(e).outputs[0] else an.inputs[0]
    if not np.allclose(st.init.get(one, np.array([0.0])), 1.0):
        return None, []
    if st.sole(an.outputs[0]) != mul:
        return None, []
    h = st.sole(st.node(mul).outputs[0])
    if h is None or st.node(h).op_type != "Mul":
        return None, []
    hn = st.node(h)
    half = hn.inputs[1] if hn.inputs[0] == st.node(mul).outputs[0] else hn.inputs[0]
    if not np.allclose(st.init.get(half, np.array([0.0])), 0.5):
        return None, []
    return hn.outputs[0], [div, e, a, mul, h]


def _match_linear(st: _State, i: int) -> bool:
    n = st.node(i)
    if n.op_type != "MatMul" or n.inputs[1] not in st.init:
        return False
    w = st.init[n.inputs[1]]
    if w.ndim != 2:
        return False
    out, used, b, act, res = n.outputs[0], [i], None, L.ACT_NONE, None
    j = st.sole(out)
    if j is not None and st.node(j).op_type == "Add":
        add = st.node(j)
        other = add.inputs[1] if add.inputs[0] == out else add.inputs[0]
        if other in st.init and st.init[other].shape == (w.shape[1],):
            b, out = st.init[other], add.outputs[0]
            used.append(j)
    g_out, g_used = _is_gelu_chain(st, out)
    if g_out is not None:
        act, out = L.ACT_GELU, g_out
        used += g_used
    j = st.sole(out)
    if act == L.ACT_NONE and j is not None and st.node(j).op_type == "Add":
        add = st.node(j)
        other = add.inputs[1] if add.inputs[0] == out else add.inputs[0]
        if other not in st.init:
            res, out = other, add.outputs[0]
            used.append(j)
    st.done.update(used)
    st.ops.append(dict(kind="linear", x=n.inputs[0], w=np.ascontiguousarray(w.T), b=b, alpha=1.0, beta=1.0,
                       act=act, res=res, out=out, gemm=False))
    return True


def _match_attention(st: _State, i: int) -> bool:
    n = st.node(i)
    if n.op_type != "Split" or len(n.outputs) != 3:
        return False
    qkv = n.inputs[0]
    heads4 = []
    used = [i]
    for k, o in enumerate(n.outputs):
        r = st.sole(o)
        if r is None or st.node(r).op_type != "Reshape":
            return False
        tr = st.sole(st.node(r).outputs[0])
        if tr is None or st.node(tr).op_type != "Transpose":
            return False
        heads4.append((st.node(r), st.node(tr)))
        used += [r, tr]
    shp = [int(v) for v in st.init[heads4[0][0].inputs[1]].reshape(-1)]
    H, D = shp[2], shp[3]
    q_t, k_t, v_t = (t.outputs[0] for _, t in heads4)
    if heads4[0][1].attrs.get("perm") != [0, 2, 1, 3] or heads4[1][1].attrs.get("perm") != [0, 2, 3, 1] \
            or heads4[2][1].attrs.get("perm") != [0, 2, 1, 3]:
        return False
    mm = st.sole(q_t)
    if mm is None or st.node(mm).op_type != "MatMul" or st.node(mm).inputs != [q_t, k_t]:
        return False
    dv = st.sole(st.node(mm).outputs[0])
    ad = st.sole(st.node(dv).outputs[0]) if dv is not None and st.node(dv).op_type == "Div" else None
    sm = st.sole(st.node(ad).outputs[0]) if ad is not None and st.node(ad).op_type == "Add" else None
    pv = st.sole(st.node(sm).outputs[0]) if sm is not None and st.node(sm).op_type == "Softmax" else None
    if pv is None or st.node(pv).op_type != "MatMul" or st.node(pv).inputs[1] != v_t:
        return False
    tr = st.sole(st.node(pv).outputs[0])
    rs = st.sole(st.node(tr).outputs[0]) if tr is not None and st.node(tr).op_type == "Transpose" else None
    if rs is None or st.node(rs).op_type != "Reshape":
        return False
    divisor = float(np.asarray(st.init[st.node(dv).inputs[1]]).reshape(-1)[0])
    addn = st.node(ad)
    mask_name = addn.inputs[1] if addn.inputs[0] == st.node(dv).outputs[0] else addn.inputs[0]
    mask = np.asarray(st.init[mask_name], np.float32)
    S = mask.shape[-1]
    ref = np.triu(np.full((S, S), -1e9, np.float32), 1)
    causal = mask.reshape(-1, S, S).shape[0] == 1 and np.array_equal(mask.reshape(S, S), ref)
    if not causal and np.any(mask):
        raise NotImplementedError("attention lowering: only an all-zero or causal (0/-1e9) mask is supported")
    used += [mm, dv, ad, sm, pv, tr, rs]
    st.done.update(used)
    st.ops.append(dict(kind="attention", x=qkv, heads=H, head_dim=D, scale=1.0 / divisor, causal=int(causal),
                       out=st.node(rs).outputs[0]))
    return True


def _match_ln(st: _State, i: int) -> bool:
    n = st.node(i)
    if n.op_type != "LayerNormalization":
        return False
    if int(n.attrs.get("axis", -1)) not in (-1,):
        raise NotImplementedError("LayerNormalization lowering: last-axis only")
    scale = st.init[n.inputs[1]]
    bias = st.init.get(n.inputs[2]) if len(n.inputs) > 2 else None
    eps = float(n.attrs.get("epsilon", 1e-5))
    out, x = n.outputs[0], n.inputs[0]
    j = st.sole(out)
    if j is not None and st.node(j).op_type == "Gather" and int(st.node(j).attrs.get("axis", 0)) == 1 \
            and st.node(j).inputs[1] in st.init:
        gat = st.node(j)
        idx = [int(v) for v in np.asarray(st.init[gat.inputs[1]]).reshape(-1)]
        k = st.sole(gat.outputs[0])
        if len(idx) == 1 and k is not None and st.node(k).op_type == "Flatten" and \
                int(st.node(k).attrs.get("axis", 1)) == 1:
            st.done.update([i, j, k])
            sel = f"{x}@row{idx[0]}"
            st.ops.append(dict(kind="select", x=x, index=idx[0], out=sel))
            st.ops.append(dict(kind="ln", x=sel, scale=scale, bias=bias, eps=eps, out=st.node(k).outputs[0]))
            return True
    st.done.add(i)
    st.ops.append(dict(kind="ln", x=x, scale=scale, bias=bias, eps=eps, out=out))
    return True


def _match_relu_add(st: _State, i: int) -> bool:
    n = st.node(i)
    if n.op_type == "Relu":
        st.done.add(i)
        st.ops.append(dict(kind="ew", prog=[(L.OP_RELU, 0, 0)], xs=[n.inputs[0]], out=n.outputs[0]))
        return True
    if n.op_type == "Add" and not any(x in st.init for x in n.inputs):
        st.done.add(i)
        st.ops.append(dict(kind="ew", prog=[(L.OP_ADD, 0, 1)], xs=list(n.inputs), out=n.outputs[0]))
        return True
    return False


_MATCHERS = [_match_conv, _match_gemm, _match_gap, _match_embed, _match_attention, _match_linear, _match_ln,
             _match_relu_add]


def _toposort(ops: List[dict], graph_inputs: List[str]) -> List[dict]:
    def ins(o):
        k = o["kind"]
        if k == "conv":
            return [o["x"]] + ([o["res"]] if o["res"] else [])
        if k == "linear":
            return [o["x"]] + ([o["res"]] if o["res"] else [])
        if k == "embed":
            return [o["ids"]]
        if k == "ew":
            return list(o["xs"])
        return [o["x"]]
    avail = set(graph_inputs)
    pending = list(ops)
    out = []
    while pending:
        for idx, o in enumerate(pending):
            if all(t in avail for t in ins(o)):
                out.append(o)
                avail.add(o["out"])
                pending.pop(idx)
                break
        else:
            raise RuntimeError("lowering: fused ops have a dependency cycle or a missing producer")
    return out


# ---------------------------------------------------------------- emission

def _gemm_simt_launch(d: Dict[str, Desc], x, w, b, out, M, N, K, act, res=None, alpha=1.0, beta=1.0):
    g = L.GemmParams()
    g.M, g.N, g.K, g.batch = M, N, K, 1
    g.trans_a, g.trans_b, g.alpha, g.beta = 0, 1, alpha, beta
    g.bias_mode = L.BIAS_COL if b else L.BIAS_NONE
    g.act, g.has_residual = act, int(res is not None)
    ins = [d[x].t((M, K)), d[w].t()] + ([d[b].t()] if b else []) + ([d[res].t((M, N))] if res else [])
    return Launch(L.K_GEMM, ins, [d[out].t((M, N))], g)


def _gemm_tc_launch(d: Dict[str, Desc], x, w, b, out, M, N, K, act, res=None):
    g = L.GemmTcParams()
    g.M, g.N, g.K = M, N, K
    g.bias_mode = L.BIAS_COL if b else L.BIAS_NONE
    g.act, g.has_residual, g.block_n = act, int(res is not None), 0
    ins = [d[x].t((M, K)), d[w].t()] + ([d[b].t()] if b else []) + ([d[res].t((M, N))] if res else [])
    return Launch(L.K_GEMM_TC, ins, [d[out].t((M, N))], g)


def _f8_linear(st: _State, op: dict, K: int) -> bool:
    """The fp8 rule of the linear lowering (c32/strategy.py:150-157) for ``op``."""
    N = op["w"].shape[0]
    return (st.profile == "fp8" and N % 32 == 0 and K % 64 == 0 and N % 16 == 0 and K >= 64 and N >= 64
            and op.get("alpha", 1.0) == 1.0)


def _ln_feeds_f8_linear(st: _State, op: dict, cols: int) -> bool:
    """True when the LayerNorm output's only consumer is a linear that takes the
    fp8 path, so the LayerNorm can write E4M3 bytes for it directly."""
    if st.profile != "fp8" or cols not in (128, 256, 512, 1024, 2048):
        return False
    out = op["out"]
    if any(o.name == out for o in st.g.outputs):
        return False
    users = [o for o in st.ops if out in (o.get("x"), o.get("res")) or out in (o.get("xs") or [])]
    return len(users) == 1 and users[0]["kind"] == "linear" and users[0]["x"] == out and _f8_linear(st, users[0], cols)


def _is_output(st: _State, name: str) -> bool:
    return any(o.name == name for o in st.g.outputs)


def _ln_feeds_logits(st: _State, op: dict) -> bool:
    """True in the bf16 / fp16 profiles when every consumer of the LayerNorm
    output (directly or through a row select) is a linear layer producing a
    graph output: the classifier head.  That LayerNorm writes f32 and the head
    runs on kind::tf32, like the ResNet classifier staying in fp32: rounding
    the head's input and weights to bf16 was about a third of the Tx-large
    logit error."""
    if st.profile not in ("bf16", "fp16"):
        return False

    def users(name):
        return [o for o in st.ops if name in (o.get("x"), o.get("res")) or name in (o.get("xs") or [])]

    us = users(op["out"])
    if not us or _is_output(st, op["out"]):
        return False
    for u in us:
        if u["kind"] == "select" and u["x"] == op["out"]:
            vs = users(u["out"])
            if not vs or any(v["kind"] != "linear" or v["x"] != u["out"] or v.get("res") or not _is_output(st, v["out"])
                             for v in vs):
                return False
        elif u["kind"] != "linear" or u["x"] != op["out"] or u.get("res") or not _is_output(st, u["out"]):
            return False
    return True


def _gap_classifier(st: _State, op: dict, C: int):
    """The linear op that is the only consumer of a flattened GAP over NHWC
    16-bit activations, when GAP and it can run as one launch: a classifier
    without activation or residual, at most 32 classes, C a multiple of 256
    up to 1024; else None."""
    if not op.get("flat") or C % 256 or C > 1024 or _is_output(st, op["out"]):
        return None
    users = [o for o in st.ops if op["out"] in (o.get("x"), o.get("res")) or op["out"] in (o.get("xs") or [])]
    if len(users) != 1:
        return None
    u = users[0]
    if u["kind"] != "linear" or u["x"] != op["out"] or u.get("res") or u.get("act", L.ACT_NONE) != L.ACT_NONE:
        return None
    w = u["w"]
    if w.ndim != 2 or w.shape[1] != C or w.shape[0] > 32 or w.shape[0] * C * 4 > 48 * 1024:
        return None
    return u


def _conv_shortcut(st: _State, op: dict, H: int, W: int, geo, O: int):
    """The 1x1 stride-2 convolution on this 3x3 (k odd, pad k/2) stride-2
    convolution's input, when one launch can compute both: the residual
    block's downsampling shortcut samples exactly the centre tap's pixels.
    It must not have been emitted yet, and has the same Cout (64 or 128), no
    activation and no residual.  C3B200_CONV_SHORTCUT=0 keeps two launches."""
    if os.environ.get("C3B200_CONV_SHORTCUT", "1") == "0" or op["res"] or O not in (64, 128):
        return None
    kh = op["w"].shape[2]
    if kh % 2 == 0 or op["w"].shape[3] != kh or geo.sh != 2 or geo.sw != 2 or geo.ph0 != kh // 2:
        return None
    for u in st.ops:
        if u is op or u["kind"] != "conv" or u.get("fused") or u.get("_emitted") or st.t(u["x"]) != st.t(op["x"]):
            continue
        w = u["w"]
        if w.shape != (O, op["w"].shape[1], 1, 1) or u["res"] or u["act"] != L.ACT_NONE:
            continue
        g1, _, _ = conv_geometry(u["attrs"], H, W, 1, 1)
        if g1.sh == 2 and g1.sw == 2 and g1.ph0 == g1.ph1 == g1.pw0 == g1.pw1 == 0 and g1.dh == 1:
            return u
    return None


def _emit(st: _State, op: dict) -> None:
    if op.get("fused"):
        return  # emitted inside the op it was fused into
    op["_emitted"] = True
    P, B, bf = st.prog, st.batch, st.profile in ("bf16", "fp16", "fp8", "mixed")
    T16 = st.t16
    k = op["kind"]
    if k == "conv":
        x = st.t(op["x"])
        lay = st.layout[x]
        shp = st.lshape[x]  # logical NCHW
        N, C, H, W = shp
        w, b = op["w"], op["b"]
        O, _, kh, kw = w.shape
        geo, Ho, Wo = conv_geometry(op["attrs"], H, W, kh, kw)
        flops = 2.0 * N * Ho * Wo * O * C * kh * kw
        bname = st.weight("bias", b.astype(np.float32), L.F32)
        res = st.t(op["res"]) if op["res"] else None
        out = op["out"]
        if not bf:
            wname = st.weight("conv", w.astype(np.float32), L.F32)
            if lay != "nchw" or (res and st.layout[res] != "nchw"):
                raise RuntimeError("fp32 conv expects NCHW activations")
            P.add_tensor(out, (N, O, Ho, Wo), L.F32)
            cp = L.ConvParams()
            cp.n, cp.c, cp.h, cp.w, cp.cout, cp.ho, cp.wo, cp.layout = N, C, H, W, O, Ho, Wo, 0
            cp.g, cp.has_bias, cp.has_residual, cp.act = geo, 1, int(res is not None), op["act"]

            def build(d, x=x, wname=wname, bname=bname, res=res, out=out, cp=cp):
                ins = [d[x].t(), d[wname].t(), d[bname].t()] + ([d[res].t()] if res else [])
                return [Launch(L.K_CONV, ins, [d[out].t()], cp)]
            P.add_step("conv_f32", [x, wname, bname] + ([res] if res else []), [out], build, flops)
            st.layout[out] = "nchw"
        elif C % 64 != 0 and C * kh * kw <= 64 and O in (16, 32, 64) and not res and lay == "nchw":
            # stem: direct conv from the NCHW f32 input to NHWC bf16 (K = C*kh*kw is tiny)
            wk = np.ascontiguousarray(w.reshape(O, -1).T, np.float32)  # [K (c,r,s)][Cout]
            wname = st.weight("stem", wk, L.F32)
            P.add_tensor(out, (N * Ho * Wo, O), T16)
            sp = L.StemParams()
            sp.n, sp.c, sp.h, sp.w, sp.ho, sp.wo, sp.kpad = N, C, H, W, Ho, Wo, 0
            sp.g = geo
            scp = L.StemConvParams(sp, O, op["act"])

            def bst(d, x=x, wname=wname, bname=bname, out=out, scp=scp):
                return [Launch(L.K_STEM_CONV, [d[x].t(), d[wname].t(), d[bname].t()], [d[out].t()], scp)]
            P.add_step("stem_conv", [x, wname, bname], [out], bst, flops)
            st.layout[out] = "nhwc"
        elif C % 64 != 0:
            # small-Cin conv: patch matrix (K ordered r,s,c; padded to 64) + tcgen05 GEMM
            if lay != "nchw" or res:
                raise RuntimeError("bf16 stem conv expects the NCHW f32 graph input and no residual")
            kpad = (C * kh * kw + 63) // 64 * 64
            wk = np.zeros((O, kpad), np.float32)
            wk[:, :C * kh * kw] = w.transpose(0, 2, 3, 1).reshape(O, -1)
            wname = st.weight("stem", st.bits16(wk), T16)
            cols = P.add_tensor(f"{out}:cols", (N * Ho * Wo, kpad), T16)
            P.add_tensor(out, (N * Ho * Wo, O), T16)
            sp = L.StemParams()
            sp.n, sp.c, sp.h, sp.w, sp.ho, sp.wo, sp.kpad = N, C, H, W, Ho, Wo, kpad
            sp.g = geo

            def b1(d, x=x, cols=cols, sp=sp):
                return [Launch(L.K_STEM_IM2COL, [d[x].t()], [d[cols].t()], sp)]
            P.add_step("stem_im2col", [x], [cols], b1, 0.0)
            M = N * Ho * Wo

            def b2(d, cols=cols, wname=wname, bname=bname, out=out, M=M, O=O, kpad=kpad, act=op["act"]):
                return [_gemm_tc_launch(d, cols, wname, bname, out, M, O, kpad, act)]
            P.add_step("conv_tc_stem", [cols, wname, bname], [out], b2, flops)
            st.layout[out] = "nhwc"
        else:
            if lay != "nhwc":
                raise RuntimeError("bf16 conv expects NHWC bf16 activations")
            wname = st.weight("conv", st.bits16(np.ascontiguousarray(w.transpose(0, 2, 3, 1))), T16)
            P.add_tensor(out, (N * Ho * Wo, O), T16)
            cp = L.ConvTcParams()
            if kh != kw or geo.ph0 != geo.ph1 or geo.pw0 != geo.ph0 or geo.sh != geo.sw or geo.dh != 1:
                raise NotImplementedError("tc conv: square kernels, symmetric padding, equal strides")
            cp.n, cp.h, cp.w, cp.cin, cp.cout, cp.ho, cp.wo = N, H, W, C, O, Ho, Wo
            cp.k, cp.stride, cp.pad = kh, geo.sh, geo.ph0
            cp.has_residual, cp.act, cp.block_n = int(res is not None), op["act"], 0
            # C3B200_CONV_MODE=1 forces one TMA window per tap (A/B comparisons)
            cp.mode = int(os.environ.get("C3B200_CONV_MODE", "0"))
            sc = _conv_shortcut(st, op, H, W, geo, O)
            extra_in, extra_out = [], []
            if sc is not None:
                # the downsampling shortcut rides along: ws [O, C], bs, output [N*Ho*Wo, O]
                sc["fused"] = True
                cp.has_shortcut = 1
                wsn = st.weight("conv", st.bits16(np.ascontiguousarray(sc["w"].reshape(O, C))), T16)
                bsn = st.weight("bias", sc["b"].astype(np.float32), L.F32)
                P.add_tensor(sc["out"], (N * Ho * Wo, O), T16)
                st.layout[sc["out"]] = "nhwc"
                st.lshape[sc["out"]] = (N, O, Ho, Wo)
                extra_in, extra_out = [wsn, bsn], [sc["out"]]
                flops += 2.0 * N * Ho * Wo * O * C

            def build(d, x=x, wname=wname, bname=bname, res=res, out=out, cp=cp, ei=extra_in, eo=extra_out):
                ins = [d[x].t(), d[wname].t(), d[bname].t()] + ([d[res].t()] if res else []) + [d[e].t() for e in ei]
                return [Launch(L.K_CONV_TC, ins, [d[out].t()] + [d[e].t() for e in eo], cp)]
            P.add_step("conv_tc", [x, wname, bname] + ([res] if res else []) + extra_in, [out] + extra_out, build,
                       flops)
            st.layout[out] = "nhwc"
        st.lshape[out] = (N, O, Ho, Wo)
    elif k == "gap":
        x = st.t(op["x"])
        N, C, H, W = st.lshape[x]
        out = op["out"]
        head = _gap_classifier(st, op, C) if st.layout[x] == "nhwc" else None
        if head is not None:
            # GAP and the classifier in one launch (C3B_K_GAP_NHWC with w, b)
            head["fused"] = True
            w = np.ascontiguousarray(head["w"], np.float32) * np.float32(head.get("alpha", 1.0))
            wname = st.weight("gap_fc", w.astype(np.float32), L.F32)
            bname = st.weight("gap_fc_bias", (head["b"] * head.get("beta", 1.0)).astype(np.float32), L.F32) \
                if head["b"] is not None else None
            hout = head["out"]
            ncls = w.shape[0]
            P.add_tensor(hout, (N, ncls), L.F32)
            gp = L.GapParams(N, H * W, C)

            def build_fc(d, x=x, wname=wname, bname=bname, hout=hout, gp=gp):
                ins = [d[x].t(), d[wname].t()] + ([d[bname].t()] if bname else [])
                return [Launch(L.K_GAP_NHWC, ins, [d[hout].t()], gp)]
            P.add_step("gap_fc", [x, wname] + ([bname] if bname else []), [hout], build_fc,
                       2.0 * N * ncls * C)
            st.layout[hout] = "rows"
            st.lshape[hout] = (N, ncls)
            return
        P.add_tensor(out, (N, C), L.F32)
        if st.layout[x] == "nhwc":
            gp = L.GapParams(N, H * W, C)

            def build(d, x=x, out=out, gp=gp):
                return [Launch(L.K_GAP_NHWC, [d[x].t()], [d[out].t()], gp)]
            P.add_step("gap_nhwc", [x], [out], build)
        else:
            rp = L.ReduceParams(N * C, H * W, 1, L.RED_MEAN, 0)

            def build(d, x=x, out=out, rp=rp):
                return [Launch(L.K_REDUCE, [d[x].t()], [d[out].t()], rp)]
            P.add_step("gap_nchw", [x], [out], build)
        st.layout[out] = "rows"
        st.lshape[out] = (N, C) if op["flat"] else (N, C, 1, 1)
    elif k == "embed":
        tok, pos = op["tok"].astype(np.float32), op["pos"].astype(np.float32)
        ids = st.t(op["ids"])
        Bb, S = st.lshape[ids]
        V, Dm = tok.shape
        tname, pname = st.weight("tok", tok, L.F32), st.weight("pos", pos, L.F32)
        out = op["out"]
        P.add_tensor(out, (Bb * S, Dm), L.F32)
        ep = L.EmbedParams(Bb, S, Dm, V)

        def build(d, ids=ids, tname=tname, pname=pname, out=out, ep=ep):
            return [Launch(L.K_EMBED, [d[ids].t(), d[tname].t(), d[pname].t()], [d[out].t()], ep)]
        P.add_step("embed", [ids, tname, pname], [out], build)
        st.layout[out] = "rows"
        st.lshape[out] = (Bb, S, Dm)
    elif k == "ln":
        x = st.t(op["x"])
        shp = st.lshape[x]
        cols = shp[-1]
        rows = int(np.prod(shp[:-1]))
        sname = st.weight("ln_scale", op["scale"].astype(np.float32), L.F32)
        bname = st.weight("ln_bias", op["bias"].astype(np.float32), L.F32) if op["bias"] is not None else None
        out = op["out"]
        lp = L.LayerNormParams(rows, cols, op["eps"], 0, int(bname is not None), 0)
        if _ln_feeds_f8_linear(st, op, cols):
            # the only consumer is an fp8 linear: LayerNorm writes its E4M3
            # bytes and row scales directly (no bf16 copy, no quant step)
            xq, xs = f"{out}:xq", f"{out}:xs"
            P.add_tensor(xq, (rows, cols), L.U8)
            P.add_tensor(xs, (rows,), L.F32)
            st.fused_q[out] = (xq, xs)

            def build_q(d, x=x, sname=sname, bname=bname, xq=xq, xs=xs, lp=lp, rows=rows, cols=cols):
                ins = [d[x].t((rows, cols)), d[sname].t()] + ([d[bname].t()] if bname else [])
                return [Launch(L.K_LAYERNORM, ins, [d[xq].t(), d[xs].t()], lp)]
            P.add_step("layernorm_e4m3", [x, sname] + ([bname] if bname else []), [xq, xs], build_q, 0.0)
            st.layout[out] = "rows"
            st.lshape[out] = shp
            return
        P.add_tensor(out, (rows, cols), T16 if bf and not _ln_feeds_logits(st, op) else L.F32)

        def build(d, x=x, sname=sname, bname=bname, out=out, lp=lp, rows=rows, cols=cols):
            ins = [d[x].t((rows, cols)), d[sname].t()] + ([d[bname].t()] if bname else [])
            return [Launch(L.K_LAYERNORM, ins, [d[out].t()], lp)]
        P.add_step("layernorm", [x, sname] + ([bname] if bname else []), [out], build, 0.0)
        st.layout[out] = "rows"
        st.lshape[out] = shp
    elif k == "select":
        x = st.t(op["x"])
        Bb, S, Dm = st.lshape[x]
        out = op["out"]
        P.add_tensor(out, (Bb, Dm), P.tensors[x].dtype)
        cpp = L.CopyParams()
        cpp.in_offset = op["index"] * Dm
        cpp.in_stride[0], cpp.in_stride[1] = S * Dm, 1

        def build(d, x=x, out=out, cpp=cpp):
            return [Launch(L.K_COPY, [d[x].t()], [d[out].t()], cpp)]
        P.add_step("select_rows", [x], [out], build)
        st.layout[out] = "rows"
        st.lshape[out] = (Bb, Dm)
    elif k == "linear":
        x = st.t(op["x"])
        shp = st.lshape[x]
        K = shp[-1]
        M = int(np.prod(shp[:-1]))
        w = op["w"]  # [N, K]
        N = w.shape[0]
        res = st.t(op["res"]) if op["res"] else None
        out = op["out"]
        flops = 2.0 * M * N * K
        use_tc = bf and N % 32 == 0 and K % 64 == 0 and (x in st.fused_q or P.tensors[x].dtype == T16)
        bname = st.weight("bias", (op["b"] * op.get("beta", 1.0)).astype(np.float32), L.F32) \
            if op["b"] is not None else None
        # the reference policy for GEMMs (c32/strategy.py:146-157): fp4 (W4A16)
        # for large aligned constant-weight GEMMs, else fp8 for aligned ones
        plain = use_tc and op.get("alpha", 1.0) == 1.0
        use_w4 = (plain and st.profile == "mixed" and K % 64 == 0 and N % 32 == 0 and K >= 128 and N >= 128
                  and K * N >= 32768)
        use_f8 = (plain and not use_w4 and st.profile in ("fp8", "mixed") and N % 16 == 0 and K % 16 == 0
                  and K >= 64 and N >= 64)
        if use_w4:
            from .fp4 import quant_groups_fp4
            wq, ws = quant_groups_fp4(w)
            wqn = st.weight("linear_fp4", wq, L.U8)
            wsn = st.weight("linear_fp4_scale", ws, L.F32)
            odt = L.F32 if (res is not None or op["out"] in [o.name for o in st.g.outputs]) else T16
            P.add_tensor(out, (M, N), odt)

            if M >= W4A16_EXPAND_ROWS:
                # many rows: expand the FP4 weights to bf16 once (a transient
                # arena tensor) and run the bf16 GEMM, instead of re-expanding
                # them next to the MMA for every 128-row tile
                wdq = f"{out}:w_bf16"
                P.add_tensor(wdq, (N, K), T16)

                def build_dq(d, wqn=wqn, wsn=wsn, wdq=wdq, N=N, K=K):
                    return [Launch(L.K_DEQUANT_FP4, [d[wqn].t(), d[wsn].t()], [d[wdq].t()], L.QuantParams(N, K))]
                P.add_step("dequant_fp4", [wqn, wsn], [wdq], build_dq, 0.0)

                def build(d, x=x, wdq=wdq, bname=bname, out=out, M=M, N=N, K=K, act=op["act"], res=res):
                    return [_gemm_tc_launch(d, x, wdq, bname, out, M, N, K, act, res)]
                P.add_step("gemm_tc", [x, wdq] + ([bname] if bname else []) + ([res] if res else []), [out],
                           build, flops)
            else:
                def build(d, x=x, wqn=wqn, wsn=wsn, bname=bname, out=out, M=M, N=N, K=K, act=op["act"], res=res):
                    g = L.GemmTcParams()
                    g.M, g.N, g.K = M, N, K
                    g.bias_mode = L.BIAS_COL if bname else L.BIAS_NONE
                    g.act, g.has_residual, g.block_n = act, int(res is not None), 0
                    ins = [d[x].t((M, K)), d[wqn].t(), d[wsn].t()] + ([d[bname].t()] if bname else []) + \
                        ([d[res].t((M, N))] if res else [])
                    return [Launch(L.K_GEMM_W4A16, ins, [d[out].t((M, N))], g)]
                P.add_step("gemm_w4a16", [x, wqn, wsn] + ([bname] if bname else []) + ([res] if res else []), [out],
                           build, flops)
        elif use_f8:
            # E4M3 bytes and row scales are computed on the GPU when the
            # program is bound (program._quantize_weights_on_device)
            wqn = st.weight("linear_e4m3", None, L.U8, shape=(N, K))
            wsn = st.weight("linear_e4m3_scale", None, L.F32, shape=(N,))
            P.tensors[wqn].quant_src = np.ascontiguousarray(w, np.float32)
            P.tensors[wqn].quant_scale = wsn
            odt = L.F32 if (res is not None or op["out"] in [o.name for o in st.g.outputs]) else T16
            P.add_tensor(out, (M, N), odt)
            if x in st.fused_q:  # quantised by the producing LayerNorm
                xq, xs = st.fused_q[x]
            else:
                xq, xs = f"{out}:xq", f"{out}:xs"
                P.add_tensor(xq, (M, K), L.U8)
                P.add_tensor(xs, (M,), L.F32)

                def build_q(d, x=x, xq=xq, xs=xs, M=M, K=K):
                    return [Launch(L.K_QUANT_E4M3, [d[x].t((M, K))], [d[xq].t(), d[xs].t()], L.QuantParams(M, K))]
                P.add_step("quant_e4m3", [x], [xq, xs], build_q, 0.0)

            def build(d, xq=xq, xs=xs, wqn=wqn, wsn=wsn, bname=bname, out=out, M=M, N=N, K=K, act=op["act"],
                      res=res):
                g = L.GemmTcParams()
                g.M, g.N, g.K = M, N, K
                g.bias_mode = L.BIAS_COL if bname else L.BIAS_NONE
                g.act, g.has_residual, g.block_n = act, int(res is not None), 0
                ins = [d[xq].t(), d[wqn].t(), d[xs].t(), d[wsn].t()] + ([d[bname].t()] if bname else []) + \
                    ([d[res].t((M, N))] if res else [])
                return [Launch(L.K_GEMM_FP8, ins, [d[out].t((M, N))], g)]
            P.add_step("gemm_fp8", [xq, xs, wqn, wsn] + ([bname] if bname else []) + ([res] if res else []), [out],
                       build, flops)
        elif use_tc:
            if op.get("alpha", 1.0) != 1.0:
                raise NotImplementedError("tc linear: alpha != 1")
            wname = st.weight("linear", st.bits16(w), T16)
            # outputs feeding a residual stream or the logits stay fp32
            odt = L.F32 if (res is not None or op["out"] in [o.name for o in st.g.outputs]) else T16
            P.add_tensor(out, (M, N), odt)

            def build(d, x=x, wname=wname, bname=bname, out=out, M=M, N=N, K=K, act=op["act"], res=res):
                return [_gemm_tc_launch(d, x, wname, bname, out, M, N, K, act, res)]
            P.add_step("gemm_tc", [x, wname] + ([bname] if bname else []) + ([res] if res else []), [out], build,
                       flops)
        elif (st.profile == "tf32" or (st.profile in ("bf16", "fp16") and _is_output(st, out))) and N % 32 == 0 \
                and K % 4 == 0 and op.get("alpha", 1.0) == 1.0 and P.tensors[x].dtype == L.F32:
            # the tf32 profile's linear layers, and the bf16 / fp16 profiles'
            # classifier head (its input stays f32, see _ln_feeds_logits)
            wname = st.weight("linear", np.ascontiguousarray(w, np.float32), L.F32)
            P.add_tensor(out, (M, N), L.F32)

            def build(d, x=x, wname=wname, bname=bname, out=out, M=M, N=N, K=K, act=op["act"], res=res):
                ln = _gemm_tc_launch(d, x, wname, bname, out, M, N, K, act, res)
                ln.kid = L.K_GEMM_TF32
                return [ln]
            P.add_step("gemm_tf32", [x, wname] + ([bname] if bname else []) + ([res] if res else []), [out], build,
                       flops)
        else:
            if P.tensors[x].dtype != L.F32:
                raise RuntimeError("SIMT linear expects f32 input")
            wname = st.weight("linear", w.astype(np.float32), L.F32)
            P.add_tensor(out, (M, N), L.F32)

            def build(d, x=x, wname=wname, bname=bname, out=out, M=M, N=N, K=K, act=op["act"], res=res,
                      alpha=op.get("alpha", 1.0)):
                return [_gemm_simt_launch(d, x, wname, bname, out, M, N, K, act, res, alpha, 1.0)]
            P.add_step("gemm_f32", [x, wname] + ([bname] if bname else []) + ([res] if res else []), [out], build,
                       flops)
        st.layout[out] = "rows"
        st.lshape[out] = tuple(shp[:-1]) + (N,)
    elif k == "attention":
        x = st.t(op["x"])
        Bb, S, three_d = st.lshape[x]
        H, D = op["heads"], op["head_dim"]
        out = op["out"]
        dt = P.tensors[x].dtype
        P.add_tensor(out, (Bb * S, H * D), dt)
        fp = L.FlashParams(Bb, S, H, D, op["scale"], op["causal"])
        flops = 4.0 * Bb * H * S * S * D * (0.5 if op["causal"] else 1.0)

        def build(d, x=x, out=out, fp=fp):
            return [Launch(L.K_FLASH_ATTN, [d[x].t()], [d[out].t()], fp)]
        P.add_step("flash_attention", [x], [out], build, flops)
        st.layout[out] = "rows"
        st.lshape[out] = (Bb, S, H * D)
    elif k == "ew":
        xs = [st.t(v) for v in op["xs"]]
        shp = st.lshape[xs[0]]
        out = op["out"]
        P.add_tensor(out, P.tensors[xs[0]].shape, P.tensors[xs[0]].dtype)
        prog = op["prog"]

        def build(d, xs=xs, out=out, prog=prog):
            from .kernels import _ew_program
            return [Launch(L.K_EW, [d[v].t() for v in xs], [d[out].t()], _ew_program(prog))]
        P.add_step("ew", xs, [out], build)
        st.layout[out] = st.layout[xs[0]]
        st.lshape[out] = shp
    else:
        raise NotImplementedError(k)


def lower(graph: ModelGraph, batch: int, profile: str = "fp32") -> Program:
    st = _State(graph, batch, profile)
    for vi in graph.inputs:
        shape = tuple(batch if isinstance(d, str) else int(d) for d in vi.shape)
        dt = L.DTYPE_CODE[vi.dtype]
        st.prog.add_tensor(vi.name, shape, dt, "input")
        st.prog.inputs.append(vi.name)
        st.layout[vi.name] = "nchw" if len(shape) == 4 else "rows"
        st.lshape[vi.name] = shape
    for i in range(len(graph.nodes)):
        if i in st.done:
            continue
        if not any(m(st, i) for m in _MATCHERS):
            raise NotImplementedError(f"lowering: no pattern for node {graph.nodes[i].op_type} "
                                      f"({graph.nodes[i].name})")
    for op in _toposort(st.ops, [v.name for v in graph.inputs]):
        _emit(st, op)
    for vi in graph.outputs:
        st.prog.outputs.append(st.t(vi.name))
        if st.prog.tensors[st.t(vi.name)].dtype != L.F32:
            raise RuntimeError("graph outputs must be fp32")
    st.prog.plan()
    return st.prog


def program_flops(prog: Program) -> float:
    return float(sum(s.flops for s in prog.steps))
