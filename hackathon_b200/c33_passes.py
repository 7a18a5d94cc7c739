"""Extra C3.3 fusion passes, run after the reference's ``PASS_ORDER``.

The reference pipeline (c33/pipeline.py:108-119) stops short of one-launch
convolutions, linear layers with their epilogues, and attention:

* ``fuse_conv_epilogues`` only matches a plain ``Conv`` (c33/fusion.py:1135-1136),
  so a ``FusedConv2dBatchNorm`` followed by ``Relu`` or by the residual
  ``Add -> Relu`` chain stays two or three nodes, and C3.2 lowers each folded
  conv to winograd (broken, c32/kernel_registry.py:534) or
  im2col -> matmul -> conv_reshape -> add_bias (c32/decompositions.py:300-378);
* ``FusedMatMulBias`` keeps its GELU chain and residual ``Add`` as separate
  nodes;
* attention keeps Split, three Reshape/Transpose pairs, the materialised
  ``[B, H, S, S]`` score tensor, the P.V ``MatMul`` and the head merge.

These passes rewrite those patterns into single nodes whose op types the
B200 backend executes as one kernel each.  C3.2 has no decomposition for them,
so ``Strategy.decompose`` emits one kernel named ``<op type lower>_<dtype>``
(c32/strategy.py:189-195) with the node's inputs, outputs and attributes as
``operator_params``; C3.4 then plans lifetimes, arena offsets, streams and
events for that kernel like any other.

* ``B200ConvBiasAct``: inputs ``[x, w, b]`` or ``[x, w, b, residual]``; the BN
  is already folded into ``w, b`` (the executor's rewrite,
  c35/executor.py:359-442).  Attributes: the conv's, plus ``_activation``
  ("Relu" or absent) and ``_residual_input_index`` (3) when a residual is added
  before the activation.
* ``B200LinearEpilogue``: inputs ``[x, w, b]`` or ``[x, w, b, residual]``,
  ``w`` stored [K, N] as in MatMul.  ``_activation`` is "Gelu" when the
  exact-erf GELU chain (Div sqrt2, Erf, Add 1, Mul x, Mul 0.5) followed; its
  constant tensors are listed in ``_gelu_constants`` for the runtime to check.
* ``B200FlashAttention``: inputs ``[qkv, heads_shape, divisor, mask,
  merge_shape]``; ``softmax(Q K^T / divisor + mask) V`` per head with the heads
  merged back to ``[B, S, H*D]``.  ``_qkv_order`` gives which Split output is
  Q, K and V.

The passes use only the IR interface the reference passes use (``nodes``,
``node_order``, ``tensor_consumers``, ``tensor_producer``, ``outputs``,
``initializers``, ``remove_node``, ``add_node``, ``set_producer``,
``topological_sort``), so they run on the reference ``Graph`` and on any
object with that interface.
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional

GELU_CHAIN = ["Div", "Erf", "Add", "Mul", "Mul"]


def _consumers(g, t: str) -> List[str]:
    return [c for c in g.tensor_consumers.get(t, []) if c in g.nodes]


def _is_output(g, t: str) -> bool:
    return any(o.name == t for o in g.outputs)


def _sole(g, t: str):
    """The single consumer node of ``t`` (None if t is a graph output or has
    zero or several consumers)."""
    c = _consumers(g, t)
    if len(c) != 1 or _is_output(g, t):
        return None
    return g.nodes[c[0]]


def _new_node(g, like, nid: str, op_type: str, inputs, outputs, attrs):
    return type(like)(id=nid, name=getattr(like, "name", nid), op_type=op_type, inputs=list(inputs),
                      outputs=list(outputs), attributes=dict(attrs), domain=getattr(like, "domain", ""))


def _replace(g, old_ids: List[str], node, log: List[Dict[str, Any]], kind: str) -> None:
    """Swap the nodes ``old_ids`` for ``node`` at the position of the first."""
    pos = min(g.node_order.index(i) for i in old_ids if i in g.node_order)
    for i in old_ids:
        g.remove_node(i)
    g.add_node(node)
    for o in node.outputs:
        if o:
            g.tensor_producer.pop(o, None)
            g.set_producer(o, node.id)
    g.node_order.insert(pos, node.id)
    log.append({"pass": kind, "fused": list(old_ids), "into": node.id})


def fuse_conv_bias_act(g, log: List[Dict[str, Any]]) -> int:
    """Folded Conv+BN [-> Relu | -> Add(residual) -> Relu] into one node."""
    if not g.node_order:
        g.topological_sort()
    fused = 0
    for nid in list(g.node_order):
        conv = g.nodes.get(nid)
        if conv is None or conv.op_type not in ("FusedConv2dBatchNorm", "Conv"):
            continue
        if conv.op_type == "FusedConv2dBatchNorm" and not conv.attributes.get("bn_folded"):
            continue  # the BN must be folded into w, b first
        if len([i for i in conv.inputs if i]) not in (2, 3) or len(conv.outputs) != 1:
            continue
        attrs = {k: v for k, v in conv.attributes.items()
                 if k in ("kernel_shape", "pads", "strides", "dilations", "group", "auto_pad")}
        ins = list(conv.inputs[:3])
        old = [conv.id]
        out = conv.outputs[0]
        nxt = _sole(g, out)
        if nxt is not None and nxt.op_type == "Relu":
            attrs["_activation"] = "Relu"
            old.append(nxt.id)
            out = nxt.outputs[0]
        elif (nxt is not None and nxt.op_type == "FusedEWChain" and list(nxt.attributes.get("chain_ops", []))
              == ["Add", "Relu"] and len(nxt.inputs) == 2 and out in nxt.inputs):
            res = nxt.inputs[1] if nxt.inputs[0] == out else nxt.inputs[0]
            prod = g.tensor_producer.get(res)
            # Fuse into the conv that runs later, so the residual is ready
            # when it starts (the other branch of a downsampling block is a
            # conv too, earlier in the order).
            order = {n: i for i, n in enumerate(g.node_order)}
            if res and res not in g.initializers and (prod not in order or order[prod] < order[conv.id]):
                attrs["_activation"] = "Relu"
                attrs["_residual_input_index"] = 3
                if len(ins) == 2:
                    ins.append("")
                ins.append(res)
                old.append(nxt.id)
                out = nxt.outputs[0]
        node = _new_node(g, conv, f"_B200ConvBiasAct_{conv.id}", "B200ConvBiasAct", ins, [out], attrs)
        _replace(g, old, node, log, "B200ConvBiasAct")
        fused += 1
    return fused


def fuse_linear_epilogue(g, log: List[Dict[str, Any]]) -> int:
    """FusedMatMulBias [-> exact-erf GELU chain | -> Add(residual)] into one node."""
    if not g.node_order:
        g.topological_sort()
    fused = 0
    for nid in list(g.node_order):
        mm = g.nodes.get(nid)
        if mm is None or mm.op_type != "FusedMatMulBias" or len(mm.outputs) != 1:
            continue
        if len(mm.inputs) != 3 or mm.inputs[1] not in g.initializers:
            continue
        attrs: Dict[str, Any] = {}
        ins = list(mm.inputs)
        old = [mm.id]
        out = mm.outputs[0]
        nxt = _sole(g, out)
        if (nxt is not None and nxt.op_type == "FusedEWChain" and list(nxt.attributes.get("chain_ops", []))
                == GELU_CHAIN and nxt.inputs and nxt.inputs[0] == out):
            attrs["_activation"] = "Gelu"
            attrs["_gelu_constants"] = list(nxt.inputs[1:])
            old.append(nxt.id)
            out = nxt.outputs[0]
        elif nxt is not None and nxt.op_type == "Add" and len(nxt.inputs) == 2:
            res = nxt.inputs[1] if nxt.inputs[0] == out else nxt.inputs[0]
            if res and res not in g.initializers:
                attrs["_residual_input_index"] = 3
                ins.append(res)
                old.append(nxt.id)
                out = nxt.outputs[0]
        node = _new_node(g, mm, f"_B200LinearEpilogue_{mm.id}", "B200LinearEpilogue", ins, [out], attrs)
        _replace(g, old, node, log, "B200LinearEpilogue")
        fused += 1
    return fused


def _head_path(g, split_out: str, perm: List[int]):
    """split output -> Reshape(heads_shape) -> Transpose(perm): (nodes, heads_shape, transposed)."""
    r = _sole(g, split_out)
    if r is None or r.op_type != "Reshape" or len(r.inputs) != 2:
        return None
    t = _sole(g, r.outputs[0])
    if t is None or t.op_type != "Transpose" or list(t.attributes.get("perm", [])) != perm:
        return None
    return [r.id, t.id], r.inputs[1], t.outputs[0]


def fuse_flash_attention(g, log: List[Dict[str, Any]]) -> int:
    """Split -> 3x(Reshape -> Transpose) -> FusedAttentionScores -> MatMul(V)
    -> FusedTransposeReshape into one node."""
    if not g.node_order:
        g.topological_sort()
    fused = 0
    for nid in list(g.node_order):
        sp = g.nodes.get(nid)
        if sp is None or sp.op_type != "Split" or len(sp.outputs) != 3:
            continue
        paths = {}
        for i, o in enumerate(sp.outputs):
            for role, perm in (("q", [0, 2, 1, 3]), ("k", [0, 2, 3, 1])):
                p = _head_path(g, o, perm)
                if p is not None:
                    paths.setdefault(i, []).append((role, p))
        sc = None
        for i, cands in paths.items():
            for role, (ids, hs, t) in cands:
                c = _sole(g, t)
                if role == "q" and c is not None and c.op_type == "FusedAttentionScores":
                    sc = c
        if sc is None or len(sc.inputs) != 4:
            continue
        q_t, k_t, divisor, mask = sc.inputs
        roles = {}
        for i, cands in paths.items():
            for role, (ids, hs, t) in cands:
                if t == q_t and role == "q":
                    roles["q"] = (i, ids, hs)
                elif t == k_t and role == "k":
                    roles["k"] = (i, ids, hs)
        pv = _sole(g, sc.outputs[0])
        if "q" not in roles or "k" not in roles or pv is None or pv.op_type != "MatMul" or pv.inputs[0] != sc.outputs[0]:
            continue
        v_i = ({0, 1, 2} - {roles["q"][0], roles["k"][0]})
        if len(v_i) != 1:
            continue
        v_i = v_i.pop()
        vp = _head_path(g, sp.outputs[v_i], [0, 2, 1, 3])
        if vp is None or vp[2] != pv.inputs[1]:
            continue
        mg = _sole(g, pv.outputs[0])
        if mg is None or mg.op_type != "FusedTransposeReshape" or list(mg.attributes.get("perm", [])) != [0, 2, 1, 3]:
            continue
        hs = roles["q"][2]
        if roles["k"][2] != hs or vp[1] != hs:
            continue
        old = [sp.id] + roles["q"][1] + roles["k"][1] + vp[0] + [sc.id, pv.id, mg.id]
        attrs = {"_qkv_order": [roles["q"][0], roles["k"][0], v_i], "axis": int(sp.attributes.get("axis", -1))}
        node = _new_node(g, sc, f"_B200FlashAttention_{sc.id}", "B200FlashAttention",
                         [sp.inputs[0], hs, divisor, mask, mg.inputs[1]], [mg.outputs[0]], attrs)
        _replace(g, old, node, log, "B200FlashAttention")
        fused += 1
    return fused


B200_PASS_ORDER = [
    ("B200ConvBiasAct", fuse_conv_bias_act),
    ("B200LinearEpilogue", fuse_linear_epilogue),
    ("B200FlashAttention", fuse_flash_attention),
]


def run_b200_passes(g) -> Dict[str, Any]:
    """Run the passes in order; returns per-pass counts and the fusion log."""
    log: List[Dict[str, Any]] = []
    counts = {name: fn(g, log) for name, fn in B200_PASS_ORDER}
    g.topological_sort()
    if hasattr(g, "validate"):
        g.validate()
    return {"counts": counts, "fusion_log": log}
