"""Load-time plan rewrites of the reference, restated on ExecPlans.

* fold_conv_batchnorm: OnnxRewrites.FoldConvBatchNorm (src/Onnx/OnnxRewrites.cs:71-111). A
  BatchNorm whose input is a Conv output read by nothing else (and not a graph output) folds into
  that conv: scale = gamma / sqrt(var + eps), w' = w * scale per output channel, b' = (b - mean) *
  scale + beta, all in fp32 like the reference's float arithmetic.
* lower_batchnorm: GraphCompiler.EmitBatchNorm (src/Engine/GraphCompiler.cs:1896-1922). Any other
  BatchNorm becomes the per-channel affine x * s + t (s = gamma / sqrt(var + eps), t = beta - mean *
  s) as two Elementwise nodes broadcasting fp32 [C] constants over the channels-last value.
"""
from __future__ import annotations

import copy

import numpy as np

from .plan import EwP, ExecPlan, Node


def _bn_scale(P: ExecPlan, p):
    gamma, beta = P.values[p.gamma].const, P.values[p.beta].const
    mean, var = P.values[p.mean].const, P.values[p.var].const
    eps = np.float32(p.eps)
    scale = (gamma / np.sqrt(var + eps, dtype=np.float32)).astype(np.float32)
    return scale, beta.astype(np.float32), mean.astype(np.float32)


def fold_conv_batchnorm(plan: ExecPlan) -> ExecPlan:
    """Returns a plan with every foldable Conv -> BatchNorm pair folded (the input plan is not changed)."""
    if not any(n.op == "BatchNorm" for n in plan.nodes):
        return plan
    P = copy.copy(plan)
    P.values = {k: copy.copy(v) for k, v in plan.values.items()}
    P.nodes = [Node(n.op, list(n.ins), list(n.outs), copy.copy(n.p), n.name) for n in plan.nodes]
    prods = {o: m for m in P.nodes for o in m.outs}
    drop = set()
    for bn in P.nodes:
        if bn.op != "BatchNorm":
            continue
        conv = prods.get(bn.ins[0])
        if (conv is None or conv.op != "Conv" or len(P.consumers(bn.ins[0])) != 1 or bn.ins[0] == P.output or
                conv.p.pool is not None or conv.p.add or conv.p.act != "none"):
            continue
        scale, beta, mean = _bn_scale(P, bn.p)
        w = P.values[conv.ins[1]].const
        oc = w.shape[0]
        if scale.shape != (oc,):
            continue
        b0 = P.values[conv.p.bias].const if conv.p.bias else np.zeros(oc, np.float32)
        wname = P.add_const(conv.ins[1] + "__bn_w", (w * scale.reshape(oc, 1, 1, 1)).astype(np.float32))
        bname = P.add_const(conv.name + "__bn_b", ((b0 - mean) * scale + beta).astype(np.float32))
        conv.ins[1] = wname
        conv.p.bias = bname
        P.values[bn.outs[0]] = copy.copy(P.values[conv.outs[0]])
        P.values[bn.outs[0]].name = bn.outs[0]
        old = conv.outs[0]
        conv.outs[0] = bn.outs[0]
        del P.values[old]
        drop.add(id(bn))
    P.nodes = [n for n in P.nodes if id(n) not in drop]
    return P


def lower_batchnorm(plan: ExecPlan) -> ExecPlan:
    """Every remaining BatchNorm -> Elementwise mul by s, then add t (fp32 [C] constants broadcast
    over the last, channel, axis of the NHWC value)."""
    if not any(n.op == "BatchNorm" for n in plan.nodes):
        return plan
    P = copy.copy(plan)
    P.values = dict(plan.values)
    out = []
    for n in plan.nodes:
        if n.op != "BatchNorm":
            out.append(n)
            continue
        scale, beta, mean = _bn_scale(P, n.p)
        shift = (beta - mean * scale).astype(np.float32)
        s = P.add_const(n.name + "__bn_scale", scale)
        t = P.add_const(n.name + "__bn_shift", shift)
        xv = P.values[n.ins[0]]
        mid = P.add_value(n.outs[0] + "__bn_scaled", xv.shape, xv.dtype, xv.layout)
        out.append(Node("Elementwise", [n.ins[0], s], [mid], EwP("mul"), n.name + ".scale"))
        out.append(Node("Elementwise", [mid, t], list(n.outs), EwP("add"), n.name + ".shift"))
    P.nodes = out
    return P
