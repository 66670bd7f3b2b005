"""Algorithmic work of each lowered node: FLOPs and HBM bytes, and the kernel class it runs on.

Definitions (fixed for every report):
  conv   FLOPs = 2 * N * OH * OW * OC * (IC / group) * KH * KW
  gemm   FLOPs = 2 * M * N * K
  convT  FLOPs = 2 * N * H * W * IC * OC * KH * KW
  bytes  = every distinct tensor the node reads once + every tensor it writes once, at storage
           precision (activations fp16, graph I/O and gates fp32, tensor-core weights fp16,
           bandwidth-kernel weights and biases fp32); halo re-reads and im2col / tile padding
           do not count.
A kernel is tensor-bound when FLOPs / bytes exceeds the ridge peak_flops / peak_bw, else HBM-bound.
"""
from __future__ import annotations

import numpy as np

from .plan import ExecPlan


def _nb(plan: ExecPlan, v: str) -> int:
    return plan.values[v].nbytes if v else 0


def _nhwc(plan, v):
    val = plan.values[v]
    s = val.shape
    return (s[0], s[2], s[3], s[1]) if val.layout == "nchw" else s


def conv_kernel_class(plan: ExecPlan, n) -> str:
    """Mirrors the routing of sdx_conv2d (csrc/sdx_api.cu conv_route)."""
    p = n.p
    xv = plan.values[n.ins[0]]
    ic = _nhwc(plan, n.ins[0])[3]
    oc = plan.values[n.ins[1]].const.shape[0]
    if p.group > 1:
        return "depthwise"
    if (xv.dtype == "f16" and xv.layout == "nhwc" and ic % 8 == 0 and p.strides == (1, 1) and oc >= 8 and
            p.pool is None):
        pointwise = p.kernel == (1, 1) and not any(p.pads)
        if pointwise:  # with in_scale too (per-image weights)
            return "conv_tc_rows"
        if getattr(p, "in_scale", None) is None:
            return "conv_tc"
    if ic <= 4 and p.pool is None:
        return "stem"  # graph-input stems: the small-channel tensor-core / TMA stem kernels
    return "direct_conv"


def node_cost(plan: ExecPlan, n) -> tuple:
    """(kernel class, FLOPs, bytes) of one lowered node."""
    op, p = n.op, n.p
    out = n.outs[0]
    if op == "Conv":
        cls = conv_kernel_class(plan, n)
        nb, ih, iw, ic = _nhwc(plan, n.ins[0])
        _, oh, ow, oc = plan.values[out].shape
        W = plan.values[n.ins[1]].const
        kh, kw = W.shape[2], W.shape[3]
        flops = 2 * nb * oh * ow * oc * (ic // p.group) * kh * kw
        wbytes = W.size * (2 if cls.startswith("conv_tc") else 4)
        byt = _nb(plan, n.ins[0]) + wbytes + (4 * oc if p.bias else 0) + _nb(plan, p.add) + _nb(plan, out)
        sc = getattr(p, "in_scale", None)
        if sc:
            byt += _nb(plan, sc)
        for o in n.outs[1:]:  # fused 32-pixel channel sums for the SE gate (not the per-image weight scratch)
            if o != getattr(p, "w_scaled", None):
                byt += _nb(plan, o)
        return cls, flops, byt
    if op == "ConvTranspose":
        nb, ih, iw, ic = plan.values[n.ins[0]].shape
        W = plan.values[n.ins[1]].const
        _, oc, kh, kw = W.shape
        cls = "convt_tc" if oc >= 8 else "convt_dot"
        flops = 2 * nb * ih * iw * ic * oc * kh * kw
        byt = _nb(plan, n.ins[0]) + W.size * (2 if oc >= 8 else 4) + 4 * oc + _nb(plan, out)
        return cls, flops, byt
    if op == "DwPw":
        # depthwise 3x3 + 1x1 with the depthwise output kept on chip: input, weights, output (+ sums)
        pd, pp, (oh, ow) = p
        nb, ih, iw, c = _nhwc(plan, n.ins[0])
        Wd, Wp = plan.values[n.ins[1]].const, plan.values[n.ins[2]].const
        oc = Wp.shape[0]
        flops = 2 * nb * oh * ow * c * Wd.shape[2] * Wd.shape[3] + 2 * nb * oh * ow * oc * c
        byt = _nb(plan, n.ins[0]) + Wd.size * 4 + 4 * c + Wp.size * 2 + (4 * oc if pp.bias else 0) + _nb(plan, out)
        sc = getattr(pd, "in_scale", None)
        if sc:
            byt += _nb(plan, sc)
        for o in n.outs[1:]:
            byt += _nb(plan, o)
        return "dw_pw", flops, byt
    if op == "ConvTChain":
        # two ConvTs with the intermediate kept on chip: traffic = input, weights, final output
        nb, ih, iw, ic = plan.values[n.ins[0]].shape
        W1, W2 = plan.values[n.ins[1]].const, plan.values[n.ins[2]].const
        _, oc1, kh, kw = W1.shape
        flops = 2 * nb * ih * iw * ic * oc1 * kh * kw + 2 * nb * ih * kh * iw * kw * oc1 * W2[0].size
        byt = _nb(plan, n.ins[0]) + W1.size * 2 + W2.size * 4 + 4 * oc1 + _nb(plan, out)
        return "convt_chain", flops, byt
    if op == "ImageConv":
        # u8 image normalisation fused into the stem conv: traffic = image bytes, weights, output
        W = plan.values[n.ins[1]].const
        nb, oh, ow, oc = plan.values[out].shape
        flops = 2 * nb * oh * ow * oc * W.shape[1] * W.shape[2] * W.shape[3]
        return "stem_image", flops, _nb(plan, n.ins[0]) + W.size * 4 + _nb(plan, out)
    if op == "Gemm" and getattr(p, "ctc", False):
        # fused CTC head: the logits stay on chip; traffic = features, weights, bias, [2, rows] result
        a = n.ins[0]
        Wb = plan.values[n.ins[1]].const
        k, nn = (Wb.shape[1], Wb.shape[0]) if p.trans_b else Wb.shape
        m = int(np.prod(plan.values[a].shape)) // k
        return "ctc_head", 2 * m * nn * k, _nb(plan, a) + Wb.size * 2 + 4 * nn + _nb(plan, out)
    if op == "Gemm":
        a = n.ins[0]
        Wb = plan.values[n.ins[1]].const
        k, nn = (Wb.shape[1], Wb.shape[0]) if p.trans_b else Wb.shape
        m = int(np.prod(plan.values[a].shape)) // k
        byt = _nb(plan, a) + Wb.size * 2 + (4 * nn if p.bias else 0) + _nb(plan, p.add) + _nb(plan, out)
        return "gemm_tc", 2 * m * nn * k, byt
    if op == "ChannelGate":
        # reads the producing conv's 32-pixel channel sums when it wrote them, else the tensor
        src = n.ins[3] if len(n.ins) > 3 else n.ins[0]
        byt = _nb(plan, src) + plan.values[n.ins[1]].const.size * 4 + plan.values[n.ins[2]].const.size * 4
        return "channel_gate", 0, byt + _nb(plan, out)
    if op == "Elementwise":
        cls = "broadcast" if plan.values[n.ins[0]].shape != plan.values[n.ins[1]].shape else "binary"
        return cls, 0, _nb(plan, n.ins[0]) + _nb(plan, n.ins[1]) + _nb(plan, out)
    if op == "ResizeNearest":
        return "resize_nearest", 0, sum(_nb(plan, v) for v in n.ins) + _nb(plan, out)
    if op in ("MaxPool", "AvgPool"):
        return "pool", 0, _nb(plan, n.ins[0]) + _nb(plan, out)
    if op == "Concat":
        return "concat", 0, sum(_nb(plan, v) for v in n.ins) + _nb(plan, out)
    if op == "ConcatNearest":
        return "concat_nearest", 0, sum(_nb(plan, v) for v in n.ins) + _nb(plan, out)
    if op == "Convert":
        return "convert", 0, _nb(plan, n.ins[0]) + _nb(plan, out)
    if op in ("LayerNorm", "Softmax", "Act"):
        return op.lower(), 0, _nb(plan, n.ins[0]) + _nb(plan, out)
    if op in ("SafeDiv", "ChannelShift"):
        return op.lower(), 0, sum(_nb(plan, v) for v in n.ins) + _nb(plan, out)
    if op == "UpHead":
        nb, oh, ow, oc = plan.values[out].shape
        c = plan.values[n.ins[0]].shape[3]
        return "uphead", 2 * nb * oh * ow * oc * c, (_nb(plan, n.ins[0]) + _nb(plan, n.ins[1]) + 4 * oc * c +
                                                     _nb(plan, out))
    if op == "MatMul":
        sa, sb = plan.values[n.ins[0]].shape, plan.values[n.ins[1]].shape
        so = plan.values[out].shape
        batch = int(np.prod(so[:-2])) if len(so) > 2 else 1
        return "matmul", 2 * batch * sa[-2] * sa[-1] * sb[-1], _nb(plan, n.ins[0]) + _nb(plan, n.ins[1]) + _nb(plan, out)
    if op == "Attention":
        nb, t, _ = plan.values[n.ins[0]].shape
        flops = 4 * nb * p.heads * t * t * p.head_dim
        return "attention", flops, _nb(plan, n.ins[0]) + _nb(plan, out)
    return op.lower(), 0, 0


def plan_totals(plan: ExecPlan) -> dict:
    flops = byt = 0
    for n in plan.nodes:
        _, f, b = node_cost(plan, n)
        flops += f
        byt += b
    return {"flops": flops, "bytes": byt}
