"""The benchmark configs of BASELINE.json as fused NHWC plans with seeded synthetic weights.

BASELINE.json leaves the layer schedules open; the ones below are pinned here and never change
(they are what the CUDA path, the CPU oracle and the CPU baseline all run):

  C1  single fused node: NHWC 3x3 s1 p1 conv, N=8, 128x128, 64->64, bias, + residual, ReLU.
  C2  OCR text-detection backbone (DB-style): stem 3x3 s2 3->16 HardSwish; 12 blocks of
      depthwise k x k (+HardSwish) -> pointwise 1x1 (+HardSwish) -> squeeze-excitation
      (GAP -> 1x1 C->C/4 + ReLU -> 1x1 -> HardSigmoid(0.2, 0.5) -> x*s); FPN laterals 1x1 -> 96,
      nearest x2 top-down adds, 3x3 96->24 per level, nearest up to 1/4 scale + concat -> 96;
      head 3x3 96->24 + ReLU, ConvT 2x2 s2 24->24 + bias + ReLU, ConvT 2x2 s2 24->1 + bias + Sigmoid.
  C3  OCR text recognition: the same block type (strides (2,2)@2, (2,2)@4, (2,1)@7, (2,1)@12 after a
      s2 stem) to 480 ch at H=1, W=40 via AvgPool (2,1); 1x1 480->120 + HardSwish; 2 transformer
      blocks (dim 120, 8 heads of 15, MLP 240 + GELU, pre-LN); LN; Gemm 120->6625.
  C4  document-enhancement UNet: (3x3+ReLU)x2 at 32/64/128/256 with maxpool 2x2 between, bottleneck
      512, decoder ConvT 2x2 s2 (+bias) -> skip concat -> (3x3+ReLU)x2, final 1x1 32->3 + input residual.
  C5  C2 at N=256 per GPU (the large-batch sweep).

Inputs: C1 x, residual N(0,1)*0.1, W N(0,1)*0.1, bias N(0,0.01); C2-C4 inputs U[0,1]; weights
He-init N(0, 2/fan_in) (C3 N(0, 0.02) for the transformer), biases N(0, 0.02) (BN pre-folded).
Values come from simdonnx_b200.synth (SplitMix64 + Box-Muller) keyed by tensor name.
"""
from __future__ import annotations

import math

from .plan import (AttentionP, ChannelGateP, ConvP, ConvTP, EwP, ExecPlan, GemmP, LnP, PoolP, ResizeNearestP,
                   conv_out)
from .synth import Rng

DET_BLOCKS = [  # (dw kernel, stride, cin, cout)
    (3, 1, 16, 32), (3, 2, 32, 64), (3, 1, 64, 64), (3, 2, 64, 128), (3, 1, 128, 128), (5, 1, 128, 128),
    (3, 2, 128, 256), (5, 1, 256, 256), (5, 1, 256, 256), (5, 1, 256, 256), (5, 1, 256, 256), (5, 2, 256, 512),
]
DET_TAPS = {3: "c2", 6: "c3", 11: "c4", 12: "c5"}


class _Builder:
    def __init__(self, seed: int):
        self.P = ExecPlan()
        self.rng = Rng(seed)
        self.dw_gain, self.pw_gain, self.se_gain = 1.0, 1.0, 1.0

    def nhwc(self, v):
        s = self.P.shape(v)
        return (s[0], s[2], s[3], s[1]) if self.P.values[v].layout == "nchw" else s

    def conv(self, name, x, cout, k, s=1, group=1, act="none", bias=True, add=None, pad=None, gain=1.0,
             w_std=None, pool=None):
        n, h, w, cin = self.nhwc(x)
        p = k // 2 if pad is None else pad
        fan_in = cin // group * k * k
        std = w_std if w_std is not None else gain * math.sqrt(2.0 / fan_in)
        W = self.P.add_const(name + ".w", self.rng.normal(name + ".w", (cout, cin // group, k, k), std))
        B = self.P.add_const(name + ".b", self.rng.normal(name + ".b", (cout,), 0.02)) if bias else None
        oh, ow = conv_out(h, k, s, p, p), conv_out(w, k, s, p, p)
        if pool is not None:
            oh, ow = oh // 2, ow // 2
        y = self.P.add_value(name, (n, oh, ow, cout))
        self.P.add_node("Conv", [x, W], [y], ConvP((k, k), (s, s), (p, p, p, p), group, act, B, add, pool), name)
        return y

    def se(self, name, x):
        n, h, w, c = self.nhwc(x)
        r = c // 4
        W1 = self.P.add_const(name + ".w1", self.rng.normal(name + ".w1", (r, c), math.sqrt(2.0 / c)))
        B1 = self.P.add_const(name + ".b1", self.rng.normal(name + ".b1", (r,), 0.02))
        W2 = self.P.add_const(name + ".w2", self.rng.normal(name + ".w2", (c, r), self.se_gain * math.sqrt(2.0 / r)))
        B2 = self.P.add_const(name + ".b2", self.rng.normal(name + ".b2", (c,), 0.02))
        g = self.P.add_value(name + ".s", (n, c), "f32", "raw")
        self.P.add_node("ChannelGate", [x, W1, W2], [g], ChannelGateP(B1, B2, "relu", True, 0.2, 0.5, 0.0), name)
        y = self.P.add_value(name + ".y", (n, h, w, c))
        self.P.add_node("Elementwise", [x, g], [y], EwP("mul"), name + ".mul")
        return y

    def block(self, name, x, k, s, cout):
        c = self.nhwc(x)[3]
        h = self.conv(name + ".dw", x, c, k, s, group=c, act="hardswish", gain=self.dw_gain)
        h = self.conv(name + ".pw", h, cout, 1, 1, act="hardswish", gain=self.pw_gain)
        return self.se(name + ".se", h)

    def up(self, name, x, f, add=None):
        n, h, w, c = self.nhwc(x)
        y = self.P.add_value(name, (n, h * f, w * f, c))
        self.P.add_node("ResizeNearest", [x] + ([add] if add else []), [y], ResizeNearestP((f, f)), name)
        return y


def build_c1(batch=8, hw=128, c=64, seed=1) -> ExecPlan:
    b = _Builder(seed)
    P, rng = b.P, b.rng
    x = P.add_value("c1.x", (batch, hw, hw, c), "f32", "nhwc")
    res = P.add_value("c1.res", (batch, hw, hw, c), "f32", "nhwc")
    P.inputs = [x, res]
    P.input = x
    W = P.add_const("c1.w", rng.normal("c1.w", (c, c, 3, 3), 0.1))
    B = P.add_const("c1.b", rng.normal("c1.b", (c,), 0.01))
    y = P.add_value("c1.y", (batch, hw, hw, c), "f32", "nhwc")
    P.add_node("Conv", [x, W], [y], ConvP((3, 3), (1, 1), (1, 1, 1, 1), 1, "relu", B, res), "c1")
    P.output = y
    P.feeds = {x: lambda: rng.normal("c1.x", (batch, hw, hw, c), 0.1),
               res: lambda: rng.normal("c1.res", (batch, hw, hw, c), 0.1)}
    return P


def build_det(batch=1, hw=640, seed=2) -> ExecPlan:
    """C2 / C5: the text-detection backbone + FPN + DB head."""
    b = _Builder(seed)
    # weight gains (x He std) that keep activations O(1) through the SE-gated blocks and give the
    # sigmoid head a spread of probabilities (a vanishing net would make parity trivially met)
    b.dw_gain, b.pw_gain, b.se_gain = 1.2, 1.6, 4.0
    P = b.P
    x = P.add_value("input", (batch, 3, hw, hw), "f32", "nchw")
    P.inputs = [x]
    P.input = x
    h = b.conv("stem", x, 16, 3, 2, act="hardswish", gain=1.2)
    feats = {}
    for i, (k, s, cin, cout) in enumerate(DET_BLOCKS, 1):
        h = b.block(f"b{i}", h, k, s, cout)
        if i in DET_TAPS:
            feats[DET_TAPS[i]] = h
    in5 = b.conv("fpn.in5", feats["c5"], 96, 1, bias=False)
    in4 = b.conv("fpn.in4", feats["c4"], 96, 1, bias=False)
    in3 = b.conv("fpn.in3", feats["c3"], 96, 1, bias=False)
    in2 = b.conv("fpn.in2", feats["c2"], 96, 1, bias=False)
    out4 = b.up("fpn.out4", in5, 2, add=in4)
    out3 = b.up("fpn.out3", out4, 2, add=in3)
    out2 = b.up("fpn.out2", out3, 2, add=in2)
    p5 = b.conv("fpn.p5", in5, 24, 3, bias=False, gain=0.6)
    p4 = b.conv("fpn.p4", out4, 24, 3, bias=False, gain=0.6)
    p3 = b.conv("fpn.p3", out3, 24, 3, bias=False, gain=0.6)
    p2 = b.conv("fpn.p2", out2, 24, 3, bias=False, gain=0.6)
    ups = [b.up("fpn.p5u", p5, 8), b.up("fpn.p4u", p4, 4), b.up("fpn.p3u", p3, 2), p2]
    n, fh, fw, _ = P.shape(p2)
    fuse = P.add_value("fpn.fuse", (n, fh, fw, 96))
    P.add_node("Concat", ups, [fuse], None, "fpn.concat")
    hd = b.conv("head.conv", fuse, 24, 3, act="relu", gain=0.7)
    t1 = _convt(b, "head.ct1", hd, 24, "relu")
    out = _convt(b, "head.ct2", t1, 1, "sigmoid", dtype="f32")
    P.output = out
    rng = b.rng
    P.feeds = {x: lambda: rng.uniform("input", (batch, 3, hw, hw))}
    return P


def _convt(b: _Builder, name, x, cout, act, dtype="f16"):
    n, h, w, cin = b.nhwc(x)
    W = b.P.add_const(name + ".w", b.rng.normal(name + ".w", (cin, cout, 2, 2), math.sqrt(2.0 / cin)))
    B = b.P.add_const(name + ".b", b.rng.normal(name + ".b", (cout,), 0.02))
    y = b.P.add_value(name, (n, h * 2, w * 2, cout), dtype)
    b.P.add_node("ConvTranspose", [x, W], [y], ConvTP((2, 2), B, act), name)
    return y


CONFIGS = {
    "c1": dict(builder=build_c1, batches=(8,)),
    "det": dict(builder=build_det, batches=(1, 8, 32)),
    "det256": dict(builder=build_det, batches=(256,)),
}
