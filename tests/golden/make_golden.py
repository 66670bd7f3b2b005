"""Generates tests/golden/oracle_fixtures.npz: small seeded known-answer outputs of the CPU oracle
(the reference's CPU kernels restated), so any change to the oracle's arithmetic shows up as a bit
difference in tests/test_oracle.py.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402
from simdonnx_b200.synth import Rng  # noqa: E402


def cases():
    r = Rng(77)
    x = r.normal("g.x", (1, 9, 11, 16), 0.5)
    w = r.normal("g.w", (24, 16, 3, 3), 0.2)
    b = r.normal("g.b", (24,), 0.1)
    res = r.normal("g.res", (1, 9, 11, 24), 0.5)
    dw = r.normal("g.dw", (16, 1, 5, 5), 0.3)
    return {
        "conv_direct": lambda: O.conv(x, O.ConvPlan(w, b, winograd=False), pads=(1, 1, 1, 1), act="hardswish", add=res),
        "conv_winograd": lambda: O.conv(x, O.ConvPlan(w, b, winograd=True), pads=(1, 1, 1, 1), act="relu", add=res),
        "conv_s2": lambda: O.conv(x, O.ConvPlan(w, b, strides=(2, 2)), strides=(2, 2), pads=(1, 1, 1, 1), act="gelu"),
        "depthwise": lambda: O.conv(x, O.ConvPlan(dw, b[:16], group=16), pads=(2, 2, 2, 2), act="hardswish"),
        "convt": lambda: O.convt(x, r.normal("g.ct", (16, 8, 2, 2), 0.3), b[:8], act="relu"),
        "gate": lambda: O.channel_gate(x, r.normal("g.w1", (4, 16), 0.3), b[:4], r.normal("g.w2", (16, 4), 0.3), b[:16]),
        "softmax": lambda: O.softmax(r.normal("g.sm", (7, 40), 2.0)),
        "layernorm": lambda: O.layernorm(r.normal("g.ln", (5, 120), 1.0), b.repeat(5), b.repeat(5)),
    }


if __name__ == "__main__":
    out = {k: fn() for k, fn in cases().items()}
    np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "oracle_fixtures.npz"), **out)
    print("wrote", list(out))
