"""Generates DET_SCALES in simdonnx_b200/configs.py (run by hand; output pasted there).

A random He-initialised det net with squeeze-excitation gates is bistable: its deep activations
either vanish (gates ~0.5 everywhere, output ~constant) or blow up (gates saturate at 0/1, and
fp16 rounding gets amplified 10x). This script fixes one well-conditioned instance, LSUV-style:
walking the plan in order on a seeded calibration batch (the CPU oracle, fp32), each conv's He
weights get the scale that gives its pre-activation output RMS 1.0, each gate's second FC the scale that gives
its pre-gate logits RMS 0.75 (HardSigmoid(0.2, 0.5) then spreads gates over ~[0.2, 0.8]) and the
output ConvT logits RMS 1.0 (probabilities spread around 0.5 without saturating). Targets that push
the net towards the edge of chaos (gate logits RMS 1.5, output logits 2.0) amplify fp16 storage
rounding of the first layers about 3x by the output. Biases keep their seeded values. The scales are a property of the config, like a
checkpoint; the product only reads the frozen table.

    python tests/golden/calibrate_det.py
"""
import copy
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402
from oracle.runner import OracleSession  # noqa: E402
from simdonnx_b200 import configs  # noqa: E402

TARGET_ACT = 1.0
TARGET_GATE = 0.75
TARGET_OUT = 1.0


def forward_until(P, feeds, stop_node):
    env = {}
    sess = OracleSession(P, keep_all=True)
    for name, v in P.values.items():
        if v.is_const:
            env[name] = v.const
    for name in P.inputs:
        env[name] = feeds[name]
    for n in P.nodes:
        if n is stop_node:
            return env, sess
        out = sess._exec(n, env)
        env[n.outs[0]] = out
    return env, sess


def main(hw=640, batch=1):
    P = configs.build_det(batch=batch, hw=hw, scales={})
    feeds = {k: f() for k, f in P.feeds.items()}
    scales = {}
    for n in P.nodes:
        if n.op == "Conv":
            env, sess = forward_until(P, feeds, n)
            p0 = copy.copy(n.p)
            n.p.act = "none"
            sess._packs.pop(n.name, None)
            pre = sess._exec(n, env)
            n.p = p0
            rms = float(np.sqrt(np.mean(pre.astype(np.float64) ** 2)))
            s = TARGET_ACT / max(rms, 1e-12)
            scales[n.name] = s
            P.values[n.ins[1]].const = (P.values[n.ins[1]].const * s).astype(np.float32)
        elif n.op == "ChannelGate":
            env, _ = forward_until(P, feeds, n)
            x = env[n.ins[0]]
            mean = O.global_avg_pool(x).astype(np.float64)
            w1, w2 = P.values[n.ins[1]], P.values[n.ins[2]]
            b1 = P.values[n.p.b1].const
            b2 = P.values[n.p.b2].const
            pre = mean @ w1.const.T.astype(np.float64) + b1
            s1 = TARGET_ACT / max(float(np.sqrt(np.mean(pre ** 2))), 1e-12)
            w1.const = (w1.const * s1).astype(np.float32)
            hid = np.maximum(mean @ w1.const.T.astype(np.float64) + b1, 0)
            z = hid @ w2.const.T.astype(np.float64) + b2
            s2 = TARGET_GATE / max(float(np.sqrt(np.mean(z ** 2))), 1e-12)
            w2.const = (w2.const * s2).astype(np.float32)
            scales[n.name + ".w1"] = s1
            scales[n.name + ".w2"] = s2
        elif n.op == "ConvTranspose":
            env, sess = forward_until(P, feeds, n)
            p0 = copy.copy(n.p)
            n.p.act = "none"
            pre = sess._exec(n, env)
            n.p = p0
            rms = float(np.sqrt(np.mean(pre.astype(np.float64) ** 2)))
            s = (TARGET_OUT if n.outs[0] == P.output else TARGET_ACT) / max(rms, 1e-12)
            scales[n.name] = s
            P.values[n.ins[1]].const = (P.values[n.ins[1]].const * s).astype(np.float32)
    print("DET_SCALES = {")
    for k, v in scales.items():
        print(f'    "{k}": {v:.6g},')
    print("}")


if __name__ == "__main__":
    main()
