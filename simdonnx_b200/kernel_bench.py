"""Micro-benchmark of one fused node kind at one shape (the role of the reference's
bench/Sdcb.SimdOnnx.Bench/Micro.cs): times the sdx_* call with CUDA events and reports achieved
GB/s and TFLOP/s against the algorithmic work. Small enough to run under ncu.

    python -m simdonnx_b200.kernel_bench --op pw --batch 64 --hw 80 --cin 64 --cout 128 --iters 20
ops: pw (1x1 conv, tensor cores), conv3 (3x3 s1, tensor cores), dw (depthwise), stem (3x3 s2 from
fp32 NCHW), convt (2x2 s2 ConvTranspose), gate (squeeze-excitation gate), dwpw (depthwise 3x3 ->
1x1 fused, sdx_dw_pw; --unfused: the same two convs as two launches), copy (torch copy, the
HBM reference point), fill (write-only reference), expand (1:2 read:write reference, torch cat)
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from . import backend as B
from . import _native as N


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="pw")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--hw", type=int, default=80)
    ap.add_argument("--cin", type=int, default=64)
    ap.add_argument("--cout", type=int, default=128)
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--stride", type=int, default=1)
    ap.add_argument("--act", default="hardswish")
    ap.add_argument("--gap", action="store_true", help="pw: also write the 32-pixel channel sums (SE pooling)")
    ap.add_argument("--scale", action="store_true", help="dwpw: per-image SE scale on the depthwise input")
    ap.add_argument("--unfused", action="store_true", help="dwpw: depthwise and pointwise as two launches")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    be = B.CudaBackend.get(0)
    rng = np.random.default_rng(0)
    n, hw, ci, co = a.batch, a.hw, a.cin, a.cout
    dev = "cuda"
    flops = 0
    if a.op in ("pw", "conv3", "dw", "stem"):
        k = {"pw": 1, "conv3": a.k, "dw": a.k, "stem": 3}[a.op]
        s = {"stem": 2}.get(a.op, a.stride if a.op == "dw" else 1)
        p = k // 2
        group = ci if a.op == "dw" else 1
        if a.op == "dw":
            co = ci
        if a.op == "stem":
            ci = 3
            x = torch.rand((n, ci, hw, hw), device=dev)
            d = B.conv_desc(n, hw, hw, ci, co, k, k, stride=(s, s), pads=(p,) * 4, act=a.act, x_dtype=torch.float32,
                            x_layout=N.NCHW)
        else:
            x = torch.randn((n, hw, hw, ci), device=dev).half()
            d = B.conv_desc(n, hw, hw, ci, co, k, k, stride=(s, s), pads=(p,) * 4, group=group, act=a.act)
        w = (rng.standard_normal((co, ci // group, k, k)) * 0.1).astype(np.float32)
        wp = B.pack_conv(d, w)
        bias = torch.zeros(co, device=dev)
        sums = None
        if a.gap:
            sums = torch.empty((n * d.oh * d.ow // 32, co), dtype=torch.float32, device=dev)
            d.gap_sums = B.ptr(sums)
        y = B.conv2d(be, d, x, wp, bias=bias)
        run = lambda: B.conv2d(be, d, x, wp, bias=bias, y=y)
        flops = 2 * n * d.oh * d.ow * co * (ci // group) * k * k
        wbytes = w.size * (4 if a.op in ("dw", "stem") else 2)
        byts = x.numel() * x.element_size() + wbytes + 4 * co + y.numel() * y.element_size()
        if sums is not None:
            byts += sums.numel() * 4
        shape = dict(n=n, h=hw, w=hw, cin=ci, cout=co, k=k, stride=s, oh=d.oh, ow=d.ow)
    elif a.op == "dwpw":
        x = torch.randn((n, hw, hw, ci), device=dev).half()
        dwd = B.conv_desc(n, hw, hw, ci, ci, 3, 3, pads=(1,) * 4, group=ci, act=a.act)
        pwd = B.conv_desc(n, hw, hw, ci, co, 1, 1, act=a.act)
        pdw = B.pack_conv(dwd, (rng.standard_normal((ci, 1, 3, 3)) * 0.3).astype(np.float32))
        ppw = B.pack_conv(pwd, (rng.standard_normal((co, ci, 1, 1)) * 0.1).astype(np.float32))
        bdw, bpw = torch.zeros(ci, device=dev), torch.zeros(co, device=dev)
        scale = torch.rand((n, ci), device=dev) if a.scale else None
        sums = torch.empty((n * hw * hw // 32, co), dtype=torch.float32, device=dev) if a.gap else None
        y = torch.empty((n, hw, hw, co), dtype=torch.float16, device=dev)
        byts = x.numel() * 2 + y.numel() * 2 + (sums.numel() * 4 if a.gap else 0)
        if a.unfused:
            mid = torch.empty_like(x)
            pwd.gap_sums = B.ptr(sums)
            run = lambda: (B.conv2d(be, dwd, x, pdw, bias=bdw, y=mid, in_scale=scale),
                           B.conv2d(be, pwd, mid, ppw, bias=bpw, y=y))
        else:
            run = lambda: B.dw_pw(be, dwd, pwd, x, pdw, bdw, ppw, bpw, in_scale=scale, gap=sums, y=y)
        flops = 2 * n * hw * hw * ci * (9 + co)
        shape = dict(n=n, h=hw, w=hw, cin=ci, cout=co, unfused=a.unfused)
    elif a.op == "convt":
        x = torch.randn((n, hw, hw, ci), device=dev).half()
        w = (rng.standard_normal((ci, co, 2, 2)) * 0.1).astype(np.float32)
        wp = B.pack_convt(w) if co >= 8 else torch.from_numpy(w).to(dev)
        bias = torch.zeros(co, device=dev)
        y = B.convt(be, x, wp, ci, co, 2, 2, bias=bias, act="relu")
        run = lambda: B.convt(be, x, wp, ci, co, 2, 2, bias=bias, act="relu")
        flops = 2 * n * hw * hw * ci * co * 4
        byts = x.numel() * 2 + w.size * 2 + 4 * co + y.numel() * y.element_size()
        shape = dict(n=n, h=hw, w=hw, cin=ci, cout=co)
    elif a.op == "gate":
        x = torch.randn((n, hw, hw, ci), device=dev).half()
        r = ci // 4
        w1, w2 = torch.randn(r, ci, device=dev), torch.randn(ci, r, device=dev)
        b1, b2 = torch.zeros(r, device=dev), torch.zeros(ci, device=dev)
        run = lambda: B.channel_gate(be, x, w1, b1, w2, b2)
        byts = x.numel() * 2
        shape = dict(n=n, h=hw, w=hw, c=ci)
    elif a.op == "fill":
        # write-only reference: bytes / time of a plain fill of the output-sized tensor
        y = torch.empty((n, hw, hw, co), device=dev).half()
        run = lambda: y.fill_(1.0)
        byts = y.numel() * 2
        shape = dict(n=n, h=hw, w=hw, c=co)
    elif a.op == "expand":
        # 1:2 read:write reference (the pointwise conv's traffic shape): y = cat(x, x) on channels
        x = torch.randn((n, hw, hw, ci), device=dev).half()
        y = torch.empty((n, hw, hw, 2 * ci), device=dev).half()
        run = lambda: torch.cat([x, x], dim=-1, out=y)
        byts = x.numel() * 2 + y.numel() * 2
        shape = dict(n=n, h=hw, w=hw, c=ci)
    elif a.op == "copy":
        x = torch.randn((n, hw, hw, ci), device=dev).half()
        y = torch.empty_like(x)
        run = lambda: y.copy_(x)
        byts = 2 * x.numel() * 2
        shape = dict(n=n, h=hw, w=hw, c=ci)
    else:
        raise SystemExit(f"unknown op {a.op}")
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.iters):
        run()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / a.iters
    print(json.dumps({"op": a.op, **shape, "ms": ms, "gbs": byts / ms / 1e6, "tflops": flops / ms / 1e9,
                      "bytes": byts, "flops": flops}))


if __name__ == "__main__":
    main()
