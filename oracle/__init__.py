"""CPU oracle for the fused conv/GEMM hot path -- TEST INFRASTRUCTURE ONLY.

This package restates SimdOnnx's NHWC CPU kernels (the reference's own CPU path) in C++
(``nhwc_oracle.cpp``; every function cites the reference file:line it follows) and wraps them for
numpy. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it, and only as the checker or the timed CPU baseline: the product (``simdonnx_b200``)
never imports, links or calls anything here.

Parity pins (reference tests restated in ``tests/test_oracle.py``):
  * direct conv vs an fp64 loop and vs torch fp64 conv;
  * Winograd vs direct <= 1e-4 * max|out| (tests/Sdcb.SimdOnnx.Tests/EngineTests.cs:184-214);
  * conv + residual vs conv then add <= 1e-4 (EngineTests.cs:163-182);
  * ConvPool == Conv -> MaxPool bit for bit (Avx512KernelTests.cs:145-154);
  * AVX-512 build == AVX2 build bit for bit over the AVX-512 shape matrix (Avx512KernelTests.cs:35-93).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_DIR = os.path.dirname(os.path.abspath(__file__))

ACT = {"none": 0, "relu": 1, "sigmoid": 2, "gelu": 3, "hardswish": 4, "swish": 5}
PAD_CONSTANT, PAD_REFLECT = 0, 1
EW = {"add": 0, "sub": 1, "mul": 2, "div": 3}


def _host_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            return " avx512f " in f.read().replace("\n", " ")
    except OSError:
        return False


def build(force: bool = False) -> None:
    """Compile both ISA builds of the oracle with the Makefile beside this file."""
    cmd = ["make", "-C", _DIR] + (["-B"] if force else [])
    subprocess.run(cmd, check=True, stdout=subprocess.DEVNULL)


_libs: dict[str, ctypes.CDLL] = {}

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float

_SIGS = {
    "orc_set_threads": (None, [_I]),
    "orc_get_threads": (_I, []),
    "orc_isa_avx512": (_I, []),
    "orc_pack_conv_floats": (_L, [_I, _I, _I, _I]),
    "orc_pack_conv": (None, [_P, _P, _I, _I, _I, _I, _P, _P]),
    "orc_pack_depthwise": (None, [_P, _P, _I, _I, _I, _P, _P]),
    "orc_pack_winograd_floats": (_L, [_I, _I]),
    "orc_pack_winograd": (None, [_P, _I, _I, _P]),
    "orc_pack_gemm": (None, [_P, _I, _I, _I, _P, _P, _P]),
    "orc_winograd_eligible": (_I, [_I, _I, _I, _I, _I, _I]),
    "orc_conv": (None, [_P, _I, _I, _I, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _I, _P, _I]),
    "orc_conv_pool": (None, [_P, _I, _I, _I, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _I, _I]),
    "orc_conv_ref64": (None, [_P, _I, _I, _I, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P, _I]),
    "orc_gemm": (None, [_P, _I, _I, _P, _I, _P, _P, _I]),
    "orc_matmul": (None, [_P, _P, _P, _I, _I, _I, _I]),
    "orc_convt": (None, [_P, _I, _I, _I, _I, _P, _I, _I, _I, _P, _P, _I]),
    "orc_maxpool": (None, [_P, _I, _I, _I, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I]),
    "orc_avgpool": (None, [_P, _I, _I, _I, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I]),
    "orc_global_avg_pool": (None, [_P, _I, _I, _I, _P]),
    "orc_channel_gate": (None, [_P, _I, _I, _I, _P, _P, _P, _P, _I, _I, _I, _F, _F, _F, _P]),
    "orc_channel_broadcast": (None, [_P, _P, _P, _I, _L, _I, _I, _I, _I]),
    "orc_resize_nearest": (None, [_P, _I, _I, _I, _I, _P, _I, _I, _F, _F, _P, _I]),
    "orc_concat_inner": (None, [_P, _P, _I, _L, _P]),
    "orc_act": (None, [_P, _P, _L, _I]),
    "orc_binary": (None, [_P, _P, _P, _L, _I, _I]),
    "orc_hardsigmoid": (None, [_P, _P, _L, _F, _F]),
    "orc_layernorm": (None, [_P, _L, _I, _P, _P, _P, _F]),
    "orc_softmax": (None, [_P, _P, _L, _I]),
    "orc_exp_core": (_F, [_F]),
    "orc_erf_core": (_F, [_F]),
    "orc_act_scalar": (_F, [_F, _I]),
}


def lib(isa: str | None = None) -> ctypes.CDLL:
    """The oracle library for ``isa`` ('avx512' | 'avx2'; default: the best the host runs)."""
    if isa is None:
        isa = "avx512" if _host_has_avx512() else "avx2"
    if isa in _libs:
        return _libs[isa]
    path = os.path.join(_DIR, f"liboracle_{isa}.so")
    if not os.path.exists(path):
        build()
    so = ctypes.CDLL(path)
    for name, (res, args) in _SIGS.items():
        fn = getattr(so, name)
        fn.restype = res
        fn.argtypes = args
    _libs[isa] = so
    return so


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int, isa: str | None = None) -> None:
    lib(isa).orc_set_threads(int(n))


def conv_out_size(i: int, k: int, s: int, p0: int, p1: int, d: int = 1) -> int:
    """ONNX conv output size (src/Engine/GraphCompiler.cs:1790-1794)."""
    return (i + p0 + p1 - (d * (k - 1) + 1)) // s + 1


class ConvPlan:
    """Packed conv weights (the reference's NhwcConvPlan, src/Kernels/Nhwc.cs:16-23)."""

    def __init__(self, w: np.ndarray, bias: np.ndarray | None, group: int = 1, winograd: bool | None = None,
                 strides=(1, 1), isa: str | None = None):
        L = lib(isa)
        w = _f32(w)
        self.oc, icg, self.kh, self.kw = w.shape
        self.ic = icg * group
        self.depthwise = group > 1
        b = _f32(bias)
        if self.depthwise:
            if not (group == self.ic and icg == 1 and self.oc == self.ic):
                raise NotImplementedError("NHWC grouped conv supports depthwise only")
            self.pw = np.empty(self.kh * self.kw * self.oc, np.float32)
            self.pb = np.empty(self.oc, np.float32)
            L.orc_pack_depthwise(_p(w), _p(b), self.oc, self.kh, self.kw, _p(self.pw), _p(self.pb))
            self.u = None
            return
        n = L.orc_pack_conv_floats(self.oc, self.ic, self.kh, self.kw)
        self.pw = np.empty(n, np.float32)
        self.pb = np.empty((self.oc + 15) // 16 * 16, np.float32)
        L.orc_pack_conv(_p(w), _p(b), self.oc, self.ic, self.kh, self.kw, _p(self.pw), _p(self.pb))
        elig = bool(L.orc_winograd_eligible(group, self.kh, self.kw, strides[0], strides[1], self.ic))
        if winograd is None:
            winograd = elig
        self.u = None
        if winograd:
            if not elig:
                raise ValueError("conv is not Winograd-eligible")
            self.u = np.empty(L.orc_pack_winograd_floats(self.oc, self.ic), np.float32)
            L.orc_pack_winograd(_p(w), self.oc, self.ic, _p(self.u))


def conv(x: np.ndarray, plan: ConvPlan, strides=(1, 1), pads=(0, 0, 0, 0), act="none", add=None,
         pad_mode=PAD_CONSTANT, pad_value=0.0, isa: str | None = None) -> np.ndarray:
    """NHWC conv over a batch (Nhwc.Conv, src/Kernels/Nhwc.cs:172-217). x [N,H,W,C] fp32."""
    L = lib(isa)
    x = _f32(x)
    n, ih, iw, ic = x.shape
    assert ic == plan.ic
    if plan.u is not None and tuple(strides) != (1, 1):
        raise ValueError("Winograd plan used for a strided conv: build the ConvPlan with the conv's strides")
    oh = conv_out_size(ih, plan.kh, strides[0], pads[0], pads[2])
    ow = conv_out_size(iw, plan.kw, strides[1], pads[1], pads[3])
    y = np.empty((n, oh, ow, plan.oc), np.float32)
    a = _f32(add)
    if a is not None:
        assert a.shape == y.shape
    L.orc_conv(_p(x), n, ih, iw, ic, _p(y), oh, ow, plan.oc, plan.kh, plan.kw, strides[0], strides[1],
               pads[0], pads[1], pad_mode, float(pad_value), _p(plan.pw), _p(plan.pb), _p(plan.u),
               int(plan.depthwise), _p(a), ACT[act])
    return y


def conv_pool(x, plan: ConvPlan, pads=(1, 1, 1, 1), act="none", pool_relu=False, pad_mode=PAD_CONSTANT,
              pad_value=0.0, isa: str | None = None) -> np.ndarray:
    """Conv + fused 2x2/2 max pool (Nhwc.ConvPool, src/Kernels/Nhwc.cs:666-727)."""
    L = lib(isa)
    x = _f32(x)
    n, ih, iw, ic = x.shape
    oh = conv_out_size(ih, plan.kh, 1, pads[0], pads[2])
    ow = conv_out_size(iw, plan.kw, 1, pads[1], pads[3])
    y = np.empty((n, oh // 2, ow // 2, plan.oc), np.float32)
    L.orc_conv_pool(_p(x), n, ih, iw, ic, _p(y), oh, ow, plan.oc, plan.kh, plan.kw, 1, 1, pads[0], pads[1],
                    pad_mode, float(pad_value), _p(plan.pw), _p(plan.pb), _p(plan.u), ACT[act], int(pool_relu))
    return y


def conv_ref64(x, w, bias, strides=(1, 1), pads=(0, 0, 0, 0), group=1, act="none", add=None,
               pad_mode=PAD_CONSTANT, pad_value=0.0) -> np.ndarray:
    """Plain fp64 loop conv (ONNX weights [oc, ic/g, kh, kw]); the independent check."""
    L = lib()
    x = _f32(x)
    w = _f32(w)
    n, ih, iw, ic = x.shape
    oc, _, kh, kw = w.shape
    oh = conv_out_size(ih, kh, strides[0], pads[0], pads[2])
    ow = conv_out_size(iw, kw, strides[1], pads[1], pads[3])
    y = np.empty((n, oh, ow, oc), np.float64)
    L.orc_conv_ref64(_p(x), n, ih, iw, ic, _p(y), oh, ow, oc, kh, kw, strides[0], strides[1], pads[0], pads[1],
                     group, pad_mode, float(pad_value), _p(w), _p(_f32(bias)), _p(_f32(add)), ACT[act])
    return y


class GemmPlan:
    """Packed Gemm B panel (Nhwc.PackGemm, src/Kernels/Nhwc.cs:127-138)."""

    def __init__(self, b: np.ndarray, bias: np.ndarray | None, trans_b: bool = False, isa: str | None = None):
        b = _f32(b)
        self.k, self.n = (b.shape[1], b.shape[0]) if trans_b else b.shape
        nb = (self.n + 15) // 16
        self.pw = np.empty(nb * self.k * 16, np.float32)
        self.pb = np.empty(nb * 16, np.float32)
        lib(isa).orc_pack_gemm(_p(b), self.k, self.n, int(trans_b), _p(_f32(bias)), _p(self.pw), _p(self.pb))


def gemm(a: np.ndarray, plan: GemmPlan, act="none", isa: str | None = None) -> np.ndarray:
    a = _f32(a)
    m = a.size // plan.k
    y = np.empty(a.shape[:-1] + (plan.n,), np.float32)
    lib(isa).orc_gemm(_p(a), m, plan.k, _p(y), plan.n, _p(plan.pw), _p(plan.pb), ACT[act])
    return y


def matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    *bs, m, k = a.shape
    n = b.shape[-1]
    batch = int(np.prod(bs)) if bs else 1
    y = np.empty(tuple(bs) + (m, n), np.float32)
    lib().orc_matmul(_p(a), _p(b), _p(y), batch, m, k, n)
    return y


def convt(x, w, bias, act="none") -> np.ndarray:
    """stride == kernel ConvTranspose; w [ic, oc, kh, kw] (Nhwc.ConvTranspose, src/Kernels/Nhwc.Det.cs:51-131)."""
    x, w = _f32(x), _f32(w)
    n, ih, iw, ic = x.shape
    _, oc, kh, kw = w.shape
    y = np.empty((n, ih * kh, iw * kw, oc), np.float32)
    lib().orc_convt(_p(x), n, ih, iw, ic, _p(y), oc, kh, kw, _p(w), _p(_f32(bias)), ACT[act])
    return y


def maxpool(x, k=(2, 2), s=(2, 2), pads=(0, 0, 0, 0), relu=False) -> np.ndarray:
    x = _f32(x)
    n, ih, iw, c = x.shape
    oh = conv_out_size(ih, k[0], s[0], pads[0], pads[2])
    ow = conv_out_size(iw, k[1], s[1], pads[1], pads[3])
    y = np.empty((n, oh, ow, c), np.float32)
    lib().orc_maxpool(_p(x), n, ih, iw, c, _p(y), oh, ow, k[0], k[1], s[0], s[1], pads[0], pads[1], int(relu))
    return y


def avgpool(x, k, s, pads=(0, 0, 0, 0), count_include_pad=False) -> np.ndarray:
    x = _f32(x)
    n, ih, iw, c = x.shape
    oh = conv_out_size(ih, k[0], s[0], pads[0], pads[2])
    ow = conv_out_size(iw, k[1], s[1], pads[1], pads[3])
    y = np.empty((n, oh, ow, c), np.float32)
    lib().orc_avgpool(_p(x), n, ih, iw, c, _p(y), oh, ow, k[0], k[1], s[0], s[1], pads[0], pads[1],
                      int(count_include_pad))
    return y


def global_avg_pool(x) -> np.ndarray:
    x = _f32(x)
    n, h, w, c = x.shape
    y = np.empty((n, c), np.float32)
    lib().orc_global_avg_pool(_p(x), n, h * w, c, _p(y))
    return y


def channel_gate(x, w1, b1, w2, b2, act1_relu=True, hard=True, alpha=1.0 / 6, beta=0.5, offset=0.0) -> np.ndarray:
    """SE gate s [N, C] (Nhwc.ChannelGate, src/Kernels/Nhwc.Det.cs:287-314); w1 [R, C], w2 [C, R]."""
    x = _f32(x)
    n, h, w, c = x.shape
    w1, w2 = _f32(w1).reshape(-1, c), _f32(w2).reshape(c, -1)
    r = w1.shape[0]
    y = np.empty((n, c), np.float32)
    lib().orc_channel_gate(_p(x), n, h * w, c, _p(w1), _p(_f32(b1)), _p(w2), _p(_f32(b2)), r, int(act1_relu),
                           int(hard), float(alpha), float(beta), float(offset), _p(y))
    return y


def channel_broadcast(full, vec, op="mul", rev=False, relu=False) -> np.ndarray:
    full, vec = _f32(full), _f32(vec)
    n, c = full.shape[0], full.shape[-1]
    rows = full.size // (n * c)
    y = np.empty_like(full)
    lib().orc_channel_broadcast(_p(full), _p(vec), _p(y), n, rows, c, EW[op], int(rev), int(relu))
    return y


def resize_nearest(x, scale=(2.0, 2.0), add=None, add_relu=False) -> np.ndarray:
    x = _f32(x)
    n, ih, iw, c = x.shape
    oh, ow = int(ih * scale[0]), int(iw * scale[1])
    y = np.empty((n, oh, ow, c), np.float32)
    a = _f32(add)
    lib().orc_resize_nearest(_p(x), n, ih, iw, c, _p(y), oh, ow, float(scale[0]), float(scale[1]), _p(a),
                             int(add_relu))
    return y


def concat_channels(xs) -> np.ndarray:
    xs = [_f32(x) for x in xs]
    outer = xs[0].size // xs[0].shape[-1]
    counts = (ctypes.c_int * len(xs))(*[x.shape[-1] for x in xs])
    ptrs = (ctypes.c_void_p * len(xs))(*[x.ctypes.data for x in xs])
    y = np.empty(xs[0].shape[:-1] + (sum(x.shape[-1] for x in xs),), np.float32)
    lib().orc_concat_inner(ctypes.cast(ptrs, ctypes.c_void_p), ctypes.cast(counts, ctypes.c_void_p), len(xs),
                           outer, _p(y))
    return y


def act(x, kind: str) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    lib().orc_act(_p(x), _p(y), x.size, ACT[kind])
    return y


def binary(a, b, op="add", relu=False) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    y = np.empty_like(a)
    lib().orc_binary(_p(a), _p(b), _p(y), a.size, EW[op], int(relu))
    return y


def layernorm(x, w, b, eps=1e-5) -> np.ndarray:
    x = _f32(x)
    c = x.shape[-1]
    y = np.empty_like(x)
    lib().orc_layernorm(_p(x), x.size // c, c, _p(_f32(w)), _p(_f32(b)), _p(y), float(eps))
    return y


def softmax(x) -> np.ndarray:
    x = _f32(x)
    c = x.shape[-1]
    y = np.empty_like(x)
    lib().orc_softmax(_p(x), _p(y), x.size // c, c)
    return y


# ---------------------------------------------------------------------------------------------
# Elementwise with numpy broadcast, the built-in fused ops, batched MatMul and the fused CTC head,
# restated in numpy (fp32 storage and arithmetic; IEEE per element like the reference's scalar and
# Vector<float> code).
# ---------------------------------------------------------------------------------------------
def binary_bcast(a, b, op="add", act_kind="none") -> np.ndarray:
    """Ops.Elementwise (src/Kernels/Ops.cs:388-441): numpy broadcasting of a and b, one IEEE fp32
    op per element (Ew.Binary / Ew.Scalar / Ew.Channel / Strided.Binary all compute a op b), relu
    fused, any other activation applied after (Activation)."""
    a, b = _f32(a), _f32(b)
    f = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide}[op]
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        y = f(a, b, dtype=np.float32).astype(np.float32)
    return y if act_kind == "none" else act(np.ascontiguousarray(y), act_kind)


def safe_div(a, b, eps, lo, hi) -> np.ndarray:
    """FusedKernels.SafeDiv (src/Kernels/FusedKernels.cs:32-55): clamp(a / max(b, eps), lo, hi)."""
    a, b = _f32(a), _f32(b)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        q = a / np.maximum(b, np.float32(eps))
    return np.minimum(np.maximum(q, np.float32(lo)), np.float32(hi)).astype(np.float32)


def channel_shift(x, axis, group_ends, offsets) -> np.ndarray:
    """FusedKernels.ChannelShift (src/Kernels/FusedKernels.cs:196-221), NHWC x [n, h, w, c]: channel
    group g = [end[g-1], end[g]) reads in[y + off[g], x] (axis 2) or in[y, x + off[g]] (axis 3),
    zero outside; channels from the last end on are copied."""
    x = _f32(x)
    n, h, w, c = x.shape
    y = x.copy()
    g0 = 0
    for g1, off in zip(group_ends, offsets):
        src = np.zeros((n, h, w, g1 - g0), np.float32)
        if axis == 2:
            lo, hi = max(0, -off), min(h, h - off)
            if lo < hi:
                src[:, lo:hi] = x[:, lo + off:hi + off, :, g0:g1]
        else:
            lo, hi = max(0, -off), min(w, w - off)
            if lo < hi:
                src[:, :, lo:hi] = x[:, :, lo + off:hi + off, g0:g1]
        y[..., g0:g1] = src
        g0 = g1
    return y


def _resize_axis(out_len, in_len, scale):
    """Nhwc.ResizeAxis (src/Kernels/Nhwc.cs:773-783) in fp32."""
    o = np.arange(out_len, dtype=np.float32)
    f = ((o + np.float32(0.5)) / np.float32(scale) - np.float32(0.5)).astype(np.float32)
    fl = np.floor(f)
    i0 = np.clip(fl.astype(np.int64), 0, in_len - 1)
    i1 = np.clip(fl.astype(np.int64) + 1, 0, in_len - 1)
    return i0, i1, (f - fl).astype(np.float32)


def uphead(x, skip, w, bias, scale_h, scale_w, resize_relu=False, skip_relu=False, act_kind="none") -> np.ndarray:
    """FusedKernels.UpHead (src/Kernels/FusedKernels.cs:71-193), NHWC: s = [relu](bilinear(x)) +
    [relu](skip) with ResizePixel's separate fp32 multiply and add (src/Kernels/Nhwc.cs:788-815),
    then y[o] = act(bias[o] + sum_c w[o, c] s[c]) with one fused multiply-add per channel, ascending
    (the AVX tiers' FMA chain; fp64 product and sum rounded once to fp32)."""
    x, skip, w = _f32(x), _f32(skip), _f32(w)
    n, ih, iw, c = x.shape
    oh, ow = skip.shape[1], skip.shape[2]
    y0, y1, wy = _resize_axis(oh, ih, scale_h)
    x0, x1, wx = _resize_axis(ow, iw, scale_w)
    a = x[:, y0][:, :, x0]
    b_ = x[:, y0][:, :, x1]
    e = x[:, y1][:, :, x0]
    f = x[:, y1][:, :, x1]
    wxb = wx[None, None, :, None]
    wyb = wy[None, :, None, None]
    top = (a + ((b_ - a) * wxb).astype(np.float32)).astype(np.float32)
    bot = (e + ((f - e) * wxb).astype(np.float32)).astype(np.float32)
    v = (top + ((bot - top) * wyb).astype(np.float32)).astype(np.float32)
    if resize_relu:
        v = np.maximum(v, 0)
    sk = np.maximum(skip, 0) if skip_relu else skip
    s = (v + sk).astype(np.float32)
    oc = w.shape[0]
    acc = np.broadcast_to(np.zeros(oc, np.float32) if bias is None else _f32(bias), (n, oh, ow, oc)).copy()
    for ch in range(c):
        acc = (s[..., ch:ch + 1].astype(np.float64) * w[:, ch].astype(np.float64) + acc.astype(np.float64)).astype(np.float32)
    return acc if act_kind == "none" else act(np.ascontiguousarray(acc), act_kind)


def matmul_bcast(a, b) -> np.ndarray:
    """Ops.MatMul (src/Kernels/Ops.Seq.cs:90-113): a [.., m, k] x b [.., k, n] with numpy broadcast
    over the batch dims; each batch is the oracle's GemmKN-order matmul."""
    a, b = _f32(a), _f32(b)
    bs = np.broadcast_shapes(a.shape[:-2], b.shape[:-2])
    ab = np.broadcast_to(a, bs + a.shape[-2:]).reshape((-1,) + a.shape[-2:])
    bb = np.broadcast_to(b, bs + b.shape[-2:]).reshape((-1,) + b.shape[-2:])
    out = np.stack([matmul(np.ascontiguousarray(ab[i]), np.ascontiguousarray(bb[i])) for i in range(ab.shape[0])])
    return out.reshape(bs + (a.shape[-2], b.shape[-1]))


def ctc_argmax(logits) -> tuple:
    """MatMul.TryArgMax's per-row result (src/Decoding/Kernels/MatMul.ArgMax.cs:29-70, UpdateArgMax
    :246-268) from the row's logits, columns in order: index of the first maximum and the online
    softmax denominator s (a new maximum rescales s by exp(old - new) and adds 1, any other value
    adds exp(value - max)); probability min(1, 1 / s). Vectorised over rows, sequential over columns."""
    z = _f32(logits)
    z = z.reshape(-1, z.shape[-1])
    rows = z.shape[0]
    m = np.full(rows, -np.inf, np.float32)
    s = np.zeros(rows, np.float32)
    best = np.zeros(rows, np.int64)
    with np.errstate(over="ignore", invalid="ignore"):
        for col in range(z.shape[1]):
            v = z[:, col]
            up = v > m
            s = np.where(up, (s * np.exp(m - v, dtype=np.float32) + np.float32(1)).astype(np.float32),
                         (s + np.exp(v - m, dtype=np.float32)).astype(np.float32))
            best = np.where(up, col, best)
            m = np.where(up, v, m)
    return best, np.minimum(np.float32(1), np.float32(1) / s).astype(np.float32)
