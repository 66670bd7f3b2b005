"""CudaBackend: per-device context plus thin op wrappers over the C ABI for torch CUDA tensors.

PyTorch is plumbing here (device memory, the current stream); every op runs a libsdxcuda kernel.
Op wrappers take torch tensors, pass raw device pointers and the current torch stream, and raise
SdxError on any failure.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N

_F = {torch.float16: N.F16, torch.float32: N.F32}


def ptr(t: torch.Tensor | None) -> int:
    return 0 if t is None else int(t.data_ptr())


_LEGACY_STREAM = 0x1  # cudaStreamLegacy: torch reports its default stream as handle 0


def cur_stream() -> ctypes.c_void_p:
    """torch's current stream as an sdx_stream (NULL would select the context's own stream)."""
    h = torch.cuda.current_stream().cuda_stream
    return ctypes.c_void_p(h if h else _LEGACY_STREAM)


class CudaBackend:
    """One context per GPU (the reference's VkBackend.Default per device, src/Backends/Vulkan/VkBackend.cs:26-47)."""

    _by_dev: dict[int, "CudaBackend"] = {}

    def __init__(self, ordinal: int = 0):
        self.ordinal = ordinal
        h = ctypes.c_void_p()
        N.call("sdx_open", ordinal, ctypes.byref(h))
        self.ctx = h

    @classmethod
    def get(cls, ordinal: int = 0) -> "CudaBackend":
        b = cls._by_dev.get(ordinal)
        if b is None:
            torch.cuda.set_device(ordinal)
            b = cls._by_dev[ordinal] = CudaBackend(ordinal)
        return b

    def device_error(self) -> int:
        code = ctypes.c_uint()
        N.call("sdx_device_error", self.ctx, ctypes.byref(code))
        return code.value

    def clear_device_error(self) -> None:
        N.call("sdx_clear_device_error", self.ctx)

    def sync(self, timeout_ms: int = 0) -> None:
        N.call("sdx_stream_sync", self.ctx, cur_stream(), timeout_ms)

    def close(self) -> None:
        if self.ctx:
            N.call("sdx_close", self.ctx)
            self.ctx = None
            CudaBackend._by_dev.pop(self.ordinal, None)


def launch_count() -> int:
    return int(N.lib().sdx_launch_count())


# ------------------------------------------------------------------------------- packing
def conv_desc(batch, ih, iw, ic, oc, kh, kw, stride=(1, 1), pads=(0, 0, 0, 0), group=1, act="none",
              x_dtype=torch.float16, x_layout=N.NHWC, y_dtype=torch.float16, y_layout=N.NHWC,
              add_dtype=torch.float16, add_layout=N.NHWC, pool=False, pool_relu=False, y_pix_stride=0, y_ch_off=0,
              w_terms=0) -> N.ConvDesc:
    d = N.ConvDesc()
    d.batch, d.ih, d.iw, d.ic, d.oc, d.kh, d.kw = batch, ih, iw, ic, oc, kh, kw
    d.sh, d.sw = stride
    d.pad_t, d.pad_l, d.pad_b, d.pad_r = pads
    d.oh = (ih + pads[0] + pads[2] - kh) // stride[0] + 1
    d.ow = (iw + pads[1] + pads[3] - kw) // stride[1] + 1
    d.group = group
    d.act = N.ACT[act] if isinstance(act, str) else int(act)
    d.pool, d.pool_relu = int(pool), int(pool_relu)
    d.x_dtype, d.x_layout = _F[x_dtype], x_layout
    d.y_dtype, d.y_layout = _F[y_dtype], y_layout
    d.add_dtype, d.add_layout = _F[add_dtype], add_layout
    d.y_pix_stride, d.y_ch_off = y_pix_stride, y_ch_off
    d.w_terms = w_terms
    return d


def _to_dev_bytes(buf: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(buf.view(np.uint8).copy()).to(device)


def pack_conv(d: N.ConvDesc, w: np.ndarray, device="cuda") -> torch.Tensor:
    """Packs ONNX conv weights [oc, ic/g, kh, kw] for the kernel sdx_conv2d routes `d` to."""
    w = np.ascontiguousarray(w, np.float32)
    nb = ctypes.c_size_t()
    N.call("sdx_pack_conv", ctypes.byref(d), None, None, ctypes.byref(nb))
    out = np.empty(nb.value, np.uint8)
    N.call("sdx_pack_conv", ctypes.byref(d), w.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p),
           ctypes.byref(nb))
    return _to_dev_bytes(out, device)


def pack_convt(w: np.ndarray, device="cuda") -> torch.Tensor:
    w = np.ascontiguousarray(w, np.float32)
    ic, oc, kh, kw = w.shape
    nb = ctypes.c_size_t()
    N.call("sdx_pack_convt", ic, oc, kh, kw, None, None, ctypes.byref(nb))
    out = np.empty(nb.value, np.uint8)
    N.call("sdx_pack_convt", ic, oc, kh, kw, w.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p),
           ctypes.byref(nb))
    return _to_dev_bytes(out, device)


def pack_gemm(b: np.ndarray, trans_b=False, device="cuda") -> torch.Tensor:
    b = np.ascontiguousarray(b, np.float32)
    k, n = (b.shape[1], b.shape[0]) if trans_b else b.shape
    nb = ctypes.c_size_t()
    N.call("sdx_pack_gemm", k, n, int(trans_b), None, None, ctypes.byref(nb))
    out = np.empty(nb.value, np.uint8)
    N.call("sdx_pack_gemm", k, n, int(trans_b), b.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p),
           ctypes.byref(nb))
    return _to_dev_bytes(out, device)


# ------------------------------------------------------------------------------- ops
def conv2d(be: CudaBackend, d: N.ConvDesc, x, w_packed, bias=None, add=None, y=None, in_scale=None) -> torch.Tensor:
    if y is None:
        oh, ow = (d.oh // 2, d.ow // 2) if d.pool else (d.oh, d.ow)
        dt = torch.float32 if d.y_dtype == N.F32 else torch.float16
        shape = (d.batch, d.oc, oh, ow) if d.y_layout == N.NCHW else (d.batch, oh, ow, d.oc)
        y = torch.empty(shape, dtype=dt, device=x.device)
    d.x, d.w, d.bias, d.add, d.y, d.in_scale = ptr(x), ptr(w_packed), ptr(bias), ptr(add), ptr(y), ptr(in_scale)
    scratch = None
    if in_scale is not None and d.group == 1:
        # 1x1 tensor-core conv of x * s: per-image scaled weights in a scratch buffer
        nbytes = conv_scaled_weights_bytes(d)
        scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=x.device)
        d.w_scaled = ptr(scratch)
    N.call("sdx_conv2d", be.ctx, ctypes.byref(d), cur_stream())  # scratch: freed in stream order
    return y


def conv_scaled_weights_bytes(d: N.ConvDesc) -> int:
    """Scratch bytes of a 1x1 conv with in_scale (per-image weights), 0 if that form does not apply."""
    return int(N.lib().sdx_conv_scaled_weights_bytes(ctypes.byref(d)))


def gemm(be: CudaBackend, a, w_packed, n, bias=None, act="none", add=None, y=None, y_dtype=torch.float16):
    m, k = a.shape[0], a.shape[-1]
    if y is None:
        y = torch.empty((m, n), dtype=y_dtype, device=a.device)
    d = N.GemmDesc()
    d.m, d.k, d.n, d.lda = m, k, n, a.stride(0)
    d.act = N.ACT[act]
    d.y_dtype = _F[y.dtype]
    d.add_dtype = _F[add.dtype] if add is not None else N.F16
    d.ldy, d.ldadd = y.stride(0), (add.stride(0) if add is not None else 0)
    d.a, d.w, d.bias, d.add, d.y = ptr(a), ptr(w_packed), ptr(bias), ptr(add), ptr(y)
    N.call("sdx_gemm", be.ctx, ctypes.byref(d), cur_stream())
    return y


def convt(be: CudaBackend, x, w, ic, oc, kh, kw, bias=None, act="none", y_dtype=torch.float16):
    b, ih, iw, _ = x.shape
    y = torch.empty((b, ih * kh, iw * kw, oc), dtype=y_dtype, device=x.device)
    d = N.ConvtDesc()
    d.batch, d.ih, d.iw, d.ic, d.oc, d.kh, d.kw = b, ih, iw, ic, oc, kh, kw
    d.act, d.y_dtype = N.ACT[act], _F[y_dtype]
    d.x, d.w, d.bias, d.y = ptr(x), ptr(w), ptr(bias), ptr(y)
    N.call("sdx_convt", be.ctx, ctypes.byref(d), cur_stream())
    return y


def pool(be: CudaBackend, x, k, s, pads=(0, 0, 0, 0), is_avg=False, relu=False, count_include_pad=False):
    b, ih, iw, c = x.shape
    oh = (ih + pads[0] + pads[2] - k[0]) // s[0] + 1
    ow = (iw + pads[1] + pads[3] - k[1]) // s[1] + 1
    y = torch.empty((b, oh, ow, c), dtype=torch.float16, device=x.device)
    d = N.PoolDesc()
    d.batch, d.ih, d.iw, d.c, d.oh, d.ow, d.kh, d.kw, d.sh, d.sw = b, ih, iw, c, oh, ow, k[0], k[1], s[0], s[1]
    d.pad_t, d.pad_l, d.is_avg, d.relu, d.count_include_pad = pads[0], pads[1], int(is_avg), int(relu), int(count_include_pad)
    d.x, d.y = ptr(x), ptr(y)
    N.call("sdx_pool", be.ctx, ctypes.byref(d), cur_stream())
    return y


def channel_gate(be: CudaBackend, x, w1, b1, w2, b2, act1_relu=True, hard=True, alpha=0.2, beta=0.5, offset=0.0,
                 sums=None):
    b, h, w, c = x.shape
    r = w1.shape[0]
    s = torch.empty((b, c), dtype=torch.float32, device=x.device)
    scratch = torch.empty(int(N.lib().sdx_channel_gate_scratch_bytes(b, h * w, c)), dtype=torch.uint8, device=x.device)
    d = N.GateDesc()
    d.batch, d.hw, d.c, d.r, d.act1_relu, d.hard = b, h * w, c, r, int(act1_relu), int(hard)
    d.alpha, d.beta, d.offset = alpha, beta, offset
    d.x, d.w1, d.b1, d.w2, d.b2, d.s, d.partial = ptr(x), ptr(w1), ptr(b1), ptr(w2), ptr(b2), ptr(s), ptr(scratch)
    d.sums = ptr(sums)  # a conv's 32-pixel channel sums of x (then x is not read)
    N.call("sdx_channel_gate", be.ctx, ctypes.byref(d), cur_stream())
    return s


def channel_broadcast(be: CudaBackend, x, v, op="mul", relu=False):
    b, c = x.shape[0], x.shape[-1]
    y = torch.empty_like(x)
    N.call("sdx_channel_broadcast", be.ctx, b, x.numel() // (b * c), c, N.EW[op], int(relu), ptr(x), ptr(v), ptr(y),
           cur_stream())
    return y


def resize_nearest(be: CudaBackend, x, scale=2, add=None, add_relu=False, y=None, y_pix_stride=0, y_ch_off=0):
    b, ih, iw, c = x.shape
    oh, ow = ih * scale, iw * scale
    if y is None:
        y = torch.empty((b, oh, ow, c), dtype=torch.float16, device=x.device)
    d = N.ResizeDesc()
    d.batch, d.ih, d.iw, d.c, d.oh, d.ow, d.add_relu = b, ih, iw, c, oh, ow, int(add_relu)
    d.y_pix_stride, d.y_ch_off = y_pix_stride, y_ch_off
    d.x, d.add, d.y = ptr(x), ptr(add), ptr(y)
    N.call("sdx_resize_nearest", be.ctx, ctypes.byref(d), cur_stream())
    return y


def concat_channels(be: CudaBackend, xs):
    pixels = xs[0].numel() // xs[0].shape[-1]
    counts = (ctypes.c_int * len(xs))(*[t.shape[-1] for t in xs])
    ins = (ctypes.c_uint64 * len(xs))(*[ptr(t) for t in xs])
    y = torch.empty(xs[0].shape[:-1] + (sum(t.shape[-1] for t in xs),), dtype=torch.float16, device=xs[0].device)
    N.call("sdx_concat_channels", be.ctx, pixels, len(xs), counts, ins, ptr(y), cur_stream())
    return y


def concat_nearest(be: CudaBackend, xs, scales, out_hw):
    """Channel concat of nearest-upsampled inputs: input i is upsampled by scales[i] to out_hw."""
    nb = xs[0].shape[0]
    oh, ow = out_hw
    counts = (ctypes.c_int * len(xs))(*[t.shape[-1] for t in xs])
    sc = (ctypes.c_int * len(xs))(*[int(s) for s in scales])
    ins = (ctypes.c_uint64 * len(xs))(*[ptr(t) for t in xs])
    y = torch.empty((nb, oh, ow, sum(t.shape[-1] for t in xs)), dtype=torch.float16, device=xs[0].device)
    N.call("sdx_concat_nearest", be.ctx, nb, oh, ow, len(xs), counts, sc, ins, ptr(y), cur_stream())
    return y


def binary(be: CudaBackend, a, b, op="add", relu=False):
    y = torch.empty_like(a)
    N.call("sdx_binary", be.ctx, a.numel(), N.EW[op], int(relu), ptr(a), ptr(b), ptr(y), cur_stream())
    return y


def act(be: CudaBackend, x, kind):
    y = torch.empty_like(x)
    N.call("sdx_act", be.ctx, x.numel(), N.ACT[kind], ptr(x), ptr(y), cur_stream())
    return y


def convert(be: CudaBackend, x, batch, c, hw, x_layout, y_dtype, y_layout):
    shape = (batch, c, hw) if y_layout == N.NCHW else (batch, hw, c)
    y = torch.empty(shape, dtype=y_dtype, device=x.device)
    N.call("sdx_convert", be.ctx, batch, c, hw, _F[x.dtype], x_layout, _F[y_dtype], y_layout, ptr(x), ptr(y),
           cur_stream())
    return y


def layernorm(be: CudaBackend, x, w, b, eps=1e-5):
    c = x.shape[-1]
    y = torch.empty_like(x)
    N.call("sdx_layernorm", be.ctx, x.numel() // c, c, eps, ptr(x), ptr(w), ptr(b), ptr(y), cur_stream())
    return y


def softmax(be: CudaBackend, x, y_dtype=torch.float16):
    c = x.shape[-1]
    y = torch.empty(x.shape, dtype=y_dtype, device=x.device)
    N.call("sdx_softmax", be.ctx, x.numel() // c, c, _F[y_dtype], ptr(x), ptr(y), cur_stream())
    return y


def attention(be: CudaBackend, qkv, batch, t, heads, d, scale):
    y = torch.empty((batch, t, heads * d), dtype=torch.float16, device=qkv.device)
    N.call("sdx_attention", be.ctx, batch, t, heads, d, scale, ptr(qkv), ptr(y), cur_stream())
    return y


def _dt(t: torch.Tensor) -> int:
    return N.F32 if t.dtype == torch.float32 else N.F16


def binary_bcast(be: CudaBackend, a, b, op="add", act="none", y_dtype=torch.float16):
    """y = act(a op b) with numpy broadcasting (sdx_binary_bcast)."""
    shape = torch.broadcast_shapes(a.shape, b.shape)
    r = max(1, len(shape))
    if r > N.BCAST_MAX_RANK:
        raise ValueError("rank above 6")
    y = torch.empty(shape, dtype=y_dtype, device=a.device)
    d = N.BcastDesc()
    d.rank = r
    full = lambda s: [1] * (r - len(s)) + list(s) if len(s) else [1] * r
    for i, (o, x, z) in enumerate(zip(full(shape), full(a.shape), full(b.shape))):
        d.out_shape[i], d.a_shape[i], d.b_shape[i] = o, x, z
    d.op, d.act = N.EW[op], N.ACT[act]
    d.a_dtype, d.b_dtype, d.y_dtype = _dt(a), _dt(b), _dt(y)
    d.a, d.b, d.y = ptr(a.contiguous()), ptr(b.contiguous()), ptr(y)
    N.call("sdx_binary_bcast", be.ctx, ctypes.byref(d), cur_stream())
    return y


def safe_div(be: CudaBackend, a, b, eps, lo, hi):
    y = torch.empty_like(a)
    d = N.SafeDivDesc()
    d.n, d.eps, d.lo, d.hi, d.dtype = a.numel(), eps, lo, hi, _dt(a)
    d.a, d.b, d.y = ptr(a), ptr(b), ptr(y)
    N.call("sdx_safe_div", be.ctx, ctypes.byref(d), cur_stream())
    return y


def channel_shift(be: CudaBackend, x, axis, group_ends, offsets):
    b, h, w, c = x.shape
    y = torch.empty_like(x)
    d = N.ShiftDesc()
    d.batch, d.h, d.w, d.c, d.axis, d.ngroups = b, h, w, c, axis, len(group_ends)
    for i, (e, o) in enumerate(zip(group_ends, offsets)):
        d.group_ends[i], d.offsets[i] = e, o
    d.dtype, d.x, d.y = _dt(x), ptr(x), ptr(y)
    N.call("sdx_channel_shift", be.ctx, ctypes.byref(d), cur_stream())
    return y


def uphead(be: CudaBackend, x, skip, w, bias, scale_h, scale_w, resize_relu=False, skip_relu=False, act="none",
           y_dtype=torch.float16):
    """w: fp32 [oc, c] (the 1x1 conv weights), bias fp32 [oc] or None; x, skip NHWC."""
    b, ih, iw, c = x.shape
    _, oh, ow, _ = skip.shape
    oc = w.shape[0]
    y = torch.empty((b, oh, ow, oc), dtype=y_dtype, device=x.device)
    d = N.UpHeadDesc()
    d.batch, d.ih, d.iw, d.c, d.oh, d.ow, d.oc = b, ih, iw, c, oh, ow, oc
    d.scale_h, d.scale_w = scale_h, scale_w
    d.resize_relu, d.skip_relu, d.act = int(resize_relu), int(skip_relu), N.ACT[act]
    d.x_dtype, d.skip_dtype, d.y_dtype = _dt(x), _dt(skip), _dt(y)
    d.x, d.skip, d.w, d.bias, d.y = ptr(x), ptr(skip), ptr(w), ptr(bias), ptr(y)
    N.call("sdx_uphead", be.ctx, ctypes.byref(d), cur_stream())
    return y


def matmul(be: CudaBackend, a, b, y_dtype=torch.float16):
    """a [.., m, k] x b [.., k, n] with batch broadcast (sdx_matmul)."""
    r = max(a.dim(), b.dim())
    bs = torch.broadcast_shapes(a.shape[:-2], b.shape[:-2])
    y = torch.empty(tuple(bs) + (a.shape[-2], b.shape[-1]), dtype=y_dtype, device=a.device)
    d = N.MatMulDesc()
    d.rank = r
    fa = [1] * (r - a.dim()) + list(a.shape)
    fb = [1] * (r - b.dim()) + list(b.shape)
    for i in range(r):
        d.a_shape[i], d.b_shape[i] = fa[i], fb[i]
    d.a_dtype, d.b_dtype, d.y_dtype = _dt(a), _dt(b), _dt(y)
    d.a, d.b, d.y = ptr(a), ptr(b), ptr(y)
    N.call("sdx_matmul", be.ctx, ctypes.byref(d), cur_stream())
    return y


def gemm_argmax(be: CudaBackend, a, w_packed, n, bias=None):
    """The fused CTC head: per row of a [m, k] (fp16) x packed B [k, n] + bias, (index of the first
    maximum, its softmax probability); the logits are never stored (sdx_gemm_argmax)."""
    m, k = a.shape[0], a.shape[-1]
    idx = torch.empty(m, dtype=torch.int32, device=a.device)
    prob = torch.empty(m, dtype=torch.float32, device=a.device)
    scratch = torch.empty(int(N.lib().sdx_gemm_argmax_scratch_bytes(m, n)), dtype=torch.uint8, device=a.device)
    d = N.GemmArgmaxDesc()
    g = d.gemm
    g.m, g.k, g.n, g.lda = m, k, n, a.stride(0)
    g.act, g.y_dtype, g.add_dtype = N.ACT["none"], N.F32, N.F16
    g.a, g.w, g.bias = ptr(a), ptr(w_packed), ptr(bias)
    d.indices, d.probs, d.scratch = ptr(idx), ptr(prob), ptr(scratch)
    N.call("sdx_gemm_argmax", be.ctx, ctypes.byref(d), cur_stream())
    return idx, prob


def dw_pw(be: CudaBackend, dwd: N.ConvDesc, pwd: N.ConvDesc, x, w_dw, b_dw, w_pw, b_pw=None, in_scale=None, gap=None,
          y=None) -> torch.Tensor:
    """Fused depthwise 3x3 -> 1x1 conv (sdx_dw_pw): the depthwise output is never stored. w_dw / w_pw
    packed by pack_conv for their descriptors; gap: fp32 [pixels / 32, oc] channel sums, or None."""
    if y is None:
        y = torch.empty((pwd.batch, pwd.oh, pwd.ow, pwd.oc), dtype=torch.float16, device=x.device)
    d = N.DwPwDesc()
    d.dw, d.pw = dwd, pwd
    d.dw.x, d.dw.w, d.dw.bias, d.dw.in_scale = ptr(x), ptr(w_dw), ptr(b_dw), ptr(in_scale)
    d.pw.w, d.pw.bias, d.pw.y, d.pw.gap_sums = ptr(w_pw), ptr(b_pw), ptr(y), ptr(gap)
    N.call("sdx_dw_pw", be.ctx, ctypes.byref(d), cur_stream())
    return y


def dw_pw_supported(dwd: N.ConvDesc, pwd: N.ConvDesc) -> bool:
    d = N.DwPwDesc()
    d.dw, d.pw = dwd, pwd
    return bool(N.lib().sdx_dw_pw_supported(ctypes.byref(d)))
