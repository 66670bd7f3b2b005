"""CUDA kernels vs the CPU oracle (the reference's CPU kernels restated), through the C ABI.

Tolerance: relative L2 <= 2e-3 and max-abs <= 1e-2 * max|ref| (tests/parity.py). The shape matrix
follows the reference's own kernel tests (tests/Sdcb.SimdOnnx.Tests/Avx512KernelTests.cs:35-93,
EngineTests.cs:131-214).
"""
import numpy as np
import pytest

import oracle as O
from tests.parity import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from simdonnx_b200 import backend
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return backend.CudaBackend.get(0)


def rnd(rng, *shape, scale=1.0):
    return (rng.uniform(-1, 1, size=shape) * scale).astype(np.float32)


def dev16(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda().half()


def dev32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.float().cpu().numpy()


# ------------------------------------------------------------------------------------------- C1
def test_c1_fused_conv_full_size(be):
    """NHWC 3x3 s1 p1, N=8, 128x128, 64->64, bias, residual add, ReLU."""
    from simdonnx_b200 import backend as B, synth
    rng = synth.Rng(1)
    x = rng.normal("c1.x", (8, 128, 128, 64), 0.1)
    w = rng.normal("c1.w", (64, 64, 3, 3), 0.1)
    b = rng.normal("c1.b", (64,), 0.01)
    res = rng.normal("c1.res", (8, 128, 128, 64), 0.1)
    ref = O.conv(x, O.ConvPlan(w, b), pads=(1, 1, 1, 1), act="relu", add=res)  # Winograd (the reference's path)
    d = B.conv_desc(8, 128, 128, 64, 64, 3, 3, pads=(1, 1, 1, 1), act="relu", y_dtype=torch.float32,
                    add_dtype=torch.float32)
    y = B.conv2d(be, d, dev16(x), B.pack_conv(d, w), bias=dev32(b), add=dev32(res))
    assert_close(host(y), ref, "C1")
    assert be.device_error() == 0


# ------------------------------------------------------------------------------------------- dense conv
CONV_CASES = [
    # ic, oc, k, stride, h, w, residual, act   (Avx512KernelTests.cs:35-43 with zero constant pad)
    (16, 48, 3, 1, 11, 13, True, "relu"),
    (20, 20, 3, 2, 17, 19, True, "sigmoid"),
    (32, 64, 3, 2, 12, 31, False, "gelu"),
    (24, 3, 3, 1, 9, 10, False, "none"),
    (40, 36, 1, 1, 7, 33, True, "relu"),
    (8, 32, 5, 1, 14, 9, False, "relu"),
    (3, 16, 3, 1, 37, 23, False, "hardswish"),
    (6, 32, 3, 1, 29, 41, False, "relu"),
    # Winograd-shaped (Avx512KernelTests.cs:62-66)
    (64, 16, 3, 1, 17, 23, True, "none"),
    (128, 64, 3, 1, 30, 41, False, "relu"),
    (96, 24, 3, 1, 20, 20, False, "none"),
    (256, 256, 3, 1, 8, 8, True, "relu"),
    # kx-in-N with 64-column tap blocks (33..64 outputs)
    (64, 64, 3, 1, 40, 36, False, "relu"),
    (32, 40, 3, 1, 21, 50, False, "hardswish"),
]


@pytest.mark.parametrize("w_terms", [0, 2])
@pytest.mark.parametrize("ic,oc,k,s,h,w,residual,act", CONV_CASES)
def test_conv_shapes(be, ic, oc, k, s, h, w, residual, act, w_terms):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(ic * 131 + oc * 7 + k)
    n, p = 2, k // 2
    x = rnd(rng, n, h, w, ic)
    wt = rnd(rng, oc, ic, k, k, scale=1.0 / np.sqrt(ic * k * k))
    b = rnd(rng, oc)
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    res = rnd(rng, n, oh, ow, oc) if residual else None
    ref = O.conv(x, O.ConvPlan(wt, b, winograd=False), strides=(s, s), pads=(p, p, p, p), act=act, add=res)
    d = B.conv_desc(n, h, w, ic, oc, k, k, stride=(s, s), pads=(p, p, p, p), act=act, w_terms=w_terms)
    y = B.conv2d(be, d, dev16(x), B.pack_conv(d, wt), bias=dev32(b), add=None if res is None else dev16(res))
    assert_close(host(y), ref, f"conv {ic}->{oc} k{k} s{s} terms {w_terms}")


@pytest.mark.parametrize("nb,h,w,ic,oc,residual,act", [
    (4, 128, 128, 128, 128, False, "relu"),  # the UNet 128->128 level: 512 tiles, weights streamed
    (10, 64, 64, 192, 128, True, "none"),    # residual through the TMA-staged epilogue
    (10, 64, 64, 256, 256, False, "relu"),   # two N tiles per pixel-tile pair
    (6, 40, 36, 128, 96, False, "hardswish"),
    (4, 64, 64, 64, 64, False, "relu"),      # kx-in-N, 192-column tiles
])
def test_conv3x3_streamed_weights(be, nb, h, w, ic, oc, residual, act):
    """3x3 convs whose weights do not stay in shared memory: 32-channel stages, and (with enough
    tiles) two pixel tiles per weight stage into two accumulators."""
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(nb * 7 + ic + oc)
    x = rnd(rng, nb, h, w, ic)
    wt = rnd(rng, oc, ic, 3, 3, scale=1.0 / np.sqrt(ic * 9))
    b = rnd(rng, oc)
    res = rnd(rng, nb, h, w, oc) if residual else None
    ref = O.conv(x, O.ConvPlan(wt, b, winograd=False), pads=(1, 1, 1, 1), act=act, add=res)
    d = B.conv_desc(nb, h, w, ic, oc, 3, 3, pads=(1, 1, 1, 1), act=act)
    y = B.conv2d(be, d, dev16(x), B.pack_conv(d, wt), bias=dev32(b), add=None if res is None else dev16(res))
    assert_close(host(y), ref, f"conv3x3 {nb}x{h}x{w} {ic}->{oc}")
    assert be.device_error() == 0


@pytest.mark.parametrize("ic,oc,act,res_nchw,res_f32,y_f32", [
    (32, 3, "none", True, True, True),     # the UNet's final projection + fp32 NCHW input image
    (64, 5, "relu", False, False, False),  # fp16 NHWC residual, fp16 output
    (8, 1, "sigmoid", None, None, True),   # no residual
])
def test_pointwise_small_outputs(be, ic, oc, act, res_nchw, res_f32, y_f32):
    """1x1 convs to at most 8 outputs (per-pixel kernel) against the oracle."""
    from simdonnx_b200 import _native as N, backend as B
    rng = np.random.default_rng(ic + oc)
    nb, h, w = 2, 33, 40
    x = rnd(rng, nb, h, w, ic)
    wt = rnd(rng, oc, ic, 1, 1, scale=1.0 / np.sqrt(ic))
    b = rnd(rng, oc)
    res = None if res_nchw is None else rnd(rng, nb, h, w, oc)
    ref = O.conv(x, O.ConvPlan(wt, b), act=act, add=res)
    d = B.conv_desc(nb, h, w, ic, oc, 1, 1, act=act, y_dtype=torch.float32 if y_f32 else torch.float16,
                    add_dtype=torch.float32 if res_f32 else torch.float16,
                    add_layout=N.NCHW if res_nchw else N.NHWC)
    add = None
    if res is not None:
        r = np.ascontiguousarray(res.transpose(0, 3, 1, 2)) if res_nchw else res
        add = dev32(r) if res_f32 else dev16(r)
    before = int(N.lib().sdx_launch_count())
    y = B.conv2d(be, d, dev16(x), B.pack_conv(d, wt), bias=dev32(b), add=add)
    assert int(N.lib().sdx_launch_count()) - before == 1
    assert_close(host(y), ref, f"pointwise {ic}->{oc}")


@pytest.mark.parametrize("nb,h,w,c,oc,scale,gap,dact", [
    (3, 16, 64, 64, 64, True, True, "hardswish"),     # the det b3 block's shape class, SE scale in, sums out
    (2, 20, 32, 128, 128, True, True, "hardswish"),   # b5: 128 channels (two channel blocks)
    (2, 13, 40, 64, 96, False, False, "relu"),        # ragged tiles: 40 columns, 13 rows
    (1, 8, 32, 128, 32, False, False, "none"),        # no depthwise activation
    (2, 160, 160, 64, 64, True, True, "hardswish"),   # b3 at full resolution
])
def test_depthwise_pointwise_fused(be, nb, h, w, c, oc, scale, gap, dact):
    """Depthwise 3x3 (+activation, per-image input scale) computed tile by tile in shared memory and fed
    to the 1x1 tensor-core conv (sdx_dw_pw) against the oracle's two convs; the fused channel sums
    against sums of the output."""
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(nb * 100 + c + oc)
    x = rnd(rng, nb, h, w, c)
    sc = rng.uniform(0.2, 1, size=(nb, c)).astype(np.float32) if scale else None
    wdw = rnd(rng, c, 1, 3, 3, scale=0.4)
    bdw = rnd(rng, c)
    wpw = rnd(rng, oc, c, 1, 1, scale=1.0 / np.sqrt(c))
    bpw = rnd(rng, oc)
    xin = O.channel_broadcast(x, sc) if scale else x
    mid = O.conv(xin, O.ConvPlan(wdw, bdw, group=c), pads=(1, 1, 1, 1), act=dact)
    mid = mid.astype(np.float16).astype(np.float32)  # the depthwise output is fp16 (as when stored)
    ref = O.conv(mid, O.ConvPlan(wpw, bpw), act="hardswish")
    dwd = B.conv_desc(nb, h, w, c, c, 3, 3, pads=(1, 1, 1, 1), group=c, act=dact)
    pwd = B.conv_desc(nb, h, w, c, oc, 1, 1, act="hardswish")
    if scale:
        dwd.in_scale = 1
    assert B.dw_pw_supported(dwd, pwd)
    g = torch.zeros((nb * h * w // 32, oc), dtype=torch.float32, device="cuda") if gap else None
    y = B.dw_pw(be, dwd, pwd, dev16(x), B.pack_conv(dwd, wdw), dev32(bdw), B.pack_conv(pwd, wpw), dev32(bpw),
                in_scale=dev32(sc) if scale else None, gap=g)
    got = host(y)
    assert_close(got, ref, f"dw+pw {nb}x{h}x{w} {c}->{oc}")
    assert be.device_error() == 0
    if gap:
        want = got.reshape(nb * h * w // 32, 32, oc).sum(axis=1)
        np.testing.assert_allclose(host(g), want, rtol=2e-3, atol=2e-2)


def test_conv_into_channel_slice(be):
    """Epilogue writing into a channel slice of a wider tensor (fused concat)."""
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(5)
    x = rnd(rng, 2, 20, 20, 96)
    wt = rnd(rng, 24, 96, 3, 3, scale=0.05)
    b = rnd(rng, 24)
    ref = O.conv(x, O.ConvPlan(wt, b, winograd=False), pads=(1, 1, 1, 1))
    d = B.conv_desc(2, 20, 20, 96, 24, 3, 3, pads=(1, 1, 1, 1), y_pix_stride=96, y_ch_off=48)
    big = torch.zeros((2, 20, 20, 96), dtype=torch.float16, device="cuda")
    B.conv2d(be, d, dev16(x), B.pack_conv(d, wt), bias=dev32(b), y=big)
    got = host(big)
    assert_close(got[..., 48:72], ref, "slice")
    assert np.all(got[..., :48] == 0) and np.all(got[..., 72:] == 0)


@pytest.mark.parametrize("nb,ih,iw,act", [(2, 64, 48, "hardswish"), (3, 200, 260, "relu"), (1, 640, 640, "none")])
def test_stem_nchw_fp32_input(be, nb, ih, iw, act):
    """Graph-input stem: fp32 NCHW input read directly (boundary relayout fused), 3x3 s2; partial and
    many-tile grids (the tensor-core form builds im2col rows per 128 output pixels)."""
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(9 + ih)
    x = rng.uniform(0, 1, size=(nb, 3, ih, iw)).astype(np.float32)
    wt = rnd(rng, 16, 3, 3, 3, scale=0.5)
    b = rnd(rng, 16)
    ref = O.conv(np.ascontiguousarray(x.transpose(0, 2, 3, 1)), O.ConvPlan(wt, b), strides=(2, 2),
                 pads=(1, 1, 1, 1), act=act)
    d = B.conv_desc(nb, ih, iw, 3, 16, 3, 3, stride=(2, 2), pads=(1, 1, 1, 1), act=act,
                    x_dtype=torch.float32, x_layout=1)
    y = B.conv2d(be, d, dev32(x), B.pack_conv(d, wt), bias=dev32(b))
    assert_close(host(y), ref, "stem")


# ------------------------------------------------------------------------------------------- Gemm
GEMM_CASES = [
    (57, 128, 128, False, "none"),
    (23, 160, 48, True, "gelu"),
    (5, 64, 20, False, "relu"),
    (640, 120, 360, True, "none"),
    (640, 240, 120, True, "hardswish"),
    (300, 120, 6625, True, "none"),
]


@pytest.mark.parametrize("m,k,n,trans_b,act", GEMM_CASES)
def test_gemm(be, m, k, n, trans_b, act):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(m + k + n)
    a = rnd(rng, m, k)
    bm = rnd(rng, n, k) if trans_b else rnd(rng, k, n)
    bias = rnd(rng, n)
    ref = O.gemm(a, O.GemmPlan(bm, bias, trans_b=trans_b), act=act)
    y = B.gemm(be, dev16(a), B.pack_gemm(bm, trans_b), n, bias=dev32(bias), act=act, y_dtype=torch.float32)
    assert_close(host(y), ref, f"gemm {m}x{k}x{n}")


def test_gemm_residual(be):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(77)
    a, bm, bias, r = rnd(rng, 640, 240), rnd(rng, 120, 240), rnd(rng, 120), rnd(rng, 640, 120)
    ref = O.gemm(a, O.GemmPlan(bm, bias, trans_b=True)) + r
    y = B.gemm(be, dev16(a), B.pack_gemm(bm, True), 120, bias=dev32(bias), add=dev16(r))
    assert_close(host(y), ref, "gemm+res")


# ------------------------------------------------------------------------------------------- ConvT
@pytest.mark.parametrize("ic,oc,h,w,act,f32", [(24, 24, 40, 40, "relu", False), (24, 1, 40, 40, "sigmoid", True),
                                               (16, 3, 13, 300, "none", False),
                                               (64, 32, 16, 16, "none", False), (512, 256, 8, 8, "none", False)])
def test_convt(be, ic, oc, h, w, act, f32):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(ic + oc)
    x = rnd(rng, 2, h, w, ic)
    wt = rnd(rng, ic, oc, 2, 2, scale=1 / np.sqrt(ic))
    b = rnd(rng, oc)
    ref = O.convt(x, wt, b, act=act)
    wp = B.pack_convt(wt) if oc >= 8 else dev32(wt)
    y = B.convt(be, dev16(x), wp, ic, oc, 2, 2, bias=dev32(b), act=act,
                y_dtype=torch.float32 if f32 else torch.float16)
    assert_close(host(y), ref, f"convt {ic}->{oc}")


# ------------------------------------------------------------------------------------------- bandwidth ops
@pytest.mark.parametrize("c,k,s,h,w", [(16, 3, 1, 40, 40), (32, 3, 2, 40, 40), (128, 5, 1, 20, 20),
                                       (256, 5, 2, 21, 19), (64, 3, 1, 37, 45), (256, 5, 1, 40, 40),
                                       (64, 5, 1, 23, 93), (16, 3, 1, 30, 170), (32, 5, 1, 17, 85),
                                       (192, 3, 1, 9, 7), (16, 5, 1, 24, 90), (64, 3, 2, 37, 45),
                                       (128, 5, 2, 40, 40), (32, 5, 2, 30, 61), (128, 3, 2, 80, 80)])
def test_depthwise(be, c, k, s, h, w):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(c + k)
    x = rnd(rng, 2, h, w, c)
    wt = rnd(rng, c, 1, k, k, scale=0.3)
    b = rnd(rng, c)
    p = k // 2
    ref = O.conv(x, O.ConvPlan(wt, b, group=c), strides=(s, s), pads=(p, p, p, p), act="hardswish")
    d = B.conv_desc(2, h, w, c, c, k, k, stride=(s, s), pads=(p, p, p, p), group=c, act="hardswish")
    y = B.conv2d(be, d, dev16(x), B.pack_conv(d, wt), bias=dev32(b))
    assert_close(host(y), ref, "depthwise")


@pytest.mark.parametrize("c,k", [(64, 5), (16, 3)])
def test_depthwise_residual_and_scale(be, c, k):
    """Sliding-window depthwise with the SE scale on its load and a residual add before the act."""
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(5 + c)
    h, w = 29, 51
    x = rnd(rng, 2, h, w, c)
    r = rnd(rng, 2, h, w, c)
    sc = rng.uniform(0, 1, size=(2, c)).astype(np.float32)
    wt = rnd(rng, c, 1, k, k, scale=0.3)
    b = rnd(rng, c)
    p = k // 2
    ref = O.conv(O.channel_broadcast(x, sc), O.ConvPlan(wt, b, group=c), pads=(p, p, p, p), act="hardswish", add=r)
    d = B.conv_desc(2, h, w, c, c, k, k, pads=(p, p, p, p), group=c, act="hardswish")
    y = B.conv2d(be, d, dev16(x), B.pack_conv(d, wt), bias=dev32(b), add=dev16(r), in_scale=dev32(sc))
    assert_close(host(y), ref, "dw+scale+residual")


def test_depthwise_with_input_scale(be):
    """SE gate applied on the depthwise load: dw(x * s) == dw of the materialised product."""
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(3)
    x = rnd(rng, 2, 16, 16, 32)
    sc = rng.uniform(0, 1, size=(2, 32)).astype(np.float32)
    wt = rnd(rng, 32, 1, 3, 3)
    b = rnd(rng, 32)
    ref = O.conv(O.channel_broadcast(x, sc), O.ConvPlan(wt, b, group=32), pads=(1, 1, 1, 1), act="hardswish")
    d = B.conv_desc(2, 16, 16, 32, 32, 3, 3, pads=(1, 1, 1, 1), group=32, act="hardswish")
    y = B.conv2d(be, d, dev16(x), B.pack_conv(d, wt), bias=dev32(b), in_scale=dev32(sc))
    assert_close(host(y), ref, "dw+scale")


@pytest.mark.parametrize("avg", [False, True])
def test_pools(be, avg):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(11)
    x = rnd(rng, 2, 19, 26, 32)
    if avg:
        ref = O.avgpool(x, (2, 1), (2, 1))
        y = B.pool(be, dev16(x), (2, 1), (2, 1), is_avg=True)
    else:
        ref = O.maxpool(x, (3, 3), (2, 2), pads=(1, 1, 1, 1), relu=True)
        y = B.pool(be, dev16(x), (3, 3), (2, 2), pads=(1, 1, 1, 1), relu=True)
    assert_close(host(y), ref, "pool")


@pytest.mark.parametrize("c,hw", [(32, 80), (512, 20), (64, 160)])
def test_channel_gate_and_broadcast(be, c, hw):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(c)
    r = c // 4
    x = rnd(rng, 3, hw, hw, c)
    w1, b1, w2, b2 = rnd(rng, r, c), rnd(rng, r), rnd(rng, c, r), rnd(rng, c)
    ref_s = O.channel_gate(x, w1, b1, w2, b2, act1_relu=True, hard=True, alpha=0.2, beta=0.5)
    s = B.channel_gate(be, dev16(x), dev32(w1), dev32(b1), dev32(w2), dev32(b2), alpha=0.2, beta=0.5)
    assert_close(host(s), ref_s, "gate")
    y = B.channel_broadcast(be, dev16(x), s)
    assert_close(host(y), O.channel_broadcast(x, ref_s), "x*s")


def test_channel_gate_batch_invariant(be):
    """An image's gate is bit-identical whichever batch (and FC block of images) it runs in."""
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(41)
    c, r, hw = 256, 64, 40
    x = rnd(rng, 9, hw, hw, c)
    w1, b1, w2, b2 = rnd(rng, r, c), rnd(rng, r), rnd(rng, c, r), rnd(rng, c)
    args = (dev32(w1), dev32(b1), dev32(w2), dev32(b2))
    s9 = host(B.channel_gate(be, dev16(x), *args, alpha=0.2, beta=0.5))
    s1 = host(B.channel_gate(be, dev16(x[5:6]), *args, alpha=0.2, beta=0.5))
    np.testing.assert_array_equal(s9[5:6], s1)
    ref_s = O.channel_gate(x, w1, b1, w2, b2, act1_relu=True, hard=True, alpha=0.2, beta=0.5)
    assert_close(s9, ref_s, "gate b9")


def test_concat_nearest(be):
    """Upsample-and-concat in one pass == resize each input then concat (bit exact: pure copies)."""
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(23)
    parts = [rnd(rng, 2, 5, 6, 24), rnd(rng, 2, 10, 12, 16), rnd(rng, 2, 20, 24, 8), rnd(rng, 2, 40, 48, 24)]
    scales = (8, 4, 2, 1)
    ref = O.concat_channels([O.resize_nearest(p, (s, s)) if s > 1 else p for p, s in zip(parts, scales)])
    y = B.concat_nearest(be, [dev16(p) for p in parts], scales, (40, 48))
    np.testing.assert_array_equal(host(y), ref.astype(np.float16).astype(np.float32))


def test_resize_add_and_concat(be):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(21)
    x, lat = rnd(rng, 2, 10, 10, 96), rnd(rng, 2, 20, 20, 96)
    assert_close(host(B.resize_nearest(be, dev16(x), 2, add=dev16(lat))), O.resize_nearest(x, (2, 2), add=lat), "up+add")
    parts = [rnd(rng, 2, 8, 8, 24) for _ in range(4)]
    assert_close(host(B.concat_channels(be, [dev16(p) for p in parts])), O.concat_channels(parts), "concat")
    big = torch.zeros((2, 40, 40, 96), dtype=torch.float16, device="cuda")
    B.resize_nearest(be, dev16(parts[0]), 5, y=big, y_pix_stride=96, y_ch_off=24)
    assert_close(host(big)[..., 24:48], O.resize_nearest(parts[0], (5, 5)), "up into slice")


def test_layernorm_softmax_attention(be):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(31)
    x = rnd(rng, 4, 40, 120)
    w, b = rnd(rng, 120), rnd(rng, 120)
    assert_close(host(B.layernorm(be, dev16(x), dev32(w), dev32(b))), O.layernorm(x, w, b), "layernorm")
    s = rnd(rng, 64, 40, scale=4.0)
    assert_close(host(B.softmax(be, dev16(s), torch.float32)), O.softmax(s), "softmax")
    nb, t, heads, dh = 3, 40, 8, 15
    qkv = rnd(rng, nb, t, 3, heads, dh)
    q, k, v = (np.ascontiguousarray(qkv[:, :, i].transpose(0, 2, 1, 3)) for i in range(3))
    scale = dh ** -0.5
    p = O.softmax(O.binary(O.matmul(q, np.ascontiguousarray(k.transpose(0, 1, 3, 2))),
                           np.full((nb, heads, t, t), scale, np.float32), "mul"))
    ref = O.matmul(p, v).transpose(0, 2, 1, 3).reshape(nb, t, heads * dh)
    y = B.attention(be, dev16(qkv), nb, t, heads, dh, scale)
    assert_close(host(y), ref, "attention")


def test_convert_layouts(be):
    from simdonnx_b200 import backend as B, _native as N
    rng = np.random.default_rng(41)
    x = rnd(rng, 2, 3, 7, 5)
    y = B.convert(be, dev32(x), 2, 3, 35, N.NCHW, torch.float16, N.NHWC)
    assert_close(host(y).reshape(2, 7, 5, 3), x.transpose(0, 2, 3, 1), "nchw->nhwc")
    z = B.convert(be, y, 2, 3, 35, N.NHWC, torch.float32, N.NCHW)
    assert_close(host(z).reshape(x.shape), x, "roundtrip")


@pytest.mark.parametrize("c,c_out,x32", [(3, 8, True), (3, 16, False), (8, 8, True), (5, 8, False)])
def test_convert_channel_padding(be, c, c_out, x32):
    """NCHW -> NHWC fp16 zero-padded to c_out channels (sdx_convert_pad): values exact to fp16, pad zero."""
    import ctypes
    from simdonnx_b200 import backend as B, _native as N
    rng = np.random.default_rng(c * c_out)
    x = rnd(rng, 3, c, 9, 13)
    xd = dev32(x) if x32 else dev16(x)
    y = torch.full((3, 9, 13, c_out), 7.0, dtype=torch.float16, device="cuda")
    N.call("sdx_convert_pad", be.ctx, 3, c, c_out, 9 * 13, N.F32 if x32 else N.F16, N.NCHW, N.F16, N.NHWC,
           B.ptr(xd), B.ptr(y), B.cur_stream())
    got = host(y)
    want = np.zeros((3, 9, 13, c_out), np.float32)
    want[..., :c] = x.transpose(0, 2, 3, 1).astype(np.float16).astype(np.float32)
    np.testing.assert_array_equal(got, want)


def test_bounded_wait_reports_and_recovers(be):
    """A kernel whose wait can never end gives up after its limit, records its code and returns;
    the host sees SDX_ERR_DEVICE, and the context is usable again after clearing."""
    from simdonnx_b200 import _native as N, backend as B
    be.clear_device_error()
    N.call("sdx_selftest_bounded_wait", be.ctx, 50, B.cur_stream())
    with pytest.raises(N.SdxError) as ei:
        be.sync()
    assert ei.value.code == 5
    assert be.device_error() == 0x1F0
    be.clear_device_error()
    test_resize_add_and_concat(be)
    assert be.device_error() == 0


# ------------------------------------------------------------------------------------------- image session
def _image_tensor_ref(img, lut, oh, ow, pads, swap):
    """ImageToTensor as the oracle runner computes it (replicate padding, lut, optional R/B swap)."""
    ih, iw = img.shape[1], img.shape[2]
    sy = np.clip(np.arange(oh) - pads[0], 0, ih - 1)
    sx = np.clip(np.arange(ow) - pads[1], 0, iw - 1)
    px = img[:, sy][:, :, sx]
    order = (2, 1, 0) if swap else (0, 1, 2)
    return np.stack([lut[c][px[..., order[c]]] for c in range(3)], axis=1).astype(np.float32)


@pytest.mark.parametrize("bpp,swap,ih,iw,oh,ow,pads", [(3, False, 64, 96, 64, 96, (0, 0)),
                                                       (4, True, 30, 41, 37, 53, (3, 5)),
                                                       (3, True, 70, 33, 70, 33, (0, 0))])
def test_image_conv_fused_stem(be, bpp, swap, ih, iw, oh, ow, pads):
    """u8 images -> lut -> the 3->16 3x3 s2 stem in one kernel == image_to_tensor then the conv."""
    import ctypes
    from simdonnx_b200 import backend as B, _native as N
    rng = np.random.default_rng(ih * iw + bpp)
    nb = 2
    img = rng.integers(0, 256, size=(nb, ih, iw, bpp), dtype=np.uint8)
    lut = rng.uniform(-2, 2, size=(3, 256)).astype(np.float32)
    wt = rnd(rng, 16, 3, 3, 3, scale=0.3)
    b = rnd(rng, 16)
    x = _image_tensor_ref(img, lut, oh, ow, pads, swap)          # NCHW fp32
    ref = O.conv(np.ascontiguousarray(x.transpose(0, 2, 3, 1)), O.ConvPlan(wt, b), strides=(2, 2), pads=(1, 1, 1, 1),
                 act="hardswish")
    cd = B.conv_desc(nb, oh, ow, 3, 16, 3, 3, stride=(2, 2), pads=(1, 1, 1, 1), act="hardswish",
                     x_dtype=torch.float32, x_layout=N.NCHW)
    wp = B.pack_conv(cd, wt)
    y = torch.empty((nb, cd.oh, cd.ow, 16), dtype=torch.float16, device="cuda")
    src, lut_d, bias_d = torch.from_numpy(img).cuda(), dev32(lut), dev32(b)
    d = N.ImageConvDesc()
    im = d.image
    im.batch, im.ih, im.iw, im.bpp, im.swap_rb = nb, ih, iw, bpp, int(swap)
    im.oh, im.ow, im.pad_t, im.pad_l, im.y_nhwc_f16 = oh, ow, pads[0], pads[1], 0
    im.stride, im.image_bytes = iw * bpp, ih * iw * bpp
    im.src, im.lut, im.y = B.ptr(src), B.ptr(lut_d), 0
    cd.x, cd.w, cd.bias, cd.y = 0, B.ptr(wp), B.ptr(bias_d), B.ptr(y)
    d.conv = cd
    N.call("sdx_image_conv", be.ctx, ctypes.byref(d), B.cur_stream())
    assert_close(host(y), ref, "image conv")
    assert be.device_error() == 0


@pytest.mark.parametrize("ic,oc1,h,w,act1,f32", [(24, 24, 20, 30, "relu", True), (16, 8, 9, 17, "none", False),
                                                 (32, 16, 13, 64, "relu", True)])
def test_convt_chain(be, ic, oc1, h, w, act1, f32):
    """ConvT 2x2 (ic -> oc1, act1) then ConvT 2x2 (oc1 -> 1, sigmoid) in one kernel == the two ConvTs
    one after the other (the intermediate kept in fp32)."""
    import ctypes
    from simdonnx_b200 import backend as B, _native as N
    rng = np.random.default_rng(ic * 7 + oc1)
    nb = 2
    x = rnd(rng, nb, h, w, ic)
    w1 = rnd(rng, ic, oc1, 2, 2, scale=1 / np.sqrt(ic))
    b1 = rnd(rng, oc1)
    w2 = rnd(rng, oc1, 1, 2, 2, scale=1 / np.sqrt(oc1))
    b2 = rnd(rng, 1)
    ref = O.convt(O.convt(x, w1, b1, act=act1), w2, b2, act="sigmoid")
    y = torch.empty((nb, 4 * h, 4 * w, 1), dtype=torch.float32 if f32 else torch.float16, device="cuda")
    xd, w1p, b1d, w2d, b2d = dev16(x), B.pack_convt(w1), dev32(b1), dev32(w2), dev32(b2)
    d = N.ConvtChainDesc()
    f = d.first
    f.batch, f.ih, f.iw, f.ic, f.oc, f.kh, f.kw = nb, h, w, ic, oc1, 2, 2
    f.act, f.y_dtype = N.ACT[act1], N.F16
    f.x, f.w, f.bias, f.y = B.ptr(xd), B.ptr(w1p), B.ptr(b1d), 0
    d.oc2, d.kh2, d.kw2, d.act2 = 1, 2, 2, N.ACT["sigmoid"]
    d.y_dtype = N.F32 if f32 else N.F16
    d.w2, d.bias2, d.y = B.ptr(w2d), B.ptr(b2d), B.ptr(y)
    N.call("sdx_convt_chain", be.ctx, ctypes.byref(d), B.cur_stream())
    assert_close(host(y), ref, f"convt chain {ic}->{oc1}->1")
    assert be.device_error() == 0


@pytest.mark.parametrize("nb,ic,oc,k,h,w", [
    (2, 64, 96, 1, 20, 24), (2, 32, 64, 3, 16, 22), (2, 256, 96, 1, 40, 40),
    (8, 64, 96, 1, 96, 96),  # ~4 tiles per CTA: each epilogue group prefetches its next tile's residual rows
])
def test_conv_upsampled_residual(be, nb, ic, oc, k, h, w):
    """FPN top-down add fused into the lateral conv: y = conv(x) + nearest_up2(r), r on the half grid."""
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(ic + oc + k)
    x = rnd(rng, nb, h, w, ic)
    r = rnd(rng, nb, h // 2, w // 2, oc)
    wt = rnd(rng, oc, ic, k, k, scale=1 / np.sqrt(ic * k * k))
    b = rnd(rng, oc)
    p = k // 2
    ref = O.resize_nearest(r, (2, 2), add=O.conv(x, O.ConvPlan(wt, b), pads=(p, p, p, p)))
    d = B.conv_desc(nb, h, w, ic, oc, k, k, pads=(p, p, p, p))
    d.add_up = 2
    y = B.conv2d(be, d, dev16(x), B.pack_conv(d, wt), bias=dev32(b), add=dev16(r))
    assert_close(host(y), ref, f"conv {k}x{k} + up2 residual")
    assert be.device_error() == 0


@pytest.mark.parametrize("nb,h,w,ic,oc,up,act", [
    (2, 16, 16, 64, 96, False, "hardswish"),  # two-term source weights (ic < 128)
    (2, 16, 16, 128, 96, True, "none"),       # one-term source weights, FPN top-down residual
    (64, 16, 24, 64, 96, True, "none"),       # 3 tiles per image, 2 per CTA: CTA ranges cross images
    (300, 8, 16, 40, 24, False, "relu"),      # 1 tile per image: a weight reload every tile; K padded
    (5, 40, 40, 256, 96, True, "none"),       # 1600 pixels per image: pixel tiles (rows would straddle)
    (3, 20, 12, 64, 32, False, "hardswish"),  # 240 pixels per image, thin output
])
def test_pointwise_per_image_scale(be, nb, h, w, ic, oc, up, act):
    """1x1 conv of the SE product x * s (s per image and channel) with the weights scaled per image
    (sdx_conv_desc.in_scale on the tensor-core route, sdx_conv_scaled_weights_bytes of scratch)
    against the oracle's conv of the materialised fp32 product."""
    from simdonnx_b200 import _native as N, backend as B
    rng = np.random.default_rng(nb + ic + oc)
    x = rnd(rng, nb, h, w, ic)
    sc = rng.uniform(0, 1, size=(nb, ic)).astype(np.float32)
    wt = rnd(rng, oc, ic, 1, 1, scale=1 / np.sqrt(ic))
    b = rnd(rng, oc)
    conv = O.conv(O.channel_broadcast(x, sc), O.ConvPlan(wt, b), act=act)
    d = B.conv_desc(nb, h, w, ic, oc, 1, 1, act=act)
    sd = dev32(sc)
    d.in_scale = B.ptr(sd)  # set before packing: the packed layout depends on it
    r = None
    if up:
        r = rnd(rng, nb, h // 2, w // 2, oc)
        conv = O.resize_nearest(r, (2, 2), add=conv)
        d.add_up = 2
    kpad = {40: 48, 64: 64, 128: 128, 256: 256}[ic]
    assert B.conv_scaled_weights_bytes(d) == nb * 2 * ((oc + 15) // 16 * 16) * kpad * 2  # [nb][2 terms][rows][kpad]
    wp = B.pack_conv(d, wt)
    before = int(N.lib().sdx_launch_count())
    y = B.conv2d(be, d, dev16(x), wp, bias=dev32(b), add=dev16(r) if up else None, in_scale=sd)
    assert_close(host(y), conv, f"pointwise x*s {nb}x{h}x{w} {ic}->{oc}")
    assert be.device_error() == 0
    assert int(N.lib().sdx_launch_count()) - before == 2  # the weight scaling, then the conv


def test_pointwise_per_image_scale_rejects_wide_outputs(be):
    """256 output channels (two N tiles): no per-image form, the call is refused before any launch."""
    import ctypes
    from simdonnx_b200 import _native as N, backend as B
    d = B.conv_desc(2, 40, 40, 64, 256, 1, 1)
    d.in_scale = 1
    assert B.conv_scaled_weights_bytes(d) == 0
    d.x = d.w = d.y = d.w_scaled = 1 << 20  # never dereferenced: refused before any launch
    before = int(N.lib().sdx_launch_count())
    assert N.lib().sdx_conv2d(be.ctx, ctypes.byref(d), None) != 0
    assert int(N.lib().sdx_launch_count()) == before


@pytest.mark.gpu
@pytest.mark.parametrize("ic,oc,h,w,act", [(16, 32, 32, 40, "hardswish"), (64, 128, 16, 16, "relu"),
                                           (128, 256, 8, 12, "none")])
def test_conv_channel_sums_feed_gate(be, ic, oc, h, w, act):
    """SE pooling fused into a 1x1 conv: the conv also writes fp32 channel sums of each 32-pixel run of
    its output, and the gate reading them equals the oracle gate over the reference output."""
    from simdonnx_b200 import _native as N, backend as B
    rng = np.random.default_rng(ic + oc + h)
    nb = 3
    x = rnd(rng, nb, h, w, ic)
    wt = rnd(rng, oc, ic, 1, 1, scale=1 / np.sqrt(ic))
    b = rnd(rng, oc)
    ref = O.conv(x, O.ConvPlan(wt, b), act=act)
    d = B.conv_desc(nb, h, w, ic, oc, 1, 1, act=act)
    sums = torch.full((nb * h * w // 32, oc), float("nan"), dtype=torch.float32, device="cuda")
    d.gap_sums = B.ptr(sums)
    y = B.conv2d(be, d, dev16(x), B.pack_conv(d, wt), bias=dev32(b))
    assert_close(host(y), ref, f"1x1 conv {ic}->{oc} with sums")
    assert_close(host(sums), ref.reshape(-1, 32, oc).sum(axis=1), "32-pixel channel sums")
    r = oc // 4
    w1, b1, w2, b2 = rnd(rng, r, oc), rnd(rng, r), rnd(rng, oc, r), rnd(rng, oc)
    ref_s = O.channel_gate(ref, w1, b1, w2, b2, act1_relu=True, hard=True, alpha=0.2, beta=0.5)
    s = B.channel_gate(be, y, dev32(w1), dev32(b1), dev32(w2), dev32(b2), alpha=0.2, beta=0.5, sums=sums)
    assert_close(host(s), ref_s, "gate from the conv's sums")
    assert be.device_error() == 0
    # shapes the fused sums do not cover are refused before anything is enqueued
    d3 = B.conv_desc(nb, 3, 5, ic, oc, 1, 1, act=act)
    d3.gap_sums = B.ptr(sums)
    with pytest.raises(N.SdxError):
        B.conv2d(be, d3, dev16(rnd(rng, nb, 3, 5, ic)), B.pack_conv(d3, wt), bias=dev32(b))


# thin 1x1 convs run pixel-folded (F consecutive pixels per GEMM row, block-diagonal weights)
FOLD_CASES = [
    # ic, oc, h, w, residual, act, expected fold (oc * fold = 64 columns)
    (16, 32, 16, 24, False, "hardswish", 2),   # det b1.pw shape class
    (8, 32, 32, 32, True, "gelu", 2),
    (16, 16, 16, 16, True, "relu", 4),
    (8, 16, 8, 32, False, "hardswish", 4),
    (32, 64, 16, 16, True, "relu", 1),         # det b2.pw: 64 columns already
    (16, 32, 10, 10, False, "hardswish", 1),   # 200 pixels: no fold (not whole 32-row runs)
]


@pytest.mark.parametrize("ic,oc,h,w,residual,act,fold", FOLD_CASES)
def test_pointwise_pixel_folded(be, ic, oc, h, w, residual, act, fold):
    """1x1 convs with oc * F = 128 run F pixels per GEMM row: against the oracle, with the fused
    32-pixel channel sums (per pixel run, not per folded row) and an fp16 residual."""
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(ic * 7 + oc + h)
    nb = 2
    x = rnd(rng, nb, h, w, ic)
    wt = rnd(rng, oc, ic, 1, 1, scale=1 / np.sqrt(ic))
    b = rnd(rng, oc)
    res = rnd(rng, nb, h, w, oc) if residual else None
    ref = O.conv(x, O.ConvPlan(wt, b), act=act, add=res)
    d = B.conv_desc(nb, h, w, ic, oc, 1, 1, act=act)
    packed = B.pack_conv(d, wt)
    if fold > 1:
        # F copies of the weights on the block diagonal: 2 fp16 terms x 64 rows x F * ic columns
        assert packed.numel() == 2 * 2 * 64 * ic * fold, packed.numel()
    sums = None
    if (nb * h * w) % 32 == 0:
        sums = torch.full((nb * h * w // 32, oc), float("nan"), dtype=torch.float32, device="cuda")
        d.gap_sums = B.ptr(sums)
    y = B.conv2d(be, d, dev16(x), packed, bias=dev32(b), add=None if res is None else dev16(res))
    got = host(y)
    assert_close(got, ref, f"1x1 {ic}->{oc} fold {fold}")
    if sums is not None:
        # the sums are of the stored fp16 output, per run of 32 pixels
        want = got.astype(np.float64).reshape(-1, 32, oc).sum(axis=1)
        np.testing.assert_allclose(host(sums), want, rtol=2e-5, atol=2e-4)
    assert be.device_error() == 0
