"""Pins of the CPU oracle (no GPU): the reference's own kernel tests restated against the oracle.

The reference stores no golden values for this path; its tests pin the CPU kernels relationally:
  * AVX-512 tier == AVX2 tier bit for bit over a shape matrix (tests/Sdcb.SimdOnnx.Tests/
    Avx512KernelTests.cs:35-93) -> here the AVX-512 and AVX2 builds of the oracle;
  * Winograd vs direct <= 1e-4 * max|out| (EngineTests.cs:184-214);
  * conv + residual == conv then add (EngineTests.cs:163-182);
  * ConvPool == Conv -> MaxPool bit for bit (Avx512KernelTests.cs:121-155);
plus an independent fp64 loop and torch's fp64 conv, and exact shape / index arithmetic.
"""
import os

import numpy as np
import pytest

import oracle as O

ISAS = ["avx2"] + (["avx512"] if O._host_has_avx512() else [])


def rnd(rng, *shape):
    return rng.uniform(-1, 1, size=shape).astype(np.float32)


# (ic, oc, k, stride, h, w, pad_mode, pad_value, residual, act) -- Avx512KernelTests.cs:36-43
DIRECT = [
    (3, 16, 3, 1, 37, 23, 1, 0.0, False, "none"),
    (6, 32, 3, 1, 29, 41, 1, 0.0, False, "relu"),
    (16, 48, 3, 1, 11, 13, 0, 0.25, True, "relu"),
    (20, 20, 3, 2, 17, 19, 0, 0.0, True, "sigmoid"),
    (32, 64, 3, 2, 12, 31, 1, 0.0, False, "gelu"),
    (24, 3, 3, 1, 9, 10, 0, 0.0, False, "none"),
    (40, 36, 1, 1, 7, 33, 0, 0.0, True, "relu"),
    (8, 32, 5, 1, 14, 9, 1, 0.0, False, "relu"),
]


@pytest.mark.parametrize("ic,oc,k,s,h,w,mode,pv,res,act", DIRECT)
def test_direct_conv_isa_builds_bit_identical_and_match_fp64(ic, oc, k, s, h, w, mode, pv, res, act):
    rng = np.random.default_rng(ic * 131 + oc * 7 + k)
    p = k // 2
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    x, wt, b = rnd(rng, 2, h, w, ic), rnd(rng, oc, ic, k, k), rnd(rng, oc)
    add = rnd(rng, 2, oh, ow, oc) if res else None
    outs = []
    for isa in ISAS:
        plan = O.ConvPlan(wt, b, winograd=False, isa=isa)
        outs.append(O.conv(x, plan, strides=(s, s), pads=(p,) * 4, act=act, add=add, pad_mode=mode, pad_value=pv,
                           isa=isa))
    for o in outs[1:]:
        assert np.array_equal(o.view(np.uint32), outs[0].view(np.uint32))
    ref = O.conv_ref64(x, wt, b, strides=(s, s), pads=(p,) * 4, act=act, add=add, pad_mode=mode, pad_value=pv)
    assert np.abs(outs[0] - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


# (ic, oc, h, w, pad_mode, pad_value, residual, act) -- EngineTests.cs:184-214, Avx512KernelTests.cs:62-66
WINO = [
    (16, 16, 9, 11, 0, 0.0, False, "none"),
    (24, 20, 13, 6, 1, 0.0, True, "relu"),
    (32, 48, 4, 4, 0, 0.5, False, "gelu"),
    (64, 16, 17, 23, 1, 0.0, True, "none"),
    (128, 64, 30, 41, 1, 0.0, False, "relu"),
]


@pytest.mark.parametrize("ic,oc,h,w,mode,pv,res,act", WINO)
def test_winograd_matches_direct(ic, oc, h, w, mode, pv, res, act):
    rng = np.random.default_rng(ic * 31 + oc)
    x, wt, b = rnd(rng, 1, h, w, ic), rnd(rng, oc, ic, 3, 3), rnd(rng, oc)
    add = rnd(rng, 1, h, w, oc) if res else None
    kw = dict(pads=(1, 1, 1, 1), act=act, add=add, pad_mode=mode, pad_value=pv)
    direct = O.conv(x, O.ConvPlan(wt, b, winograd=False), **kw)
    wino = O.conv(x, O.ConvPlan(wt, b, winograd=True), **kw)
    assert np.abs(direct - wino).max() < 1e-4 * np.abs(direct).max()
    outs = [O.conv(x, O.ConvPlan(wt, b, winograd=True, isa=i), isa=i, **kw) for i in ISAS]
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


def test_winograd_eligibility_follows_reference():
    # dense 3x3 s1, ic >= 16, ic % 8 == 0 (src/Kernels/NhwcWinograd.cs:28-32)
    L = O.lib()
    assert L.orc_winograd_eligible(1, 3, 3, 1, 1, 64) == 1
    assert L.orc_winograd_eligible(1, 3, 3, 2, 2, 64) == 0
    assert L.orc_winograd_eligible(1, 3, 3, 1, 1, 12) == 0
    assert L.orc_winograd_eligible(1, 5, 5, 1, 1, 64) == 0
    assert L.orc_winograd_eligible(2, 3, 3, 1, 1, 64) == 0


def test_conv_residual_equals_conv_then_add():
    rng = np.random.default_rng(7)
    x, wt, b = rnd(rng, 1, 9, 11, 4), rnd(rng, 8, 4, 3, 3), rnd(rng, 8)
    res = rnd(rng, 1, 9, 11, 8)
    plan = O.ConvPlan(wt, b)
    fused = O.conv(x, plan, pads=(1, 1, 1, 1), add=res)
    plain = O.conv(x, plan, pads=(1, 1, 1, 1))
    assert np.abs(fused - (plain + res)).max() < 1e-4


@pytest.mark.parametrize("ic,oc,wino,act", [(3, 16, False, "none"), (6, 32, False, "relu"), (32, 64, True, "none"),
                                            (24, 20, True, "gelu")])
def test_convpool_equals_conv_then_maxpool(ic, oc, wino, act):
    rng = np.random.default_rng(ic * 13 + oc)
    x, wt, b = rnd(rng, 1, 22, 30, ic), rnd(rng, oc, ic, 3, 3), rnd(rng, oc)
    plan = O.ConvPlan(wt, b, winograd=wino)
    relu = act == "none"
    fused = O.conv_pool(x, plan, act=act, pool_relu=relu)
    pooled = O.maxpool(O.conv(x, plan, pads=(1, 1, 1, 1), act=act), relu=relu)
    assert np.array_equal(fused, pooled)


def test_gemm_isa_builds_identical_and_exact_enough():
    # Avx512KernelTests.cs:83-93
    for m, k, n, tb, act in [(57, 128, 128, False, "none"), (23, 160, 48, True, "gelu"), (5, 64, 20, False, "relu")]:
        rng = np.random.default_rng(m + k + n)
        a, bm, bias = rnd(rng, m, k), (rnd(rng, n, k) if tb else rnd(rng, k, n)), rnd(rng, n)
        outs = [O.gemm(a, O.GemmPlan(bm, bias, trans_b=tb, isa=i), act=act, isa=i) for i in ISAS]
        for o in outs[1:]:
            assert np.array_equal(o, outs[0])
        ref = a.astype(np.float64) @ (bm.T if tb else bm).astype(np.float64) + bias
        if act == "relu":
            ref = np.maximum(ref, 0)
        if act == "none":
            assert np.abs(outs[0] - ref).max() < 1e-4


def test_conv_against_torch_fp64():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(3)
    x, wt, b = rnd(rng, 2, 15, 17, 24), rnd(rng, 32, 24, 3, 3), rnd(rng, 32)
    got = O.conv(x, O.ConvPlan(wt, b, strides=(2, 2)), strides=(2, 2), pads=(1, 1, 1, 1))
    ref = torch.nn.functional.conv2d(torch.from_numpy(np.ascontiguousarray(x.transpose(0, 3, 1, 2))).double(), torch.from_numpy(wt).double(),
                                     torch.from_numpy(b).double(), stride=2, padding=1).numpy().transpose(0, 2, 3, 1)
    assert np.abs(got - ref).max() < 1e-5


def test_depthwise_matches_fp64_and_grouped_loop():
    rng = np.random.default_rng(11)
    x, wt, b = rnd(rng, 2, 13, 9, 32), rnd(rng, 32, 1, 5, 5), rnd(rng, 32)
    got = O.conv(x, O.ConvPlan(wt, b, group=32, strides=(2, 2)), strides=(2, 2), pads=(2, 2, 2, 2), act="hardswish")
    ref = O.conv_ref64(x, wt, b, strides=(2, 2), pads=(2, 2, 2, 2), group=32, act="hardswish")
    assert np.abs(got - ref).max() < 1e-5


def test_convt_and_nearest_and_gate():
    rng = np.random.default_rng(5)
    x = rnd(rng, 1, 3, 4, 8)
    w, b = rnd(rng, 8, 5, 2, 2), rnd(rng, 5)
    y = O.convt(x, w, b)
    ref = np.zeros((1, 6, 8, 5))
    for yy in range(3):
        for xx in range(4):
            for dy in range(2):
                for dx in range(2):
                    ref[0, 2 * yy + dy, 2 * xx + dx] = x[0, yy, xx].astype(np.float64) @ w[:, :, dy, dx] + b
    assert np.abs(y - ref).max() < 1e-5
    # nearest: src = floor(dst / scale) (src/Kernels/Nhwc.Det.cs:173, :180)
    up = O.resize_nearest(x, (2, 2))
    assert np.array_equal(up[0, 5, 7], x[0, 2, 3]) and np.array_equal(up[0, 4, 6], x[0, 2, 3])
    # SE gate: mean -> FC -> relu -> FC -> hard sigmoid
    xs = rnd(rng, 2, 5, 6, 16)
    w1, b1, w2, b2 = rnd(rng, 4, 16), rnd(rng, 4), rnd(rng, 16, 4), rnd(rng, 16)
    s = O.channel_gate(xs, w1, b1, w2, b2, alpha=0.2, beta=0.5)
    m = xs.astype(np.float64).mean(axis=(1, 2))
    z = np.maximum(m @ w1.T + b1, 0) @ w2.T + b2
    assert np.abs(s - np.clip(0.2 * z + 0.5, 0, 1)).max() < 1e-5


def test_activation_cores_match_math():
    xs = np.linspace(-6, 6, 1201, dtype=np.float32)
    L = O.lib()
    import math
    for v in xs[::37]:
        assert abs(L.orc_exp_core(float(v)) - math.exp(v)) <= 2e-6 * math.exp(v)
        assert abs(L.orc_erf_core(float(v)) - math.erf(v)) <= 2e-6
    g = O.act(xs, "gelu")
    ref = 0.5 * xs * (1 + np.array([math.erf(v / math.sqrt(2)) for v in xs]))
    assert np.abs(g - ref).max() < 1e-5


def test_golden_fixture_regression():
    """Committed fixture (tests/golden/make_golden.py) reproduces bit for bit."""
    path = os.path.join(os.path.dirname(__file__), "golden", "oracle_fixtures.npz")
    if not os.path.exists(path):
        pytest.skip("fixture not generated")
    from tests.golden.make_golden import cases
    f = np.load(path)
    for name, fn in cases().items():
        np.testing.assert_array_equal(fn(), f[name], err_msg=name)
