"""Host-side plan logic: arena safety, CUDA rewrites, config shapes (no GPU needed)."""
import itertools

import numpy as np
import pytest

from simdonnx_b200 import configs
from simdonnx_b200.plan import _param_refs
from simdonnx_b200.session import cuda_rewrite


def _live_ranges(P):
    first, last = {}, {}
    for i, n in enumerate(P.nodes):
        for v in n.outs:
            t = P.values[v].alias[0] if P.values[v].alias else v
            first.setdefault(t, i)
        for v in list(n.ins) + _param_refs(n.p) + list(n.outs):
            if v in P.values and not P.values[v].is_const:
                t = P.values[v].alias[0] if P.values[v].alias else v
                last[t] = i
    for v in P.inputs:
        first[v], last[v] = -1, len(P.nodes)
    last[P.output] = len(P.nodes)
    return first, last


@pytest.mark.parametrize("builder,batch", [(configs.build_det, 2), (configs.build_c1, 8)])
def test_arena_never_overlaps_live_values(builder, batch):
    P = cuda_rewrite(builder(batch=batch))
    P.plan_arena()
    first, last = _live_ranges(P)
    size = lambda v: (P.values[v].nbytes + 255) // 256 * 256
    for a, b in itertools.combinations(list(first), 2):
        if first[a] <= last[b] and first[b] <= last[a]:
            oa, ob = P.offsets[a], P.offsets[b]
            assert not (oa < ob + size(b) and ob < oa + size(a)), (a, b)
    assert all(P.offsets[v] % 256 == 0 for v in first)
    assert P.arena_bytes >= max(P.offsets[v] + size(v) for v in first)


def test_inputs_first_and_back_to_back():
    P = cuda_rewrite(configs.build_c1())
    P.plan_arena()
    assert P.offsets[P.inputs[0]] == 0
    assert P.offsets[P.inputs[1]] == (P.values[P.inputs[0]].nbytes + 255) // 256 * 256


def test_det_rewrites():
    P = cuda_rewrite(configs.build_det(batch=1))
    # SE products folded into the convs that read them: every depthwise conv, and the FPN laterals
    # in2-in4 (per-image scaled weights, with their scratch as a second output); the product at the
    # 20x20 tap stays (in5 reads 512 channels: its per-image weights would not stay resident)
    fused = [n for n in P.nodes if n.op == "Conv" and getattr(n.p, "in_scale", None)]
    assert len(fused) == 14
    lat = sorted(n.name for n in fused if n.p.group == 1)
    assert lat == ["fpn.in2", "fpn.in3", "fpn.in4"]
    for n in fused:
        if n.p.group == 1:
            assert n.outs[-1] == n.p.w_scaled and P.values[n.p.w_scaled].dtype == "u8"
    assert [n.name for n in P.nodes if n.op == "Elementwise"] == ["b12.se.mul"]
    # the FPN concat of three upsampled maps and p2 becomes one ConcatNearest node (no resize nodes)
    assert not any(n.op == "Concat" for n in P.nodes)
    cn = [n for n in P.nodes if n.op == "ConcatNearest"]
    assert len(cn) == 1 and cn[0].ins == ["fpn.p5", "fpn.p4", "fpn.p3", "fpn.p2"] and cn[0].p == (8, 4, 2, 1)
    assert not any(n.op == "ResizeNearest" and n.outs[0] in ("fpn.p5u", "fpn.p4u", "fpn.p3u") for n in P.nodes)


def test_dw_pw_fusion_rewrite():
    """With the fusion on, the 3x3 stride-1 depthwise convs over 64 / 128 channels become DwPw nodes with
    their pointwise convs; the depthwise outputs are never stored; b3 (160 wide) keeps its fused SE sums,
    b5 (80 wide: no whole 32-pixel runs per tile row) gives them up and its gate reads the tensor."""
    from simdonnx_b200 import session as S
    old = S.DW_PW_FUSION
    S.DW_PW_FUSION = True
    try:
        P = cuda_rewrite(configs.build_det(batch=1))
    finally:
        S.DW_PW_FUSION = old
    dwpw = [n for n in P.nodes if n.op == "DwPw"]
    assert [n.name for n in dwpw] == ["b3.pw", "b5.pw"]
    assert all(getattr(n.p[0], "in_scale", None) for n in dwpw)
    assert "b3.dw" not in P.values and "b5.dw" not in P.values
    assert len(dwpw[0].outs) == 2 and len(dwpw[1].outs) == 1
    gate5 = [n for n in P.nodes if n.name == "b5.se"][0]
    assert len(gate5.ins) == 3
    P.plan_arena()


def test_dw_pw_supported_activations():
    """sdx_dw_pw applies the depthwise activation as a compile-time constant of its row loop: none,
    relu and hardswish are admitted, the others refused (the session keeps the two convs)."""
    from simdonnx_b200 import backend as B
    for act, ok in [("none", True), ("relu", True), ("hardswish", True), ("sigmoid", False), ("gelu", False)]:
        dwd = B.conv_desc(2, 16, 64, 64, 64, 3, 3, pads=(1, 1, 1, 1), group=64, act=act)
        pwd = B.conv_desc(2, 16, 64, 64, 64, 1, 1, act="sigmoid")
        assert B.dw_pw_supported(dwd, pwd) == ok, act


def test_concat_partial_aliasing_with_pool_reader():
    """UNet skip: a conv output read by a max pool and a concat is written into its concat slice
    (the pool reads the slice in place); a ConvTranspose input is still copied by the concat node."""
    from simdonnx_b200.plan import PoolP
    P = configs.build_unet(batch=1, hw=64)
    R = cuda_rewrite(P)
    cats = [n for n in R.nodes if n.op == "Concat"]
    assert len(cats) == 4
    for n in cats:
        skip, up = n.ins[1], n.ins[0]
        assert n.p == (False, True)
        assert R.values[skip].alias == (n.outs[0], R.shape(up)[3])
        assert R.values[up].alias is None
    pools = [n for n in R.nodes if n.op == "MaxPool"]
    assert all(R.values[p.ins[0]].alias for p in pools)
    # the RGB input widened to 8 fp16 channels for the first (tensor-core) conv, weights padded
    cv = R.nodes[0]
    assert cv.op == "Convert" and R.values[cv.outs[0]].shape == (1, 64, 64, 8) and R.values[cv.outs[0]].dtype == "f16"
    c1 = R.nodes[1]
    assert c1.name == "e0.c1" and c1.ins[0] == cv.outs[0] and R.values[c1.ins[1]].const.shape == (32, 8, 3, 3)
    assert not R.values[c1.ins[1]].const[:, 3:].any()


def test_concat_slice_aliasing_without_upsampling():
    """A Concat of conv outputs is written in place by its producers (slice offsets 0, c0, ...)."""
    b = configs._Builder(3)
    P = b.P
    x = P.add_value("x", (1, 8, 8, 16))
    P.inputs = [x]
    a1 = b.conv("a1", x, 16, 1)
    a2 = b.conv("a2", x, 24, 3)
    y = P.add_value("y", (1, 8, 8, 40))
    P.add_node("Concat", [a1, a2], [y], None, "cat")
    P.output = y
    R = cuda_rewrite(P)
    assert not any(n.op in ("Concat", "ConcatNearest") for n in R.nodes)
    assert (R.values["a1"].alias, R.values["a2"].alias) == (("y", 0), ("y", 16))


def test_det_shapes_follow_onnx_formulas():
    P = configs.build_det(batch=1)
    assert P.shape("stem") == (1, 320, 320, 16)
    assert P.shape("b12.se.y") == (1, 20, 20, 512)
    assert P.shape("fpn.fuse") == (1, 160, 160, 96)
    assert P.shape(P.output) == (1, 640, 640, 1)


def test_seeded_inputs_are_batch_prefix_stable():
    a = configs.build_det(batch=1)
    b = configs.build_det(batch=3)
    xa = a.feeds[a.input]()
    xb = b.feeds[b.input]()
    assert np.array_equal(xa[0], xb[0])
    assert xb.min() >= 0 and xb.max() < 1


def test_image_front_semantics_on_oracle():
    """The image front (u8 pixels -> lut -> fp32 NCHW) matches a direct restatement of the
    reference shader: replicate padding, per-channel table, optional R/B swap."""
    import numpy as np
    from oracle.runner import OracleSession
    from simdonnx_b200.plan import ExecPlan, ImageP
    P = ExecPlan()
    img = P.add_value("img", (2, 5, 7, 4), "u8", "nhwc")
    lut = P.add_const("lut", (np.arange(768, dtype=np.float32).reshape(3, 256) * 0.01))
    y = P.add_value("y", (2, 3, 9, 11), "f32", "nchw")
    P.add_node("ImageToTensor", [img], [y], ImageP(lut, bpp=4, swap_rb=True, pads=(1, 2)), "image")
    P.inputs, P.input, P.output = [img], img, y
    rng = np.random.default_rng(3)
    pix = rng.integers(0, 256, (2, 5, 7, 4), dtype=np.uint8)
    got = OracleSession(P).run({img: pix})[y]
    table = P.values[lut].const
    for n in range(2):
        for c in range(3):
            for oy in range(9):
                for ox in range(11):
                    sy, sx = min(max(oy - 1, 0), 4), min(max(ox - 2, 0), 6)
                    byte = pix[n, sy, sx, 2 - c]  # swapped: channel 0 from byte 2
                    assert got[n, c, oy, ox] == table[c, byte]


def test_conv_pool_split_for_cuda():
    """ConvP.Pool (fused 2x2/2 max pool) runs on CUDA as conv -> MaxPool (+relu) over an arena value."""
    from simdonnx_b200.plan import PoolP
    b = configs._Builder(5)
    P = b.P
    x = P.add_value("x", (1, 17, 22, 16))
    P.inputs, P.input = [x], x
    y = b.conv("cp", x, 32, 3, act="relu", pool=PoolP((2, 2), (2, 2), fuse_relu=True))
    P.output = y
    R = cuda_rewrite(P)
    ops = [(n.op, n.outs[0]) for n in R.nodes]
    assert ops == [("Conv", "cp.prepool"), ("MaxPool", "cp")]
    assert R.shape("cp.prepool") == (1, 17, 22, 32) and R.shape("cp") == (1, 8, 11, 32)
    assert R.nodes[1].p.fuse_relu


def test_device_feed_generator_matches_host_generator():
    """plan.feeds_dev (torch SplitMix64, used by bench.py for the N=256 input) produces exactly the
    values of plan.feeds (numpy SplitMix64): same bits, on small shapes and across chunk edges."""
    import torch
    from simdonnx_b200 import synth
    r = synth.Rng(2)
    assert np.array_equal(r.uniform("input", (2, 3, 40, 24)), r.uniform_torch("input", (2, 3, 40, 24), "cpu").numpy())
    assert np.array_equal(r.bytes("image", (2, 17, 9, 3)), r.bytes_torch("image", (2, 17, 9, 3), "cpu").numpy())
    assert np.array_equal(synth.uniform(99, (1001,), -1.0, 2.0),
                          synth.uniform_torch(99, (1001,), "cpu", -1.0, 2.0, chunk=64).numpy())
    p = configs.build_det(batch=1, hw=64)
    (k, f), = p.feeds.items()
    assert np.array_equal(f(), p.feeds_dev[k](torch.device("cpu")).numpy())


def test_batchnorm_fold_matches_reference_math():
    """The load-time BatchNorm fold (rewrites.fold_conv_batchnorm, FoldConvBatchNorm) and the oracle's
    own restatement give the same folded weights bit for bit, and the folded conv matches conv -> BN
    evaluated in fp64 on the oracle's reference conv."""
    import oracle as O
    from oracle.runner import OracleSession, fold_batchnorm
    from simdonnx_b200.rewrites import fold_conv_batchnorm
    plan = configs.build_c1(batch=1, hw=12, c=16, bn=True)
    ours, theirs = fold_conv_batchnorm(plan), fold_batchnorm(plan)
    cw = [n for n in ours.nodes if n.op == "Conv"][0]
    tw = [n for n in theirs.nodes if n.op == "Conv"][0]
    assert not any(n.op == "BatchNorm" for n in ours.nodes)
    assert np.array_equal(ours.values[cw.ins[1]].const, theirs.values[tw.ins[1]].const)
    assert np.array_equal(ours.values[cw.p.bias].const, theirs.values[tw.p.bias].const)
    feeds = {k: f() for k, f in plan.feeds.items()}
    got = OracleSession(plan).run(feeds)[plan.output]
    bn = [n for n in plan.nodes if n.op == "BatchNorm"][0].p
    V = lambda k: plan.values[k].const.astype(np.float64)
    conv = O.conv_ref64(feeds[plan.input], plan.values["c1.w"].const, None, pads=(1, 1, 1, 1)).astype(np.float64)
    want = (conv - V(bn.mean)) / np.sqrt(V(bn.var) + bn.eps) * V(bn.gamma) + V(bn.beta)
    want = np.maximum(want + feeds["c1.res"], 0)
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()


def test_unfoldable_batchnorm_lowers_to_the_affine_pair():
    """A BatchNorm after a pool (no conv to fold into) becomes x * s + t (EmitBatchNorm); the
    lowered plan computes the same values as the oracle's BatchNorm node, bit for bit."""
    from oracle.runner import OracleSession
    from simdonnx_b200.rewrites import fold_conv_batchnorm, lower_batchnorm
    plan = configs.build_fused_tail(batch=1, hw=32)
    low = lower_batchnorm(fold_conv_batchnorm(plan))
    ops = [n.op for n in low.nodes]
    assert "BatchNorm" not in ops and ops.count("Elementwise") == 3  # bn0 -> mul + add; the gain
    feeds = {k: f() for k, f in plan.feeds.items()}
    a = OracleSession(plan).run(feeds)[plan.output]
    b = OracleSession(low).run(feeds)[low.output]
    assert np.array_equal(a, b)
