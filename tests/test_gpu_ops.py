"""The remaining node kinds and the reference's built-in fused ops on the GPU, against the oracle.

Covers elementwise binary (same shape and numpy broadcast, Ops.Elementwise src/Kernels/Ops.cs:388-441),
standalone activations (Act.Apply, src/Kernels/Act.cs:70-117), SafeDiv / ChannelShift / UpHead
(src/Engine/Fusions/*.cs, FusedKernels src/Kernels/FusedKernels.cs), batched MatMul of two
activations (Ops.MatMul, src/Kernels/Ops.Seq.cs:90-113), the fused CTC projection + argmax
(CtcProjection.ArgMax, src/Decoding/CtcProjection.cs:47-55) and conv + fused 2x2 max pool on the
small-stem kernel (Nhwc.ConvPool, src/Kernels/Nhwc.cs:666-727).

Tolerance: rel-L2 <= 2e-3, max-abs <= 1e-2 * max|ref| (tests/parity.py); inputs are rounded to
fp16 first where the kernel stores fp16, so the comparison measures the kernel, not the storage.
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


def f16(a):
    """fp16-representable fp32 copy (what the fp16 tensor on the device holds)."""
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def dev(a, dtype=torch.float16):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda().to(dtype)


def host(t):
    torch.cuda.synchronize()
    return t.float().cpu().numpy()


@pytest.mark.parametrize("kind", ["none", "relu", "sigmoid", "gelu", "hardswish", "swish"])
def test_act_node(be, kind):
    from simdonnx_b200 import backend as B
    x = f16(np.random.default_rng(3).uniform(-6, 6, (2, 37, 41, 24)))
    y = B.act(be, dev(x), kind)
    assert_close(host(y), O.act(x, kind), f"act {kind}")


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
@pytest.mark.parametrize("relu", [False, True])
def test_binary_same_shape(be, op, relu):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(11)
    a = f16(rng.uniform(-2, 2, (3, 17, 19, 16)))
    b = f16(rng.uniform(0.5, 2, (3, 17, 19, 16)) * rng.choice([-1, 1], (3, 17, 19, 16)))
    y = B.binary(be, dev(a), dev(b), op, relu)
    assert_close(host(y), O.binary(a, b, op, relu), f"binary {op}")


BCAST_CASES = [
    # a shape, b shape, op, act, b fp32
    ((2, 5, 7, 16), (16,), "add", "none", True),          # bias vector
    ((2, 5, 7, 16), (2, 1, 1, 16), "mul", "none", True),  # SE gate [N, 1, 1, C]
    ((2, 1, 7, 16), (1, 5, 1, 1), "sub", "relu", False),  # both broadcast
    ((4, 3, 8), (3, 1), "div", "gelu", False),
    ((1,), (3, 4, 5), "mul", "sigmoid", False),            # scalar times a tensor
    ((6, 1, 2, 3, 4, 5), (1, 7, 2, 1, 4, 1), "add", "hardswish", True),  # rank 6
]


@pytest.mark.parametrize("ashape,bshape,op,act,b32", BCAST_CASES)
def test_binary_broadcast(be, ashape, bshape, op, act, b32):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(len(ashape) * 10 + len(bshape))
    a = f16(rng.uniform(-2, 2, ashape))
    b = rng.uniform(0.5, 2, bshape).astype(np.float32)
    if not b32:
        b = f16(b)
    y = B.binary_bcast(be, dev(a), dev(b, torch.float32 if b32 else torch.float16), op, act)
    assert y.shape == np.broadcast_shapes(ashape, bshape)
    assert_close(host(y), O.binary_bcast(a, b, op, act), f"broadcast {op} {ashape} {bshape}")


def test_binary_broadcast_rejects_mismatch(be):
    from simdonnx_b200 import _native as N
    import ctypes
    d = N.BcastDesc()
    d.rank = 2
    d.out_shape[0], d.out_shape[1] = 4, 5
    d.a_shape[0], d.a_shape[1] = 4, 5
    d.b_shape[0], d.b_shape[1] = 3, 5  # 3 does not broadcast to 4
    d.a = d.b = d.y = 1 << 20  # never dereferenced: rejected before any launch
    before = int(N.lib().sdx_launch_count())
    assert N.lib().sdx_binary_bcast(be.ctx, ctypes.byref(d), None) == 1
    assert int(N.lib().sdx_launch_count()) == before


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("n", [4096, 1001])
def test_safe_div(be, dtype, n):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(n)
    a = f16(rng.uniform(-3, 3, n))
    b = f16(rng.uniform(-0.01, 1, n))  # many b below eps: the floor applies
    y = B.safe_div(be, dev(a, dtype), dev(b, dtype), 0.05, -4.0, 4.0)
    assert_close(host(y), O.safe_div(a, b, 0.05, -4.0, 4.0), "safediv")


@pytest.mark.parametrize("axis,c,ends,offs,dtype", [
    (2, 40, [8, 16, 24, 32], [2, 1, -1, -2], torch.float16),      # 16-byte path, tail channels copied
    (3, 40, [8, 16, 24, 32, 40], [-2, -1, 0, 1, 2], torch.float16),
    (3, 20, [4, 8, 12, 16, 20], [3, -3, 0, 9, -9], torch.float32),  # per-element path, shifts past the edge
])
def test_channel_shift(be, axis, c, ends, offs, dtype):
    from simdonnx_b200 import backend as B
    x = f16(np.random.default_rng(c).uniform(-1, 1, (2, 9, 7, c)))
    y = B.channel_shift(be, dev(x, dtype), axis, ends, offs)
    np.testing.assert_array_equal(host(y), O.channel_shift(x, axis, ends, offs))  # a pure copy: bit-exact


@pytest.mark.parametrize("c,oc,ih,iw,scale,rr,sr,act", [
    (32, 1, 20, 24, 2.0, False, False, "sigmoid"),
    (64, 4, 10, 12, 4.0, True, False, "relu"),
    (128, 8, 16, 16, 2.0, False, True, "none"),
    (8, 3, 7, 9, 2.0, True, True, "sigmoid"),
])
def test_uphead(be, c, oc, ih, iw, scale, rr, sr, act):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(c + oc)
    x = f16(rng.uniform(-1, 1, (2, ih, iw, c)))
    oh, ow = int(ih * scale), int(iw * scale)
    skip = f16(rng.uniform(-1, 1, (2, oh, ow, c)))
    w = rng.uniform(-1, 1, (oc, c)).astype(np.float32) / np.sqrt(c)
    bias = rng.uniform(-0.1, 0.1, oc).astype(np.float32)
    ref = O.uphead(x, skip, w, bias, scale, scale, rr, sr, act)
    y = B.uphead(be, dev(x), dev(skip), dev(w, torch.float32), dev(bias, torch.float32), scale, scale, rr, sr, act,
                 y_dtype=torch.float32)
    assert_close(host(y), ref, f"uphead c{c} oc{oc}")


@pytest.mark.parametrize("ashape,bshape", [((2, 8, 40, 15), (2, 8, 15, 40)), ((3, 1, 33, 70), (4, 70, 19)),
                                           ((64, 96), (96, 50))])
def test_matmul_activations(be, ashape, bshape):
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(ashape[-1])
    a, b = f16(rng.uniform(-1, 1, ashape)), f16(rng.uniform(-1, 1, bshape))
    y = B.matmul(be, dev(a), dev(b), y_dtype=torch.float32)
    assert_close(host(y), O.matmul_bcast(a, b), f"matmul {ashape} x {bshape}")


@pytest.mark.parametrize("m,k,n", [(64 * 40, 120, 6625), (5 * 40, 120, 1000), (37, 64, 300)])
def test_ctc_head_fused_argmax(be, m, k, n):
    """C3's CTC head: per row the first maximum's index and its softmax probability, logits never
    stored; against the oracle's projection (Gemm) and UpdateArgMax walk. Indices are compared where
    the top-2 logit margin exceeds the GPU's logit error (fp16 A is exact here; the weights are two
    fp16 terms, ~22 bits)."""
    from simdonnx_b200 import backend as B
    rng = np.random.default_rng(m + n)
    a = f16(rng.normal(0, 1, (m, k)))
    w = rng.normal(0, 0.3, (k, n)).astype(np.float32)
    bias = rng.normal(0, 0.1, n).astype(np.float32)
    logits = O.gemm(a, O.GemmPlan(w, bias))
    ref_i, ref_p = O.ctc_argmax(logits)
    idx, prob = B.gemm_argmax(be, dev(a), B.pack_gemm(w), n, bias=dev(bias, torch.float32))
    got_i, got_p = host(idx).astype(np.int64), host(prob)
    top2 = np.sort(logits, axis=1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 1e-3 * np.abs(logits).max()
    assert clear.mean() > 0.9
    np.testing.assert_array_equal(got_i[clear], ref_i[clear])
    assert_close(got_p, ref_p, "ctc probabilities")
    assert be.device_error() == 0


@pytest.mark.parametrize("ic,oc,act,pool_relu,nchw", [(3, 16, "relu", False, True), (3, 32, "none", True, False),
                                                      (4, 8, "relu", True, False), (1, 16, "none", False, True)])
def test_conv_pool_fused_stem(be, ic, oc, act, pool_relu, nchw):
    """A small stem conv (ic < 8, 3x3 s1) with the 2x2/2 max pool in its epilogue: the pooled tensor
    is written directly (odd conv sizes drop the last row / column)."""
    from simdonnx_b200 import _native as N, backend as B
    rng = np.random.default_rng(ic * 10 + oc)
    nb, h, w = 2, 33, 26
    x = rng.uniform(0, 1, (nb, h, w, ic)).astype(np.float32)
    wt = rng.uniform(-1, 1, (oc, ic, 3, 3)).astype(np.float32) / 3
    b = rng.uniform(-0.2, 0.2, oc).astype(np.float32)
    ref = O.conv_pool(x, O.ConvPlan(wt, b), pads=(1, 1, 1, 1), act=act, pool_relu=pool_relu)
    xin = np.ascontiguousarray(x.transpose(0, 3, 1, 2)) if nchw else x
    d = B.conv_desc(nb, h, w, ic, oc, 3, 3, pads=(1, 1, 1, 1), act=act, pool=True, pool_relu=pool_relu,
                    x_dtype=torch.float32, x_layout=N.NCHW if nchw else N.NHWC)
    y = B.conv2d(be, d, dev(xin, torch.float32), B.pack_conv(d, wt), bias=dev(b, torch.float32))
    assert y.shape == (nb, h // 2, w // 2, oc)
    assert_close(host(y), ref, f"conv+pool {ic}->{oc}")
