"""sdx_channel_gate_static: the SE gate with library-owned fixed scratch (no allocation in the call).

Called straight through the C ABI and compared with sdx_channel_gate (caller-provided scratch) on
the same inputs, twice in a row (the second call reuses the fixed array the first one left
behind). The file name sorts last so it also runs after every other GPU test in one session.
"""
import ctypes

import numpy as np
import pytest

from simdonnx_b200 import _native as N

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_BYTES = 4 * 1024 * 1024  # SDX_GATE_STATIC_MAX_SCRATCH_BYTES in include/sdxcuda.h


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    h = ctypes.c_void_p()
    N.call("sdx_open", 0, ctypes.byref(h))
    yield h
    N.lib().sdx_close(h)


def _ptr(t):
    return t.data_ptr() if t is not None else 0


def _desc(x, w1, b1, w2, b2, s, partial=None):
    b, h, w, c = x.shape
    d = N.GateDesc()
    d.batch, d.hw, d.c, d.r, d.act1_relu, d.hard = b, h * w, c, w1.shape[0], 1, 1
    d.alpha, d.beta, d.offset = 0.2, 0.5, 0.0
    d.x, d.w1, d.b1, d.w2, d.b2, d.s = _ptr(x), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2), _ptr(s)
    d.partial = _ptr(partial)
    return d


def _inputs(seed, b, hw, c):
    g = torch.Generator().manual_seed(seed)
    r = max(8, c // 4)
    x = (torch.rand((b, hw, hw, c), generator=g) * 2 - 1).half().cuda()
    w1 = (torch.rand((r, c), generator=g) * 2 - 1).cuda()
    b1 = (torch.rand((r,), generator=g) * 2 - 1).cuda()
    w2 = (torch.rand((c, r), generator=g) * 2 - 1).cuda()
    b2 = (torch.rand((c,), generator=g) * 2 - 1).cuda()
    return x, w1, b1, w2, b2


def _run(ctx, fn, d, stream):
    """Calls `fn` on the context's own stream (stream None) or on a torch stream, then waits."""
    torch.cuda.synchronize()  # inputs were written on torch's default stream
    if stream is None:
        N.call(fn, ctx, ctypes.byref(d), None)
        N.call("sdx_stream_sync", ctx, None, 10000)
    else:
        N.call(fn, ctx, ctypes.byref(d), ctypes.c_void_p(stream.cuda_stream))
        stream.synchronize()


def _gate_with_scratch(ctx, args, sums=None, stream=None):
    x = args[0]
    b, h, w, c = x.shape
    s = torch.empty((b, c), dtype=torch.float32, device="cuda")
    scratch = torch.empty(int(N.lib().sdx_channel_gate_scratch_bytes(b, h * w, c)), dtype=torch.uint8, device="cuda")
    d = _desc(*args, s, scratch)
    d.sums = _ptr(sums)
    _run(ctx, "sdx_channel_gate", d, stream)
    return s.cpu().numpy()


def _gate_static(ctx, args, sums=None, stream=None):
    x = args[0]
    s = torch.full((x.shape[0], x.shape[-1]), float("nan"), dtype=torch.float32, device="cuda")
    d = _desc(*args, s)
    d.sums = _ptr(sums)
    _run(ctx, "sdx_channel_gate_static", d, stream)
    return s.cpu().numpy()


@pytest.mark.parametrize("b,hw,c", [(3, 80, 32), (2, 20, 512), (4, 160, 64)])
def test_static_gate_matches_scratch_gate_twice(ctx, b, hw, c):
    first = _inputs(b * 1000 + c, b, hw, c)
    second = _inputs(b * 1000 + c + 1, b, hw, c)
    for args in (first, second, first):
        ref = _gate_with_scratch(ctx, args)
        for _ in range(2):
            got = _gate_static(ctx, args)
            assert np.isfinite(got).all()
            np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)


def test_static_gate_rejects_oversized_scratch(ctx):
    # c = 4096 with 64 pixel chunks per image needs over 1 MiB per image: 5 images exceed 4 MiB
    need = int(N.lib().sdx_channel_gate_scratch_bytes(5, 512 * 512, 4096))
    assert need > MAX_BYTES
    s = torch.empty((5, 4096), dtype=torch.float32, device="cuda")
    d = N.GateDesc()
    d.batch, d.hw, d.c, d.r, d.act1_relu, d.hard = 5, 512 * 512, 4096, 8, 1, 1
    d.x, d.s = 1 << 20, _ptr(s)  # never dereferenced: the call must fail before any launch
    before = int(N.lib().sdx_launch_count())
    rc = N.lib().sdx_channel_gate_static(ctx, ctypes.byref(d), None)
    assert rc == 8, rc  # SDX_ERR_NOT_SUPPORTED
    assert "scratch" in N.last_error()
    assert int(N.lib().sdx_launch_count()) == before


def test_static_gate_from_conv_sums_wide(ctx):
    """The scratch array on the other path: a gate that reads a conv's fp32 32-pixel channel sums
    with c = 4096 (above 2048 channels those sums are reduced per chunk into the scratch array)."""
    b, hw, c = 2, 16, 4096  # 16 x 16 pixels: 8 runs of 32 per image
    args = _inputs(77, b, hw, c)
    x = args[0]
    sums = x.float().reshape(b, hw * hw // 32, 32, c).sum(dim=2).contiguous()
    assert int(N.lib().sdx_channel_gate_scratch_bytes(b, hw * hw, c)) <= MAX_BYTES
    ref = _gate_with_scratch(ctx, args, sums)
    for _ in range(2):
        got = _gate_static(ctx, args, sums)
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)


def test_static_gate_on_caller_stream(ctx):
    """Both gates enqueued on a torch stream handle passed through the C ABI (not the context's own)."""
    args = _inputs(5, 3, 40, 128)
    st = torch.cuda.Stream()
    ref = _gate_with_scratch(ctx, args, stream=st)
    for _ in range(2):
        got = _gate_static(ctx, args, stream=st)
        np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)
