"""One process, several contexts: the per-device state of the launchers.

A kernel's dynamic shared-memory limit (cudaFuncSetAttribute) belongs to the device that was
current when it was raised. The C ABI allows one context per device in one process, used from
different host threads (include/sdxcuda.h), so every launcher keeps that state per device and
thread-safe. These tests run the kernels that need more than 48 KB of shared memory (tensor-core
conv, tensor-core stem, sliding depthwise, gate FC) from two threads on device 0 and, when a
second GPU is visible, on device 1 in the same process; the results must be bit-identical to a
single-threaded run on device 0.
"""
import ctypes
import threading

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


class _Ctx:
    """A private sdx context (not the cached CudaBackend) for one thread or device."""

    def __init__(self, ordinal):
        from simdonnx_b200 import _native as N
        self.ordinal = ordinal
        h = ctypes.c_void_p()
        N.call("sdx_open", ordinal, ctypes.byref(h))
        self.ctx = h

    def close(self):
        from simdonnx_b200 import _native as N
        N.lib().sdx_close(self.ctx)


def _workload(ctx, device):
    """Runs the big-shared-memory kernels on `device` through context `ctx`; host results."""
    from simdonnx_b200 import backend as B, _native as N
    rng = np.random.default_rng(3)
    dev = torch.device("cuda", device)
    out = []
    with torch.cuda.device(device):
        st = torch.cuda.Stream(device=dev)
        with torch.cuda.stream(st):
            # sliding-window depthwise 5x5 (dw_slide, 120 KB smem)
            x = torch.from_numpy(rng.uniform(-1, 1, (2, 40, 40, 256)).astype(np.float32)).to(dev).half()
            d = B.conv_desc(2, 40, 40, 256, 256, 5, 5, pads=(2, 2, 2, 2), group=256, act="hardswish")
            w = rng.uniform(-0.2, 0.2, (256, 1, 5, 5)).astype(np.float32)
            out.append(B.conv2d(ctx, d, x, B.pack_conv(d, w, dev), bias=torch.zeros(256, device=dev)))
            # tensor-core pointwise conv (conv_tc, 227 KB limit)
            d = B.conv_desc(2, 40, 40, 256, 128, 1, 1, act="relu")
            w = rng.uniform(-0.1, 0.1, (128, 256, 1, 1)).astype(np.float32)
            out.append(B.conv2d(ctx, d, x, B.pack_conv(d, w, dev), bias=torch.zeros(128, device=dev)))
            # tensor-core stem from fp32 NCHW (stem_tc)
            xs = torch.from_numpy(rng.uniform(0, 1, (2, 3, 128, 128)).astype(np.float32)).to(dev)
            d = B.conv_desc(2, 128, 128, 3, 16, 3, 3, stride=(2, 2), pads=(1, 1, 1, 1), act="hardswish",
                            x_dtype=torch.float32, x_layout=N.NCHW)
            w = rng.uniform(-0.3, 0.3, (16, 3, 3, 3)).astype(np.float32)
            out.append(B.conv2d(ctx, d, xs, B.pack_conv(d, w, dev), bias=torch.zeros(16, device=dev)))
            # SE gate from the tensor (gap_partial + gate FC kernels, 160 KB limit)
            w1 = torch.from_numpy(rng.uniform(-0.1, 0.1, (64, 256)).astype(np.float32)).to(dev)
            w2 = torch.from_numpy(rng.uniform(-0.1, 0.1, (256, 64)).astype(np.float32)).to(dev)
            out.append(B.channel_gate(ctx, x, w1, torch.zeros(64, device=dev), w2, torch.zeros(256, device=dev)))
        st.synchronize()
    return [t.float().cpu().numpy() for t in out]


def test_two_threads_two_contexts_device0():
    base = _Ctx(0)
    want = _workload(base, 0)
    base.close()
    results, errors = {}, []

    def worker(i):
        c = _Ctx(0)
        try:
            results[i] = _workload(c, 0)
        except Exception as e:  # reported below, on the test's thread
            errors.append(e)
        finally:
            c.close()

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(120)
    assert not errors, errors
    for i in range(2):
        for k, (g, w) in enumerate(zip(results[i], want)):
            assert np.array_equal(g, w), f"thread {i}, op {k}"


def test_second_device_same_process():
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU visible")
    c0, c1 = _Ctx(0), _Ctx(1)
    want = _workload(c0, 0)  # raises every limit on device 0 first
    got = _workload(c1, 1)
    c0.close()
    c1.close()
    for k, (g, w) in enumerate(zip(got, want)):
        assert np.array_equal(g, w), f"op {k} differs on device 1"
