"""The C-ABI library loads without a GPU and exports every function include/sdxcuda.h declares;
descriptor structs agree in size between C and the ctypes mirror."""
import ctypes
import os
import re

from simdonnx_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "sdxcuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sdx_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = N.lib()
    missing = [f for f in declared_functions() if not hasattr(lib, f)]
    assert not missing, missing
    assert set(declared_functions()) == set(N.EXPORTS)
    assert lib.sdx_abi_version() == 1


def test_descriptor_sizes_match_c():
    for kind, desc in N.DESC_OF_OP.items():
        assert N.lib().sdx_desc_size(kind) == ctypes.sizeof(desc), kind
    assert N.lib().sdx_desc_size(999) == 0


def test_no_device_is_reported_cleanly():
    n = ctypes.c_int(-1)
    N.call("sdx_device_count", ctypes.byref(n))
    assert n.value >= 0
    if n.value == 0:
        h = ctypes.c_void_p()
        rc = N.lib().sdx_open(0, ctypes.byref(h))
        assert rc == 1 and "not present" in N.last_error()


def test_fault_injection_is_host_side():
    # an injected allocation fault fails the call before any CUDA work, with its own status
    N.call("sdx_fault_inject", N.FAULT_MALLOC, 1)
    p = ctypes.c_void_p()
    rc = N.lib().sdx_host_alloc_pinned(64, ctypes.byref(p))
    assert rc == 6 and "injected" in N.last_error()
    N.call("sdx_fault_inject", 0, 0)


def test_pack_sizes_cpu():
    # packing is host code: sizes follow the tile plan (N padded to 16, K to the channel block)
    from simdonnx_b200 import backend as B
    import torch
    d = B.conv_desc(1, 8, 8, 64, 64, 3, 3, pads=(1, 1, 1, 1))
    nb = ctypes.c_size_t()
    N.call("sdx_pack_conv", ctypes.byref(d), None, None, ctypes.byref(nb))
    assert nb.value == 9 * 64 * 64 * 2  # k x k kernels default to one fp16 weight term
    d.w_terms = 2
    N.call("sdx_pack_conv", ctypes.byref(d), None, None, ctypes.byref(nb))
    assert nb.value == 2 * 9 * 64 * 64 * 2  # hi + lo fp16 terms
    d = B.conv_desc(1, 8, 8, 96, 24, 1, 1)
    N.call("sdx_pack_conv", ctypes.byref(d), None, None, ctypes.byref(nb))
    assert nb.value == 2 * 32 * 96 * 2  # 1x1: two terms; 96 channels: 32-channel blocks, no K padding
    d.w_terms = 3
    assert N.lib().sdx_pack_conv(ctypes.byref(d), None, None, ctypes.byref(nb)) == 1
    d = B.conv_desc(1, 8, 8, 3, 16, 3, 3, stride=(2, 2), pads=(1, 1, 1, 1), x_dtype=torch.float32, x_layout=1)
    N.call("sdx_pack_conv", ctypes.byref(d), None, None, ctypes.byref(nb))
    assert nb.value == 9 * 3 * 16 * 4
    d.pad_mode = 1
    assert N.lib().sdx_pack_conv(ctypes.byref(d), None, None, ctypes.byref(nb)) == 8
