"""ctypes binding of libsdxcuda.so (the C ABI declared in include/sdxcuda.h).

The library is built in-tree (``python -m simdonnx_b200.build``). Loading fails loudly when it is
missing: there is no CPU fallback for any op.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libsdxcuda.so")

SDX_OK = 0
STATUS = {0: "OK", 1: "INVALID", 2: "CUDA", 3: "OOM", 4: "TIMEOUT", 5: "DEVICE", 6: "INJECTED", 7: "POISONED",
          8: "NOT_SUPPORTED"}

ACT = {"none": 0, "relu": 1, "sigmoid": 2, "gelu": 3, "hardswish": 4, "swish": 5}
EW = {"add": 0, "sub": 1, "mul": 2, "div": 3}
F16, F32 = 0, 1
NHWC, NCHW = 0, 1

OP_CONV, OP_GEMM, OP_CONVT, OP_POOL, OP_CHANNEL_GATE, OP_CHANNEL_BROADCAST, OP_RESIZE_NEAREST = 1, 2, 3, 4, 5, 6, 7
OP_CONCAT, OP_BINARY, OP_ACT, OP_CONVERT, OP_LAYERNORM, OP_SOFTMAX, OP_ATTENTION = 8, 9, 10, 11, 12, 13, 14
OP_CONCAT_NEAREST = 15
OP_IMAGE = 16
OP_IMAGE_CONV = 17
OP_CONVT_CHAIN = 18
OP_BINARY_BCAST, OP_SAFE_DIV, OP_CHANNEL_SHIFT, OP_UPHEAD, OP_MATMUL, OP_GEMM_ARGMAX = 19, 20, 21, 22, 23, 24
OP_DW_PW = 25
BCAST_MAX_RANK = 6

FAULT_MALLOC, FAULT_LAUNCH, FAULT_GRAPH, FAULT_D2H, FAULT_SYNC = 1, 2, 3, 4, 5

_i, _i64, _u64, _f, _p, _sz = ctypes.c_int, ctypes.c_int64, ctypes.c_uint64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t


class ConvDesc(ctypes.Structure):
    _fields_ = [(n, _i) for n in ("batch", "ih", "iw", "ic", "oh", "ow", "oc", "kh", "kw", "sh", "sw", "pad_t",
                                  "pad_l", "pad_b", "pad_r", "group", "act", "pool", "pool_relu", "x_dtype",
                                  "x_layout", "y_dtype", "add_dtype", "add_layout", "y_layout", "pad_mode")] + [
        ("pad_value", _f), ("y_pix_stride", _i64), ("y_ch_off", _i),
        ("x", _u64), ("w", _u64), ("bias", _u64), ("add", _u64), ("y", _u64), ("in_scale", _u64), ("w_terms", _i),
        ("add_up", _i), ("gap_sums", _u64), ("w_scaled", _u64)]


class GemmDesc(ctypes.Structure):
    _fields_ = [("m", _i), ("k", _i), ("n", _i), ("lda", _i64), ("act", _i), ("y_dtype", _i), ("add_dtype", _i),
                ("ldy", _i64), ("ldadd", _i64), ("a", _u64), ("w", _u64), ("bias", _u64), ("add", _u64),
                ("y", _u64)]


class ConvtDesc(ctypes.Structure):
    _fields_ = [(n, _i) for n in ("batch", "ih", "iw", "ic", "oc", "kh", "kw", "act", "y_dtype")] + [
        ("x", _u64), ("w", _u64), ("bias", _u64), ("y", _u64)]


class PoolDesc(ctypes.Structure):
    _fields_ = [(n, _i) for n in ("batch", "ih", "iw", "c", "oh", "ow", "kh", "kw", "sh", "sw", "pad_t", "pad_l",
                                  "is_avg", "relu", "count_include_pad")] + [("x", _u64), ("y", _u64),
                                                                              ("x_pix_stride", _i64), ("x_ch_off", _i)]


class GateDesc(ctypes.Structure):
    _fields_ = [(n, _i) for n in ("batch", "hw", "c", "r", "act1_relu", "hard")] + [
        ("alpha", _f), ("beta", _f), ("offset", _f)] + [
        (n, _u64) for n in ("x", "w1", "b1", "w2", "b2", "s", "partial", "sums")]


class ResizeDesc(ctypes.Structure):
    _fields_ = [(n, _i) for n in ("batch", "ih", "iw", "c", "oh", "ow", "add_relu")] + [
        ("y_pix_stride", _i64), ("y_ch_off", _i), ("x", _u64), ("add", _u64), ("y", _u64)]


class MiscDesc(ctypes.Structure):
    _fields_ = [("n", _i64), ("rows", _i64), ("pixels", _i64)] + [
        (n, _i) for n in ("batch", "c", "t", "heads", "d", "op", "act", "relu", "x_dtype", "x_layout", "y_dtype",
                          "y_layout", "nin")] + [
        ("counts", _i * 8), ("eps", _f), ("scale", _f)] + [
        (n, _u64) for n in ("a", "b", "x", "y", "w", "bias")] + [("ins", _u64 * 8), ("aux", _i * 8)]


class ImageDesc(ctypes.Structure):
    _fields_ = [(n, _i) for n in ("batch", "ih", "iw", "bpp", "swap_rb", "oh", "ow", "pad_t", "pad_l", "y_nhwc_f16")] + [
        ("stride", _i64), ("image_bytes", _i64), ("src", _u64), ("lut", _u64), ("y", _u64)]


class ConvtChainDesc(ctypes.Structure):
    _fields_ = [("first", ConvtDesc)] + [(n, _i) for n in ("oc2", "kh2", "kw2", "act2", "y_dtype")] + [
        (n, _u64) for n in ("w2", "bias2", "y")]


class ImageConvDesc(ctypes.Structure):
    _fields_ = [("image", ImageDesc), ("conv", ConvDesc)]


class BcastDesc(ctypes.Structure):
    _fields_ = [("rank", _i), ("out_shape", _i64 * BCAST_MAX_RANK), ("a_shape", _i64 * BCAST_MAX_RANK),
                ("b_shape", _i64 * BCAST_MAX_RANK)] + [(n, _i) for n in ("op", "act", "a_dtype", "b_dtype", "y_dtype")] + [
        (n, _u64) for n in ("a", "b", "y")]


class SafeDivDesc(ctypes.Structure):
    _fields_ = [("n", _i64), ("eps", _f), ("lo", _f), ("hi", _f), ("dtype", _i)] + [(n, _u64) for n in ("a", "b", "y")]


class ShiftDesc(ctypes.Structure):
    _fields_ = [(n, _i) for n in ("batch", "h", "w", "c", "axis", "ngroups")] + [
        ("group_ends", _i * 8), ("offsets", _i * 8), ("dtype", _i), ("x", _u64), ("y", _u64)]


class UpHeadDesc(ctypes.Structure):
    _fields_ = [(n, _i) for n in ("batch", "ih", "iw", "c", "oh", "ow", "oc")] + [("scale_h", _f), ("scale_w", _f)] + [
        (n, _i) for n in ("resize_relu", "skip_relu", "act", "x_dtype", "skip_dtype", "y_dtype")] + [
        (n, _u64) for n in ("x", "skip", "w", "bias", "y")]


class MatMulDesc(ctypes.Structure):
    _fields_ = [("rank", _i), ("a_shape", _i64 * BCAST_MAX_RANK), ("b_shape", _i64 * BCAST_MAX_RANK)] + [
        (n, _i) for n in ("a_dtype", "b_dtype", "y_dtype")] + [(n, _u64) for n in ("a", "b", "y")]


class GemmArgmaxDesc(ctypes.Structure):
    _fields_ = [("gemm", GemmDesc), ("indices", _u64), ("probs", _u64), ("scratch", _u64)]


class DwPwDesc(ctypes.Structure):
    _fields_ = [("dw", ConvDesc), ("pw", ConvDesc)]


DESC_OF_OP = {OP_CONV: ConvDesc, OP_GEMM: GemmDesc, OP_CONVT: ConvtDesc, OP_POOL: PoolDesc,
              OP_CHANNEL_GATE: GateDesc, OP_RESIZE_NEAREST: ResizeDesc, OP_CHANNEL_BROADCAST: MiscDesc,
              OP_CONCAT: MiscDesc, OP_BINARY: MiscDesc, OP_ACT: MiscDesc, OP_CONVERT: MiscDesc,
              OP_LAYERNORM: MiscDesc, OP_SOFTMAX: MiscDesc, OP_ATTENTION: MiscDesc, OP_CONCAT_NEAREST: MiscDesc,
              OP_IMAGE: ImageDesc, OP_IMAGE_CONV: ImageConvDesc, OP_CONVT_CHAIN: ConvtChainDesc,
              OP_BINARY_BCAST: BcastDesc, OP_SAFE_DIV: SafeDivDesc, OP_CHANNEL_SHIFT: ShiftDesc, OP_UPHEAD: UpHeadDesc,
              OP_MATMUL: MatMulDesc, OP_GEMM_ARGMAX: GemmArgmaxDesc, OP_DW_PW: DwPwDesc}

_SIGS = {
    "sdx_abi_version": (_i, []),
    "sdx_last_error": (_i, [ctypes.c_char_p, _i]),
    "sdx_device_count": (_i, [ctypes.POINTER(_i)]),
    "sdx_open": (_i, [_i, ctypes.POINTER(_p)]),
    "sdx_close": (_i, [_p]),
    "sdx_ctx_stream": (_i, [_p, ctypes.POINTER(_p)]),
    "sdx_device_info": (_i, [_p, ctypes.c_char_p, _i, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i),
                             ctypes.POINTER(_sz)]),
    "sdx_malloc": (_i, [_p, _sz, ctypes.POINTER(_u64)]),
    "sdx_free": (_i, [_p, _u64]),
    "sdx_host_alloc_pinned": (_i, [_sz, ctypes.POINTER(_p)]),
    "sdx_host_free": (_i, [_p]),
    "sdx_memcpy_htod_async": (_i, [_p, _u64, _p, _sz, _p]),
    "sdx_memcpy_dtoh_async": (_i, [_p, _p, _u64, _sz, _p]),
    "sdx_memcpy_dtod_async": (_i, [_p, _u64, _u64, _sz, _p]),
    "sdx_memset_async": (_i, [_p, _u64, _i, _sz, _p]),
    "sdx_stream_create": (_i, [_p, ctypes.POINTER(_p)]),
    "sdx_stream_destroy": (_i, [_p, _p]),
    "sdx_stream_sync": (_i, [_p, _p, _i]),
    "sdx_stream_query": (_i, [_p, _p, ctypes.POINTER(_i)]),
    "sdx_event_create": (_i, [_p, ctypes.POINTER(_p)]),
    "sdx_event_record": (_i, [_p, _p, _p]),
    "sdx_event_elapsed_ms": (_i, [_p, _p, ctypes.POINTER(_f)]),
    "sdx_event_destroy": (_i, [_p]),
    "sdx_graph_begin": (_i, [_p, _p]),
    "sdx_graph_end": (_i, [_p, _p, ctypes.POINTER(_p)]),
    "sdx_graph_launch": (_i, [_p, _p, _p]),
    "sdx_graph_destroy": (_i, [_p]),
    "sdx_device_error": (_i, [_p, ctypes.POINTER(ctypes.c_uint)]),
    "sdx_clear_device_error": (_i, [_p]),
    "sdx_fault_inject": (_i, [_i, _i]),
    "sdx_launch_count": (_u64, []),
    "sdx_selftest_bounded_wait": (_i, [_p, _i, _p]),
    "sdx_pack_conv": (_i, [ctypes.POINTER(ConvDesc), _p, _p, ctypes.POINTER(_sz)]),
    "sdx_pack_convt": (_i, [_i, _i, _i, _i, _p, _p, ctypes.POINTER(_sz)]),
    "sdx_conv_scaled_weights_bytes": (_sz, [ctypes.POINTER(ConvDesc)]),
    "sdx_pack_gemm": (_i, [_i, _i, _i, _p, _p, ctypes.POINTER(_sz)]),
    "sdx_conv2d": (_i, [_p, ctypes.POINTER(ConvDesc), _p]),
    "sdx_gemm": (_i, [_p, ctypes.POINTER(GemmDesc), _p]),
    "sdx_convt": (_i, [_p, ctypes.POINTER(ConvtDesc), _p]),
    "sdx_pool": (_i, [_p, ctypes.POINTER(PoolDesc), _p]),
    "sdx_channel_gate_scratch_bytes": (_sz, [_i, _i, _i]),
    "sdx_channel_gate": (_i, [_p, ctypes.POINTER(GateDesc), _p]),
    "sdx_channel_gate_static": (_i, [_p, ctypes.POINTER(GateDesc), _p]),
    "sdx_channel_broadcast": (_i, [_p, _i, _i64, _i, _i, _i, _u64, _u64, _u64, _p]),
    "sdx_resize_nearest": (_i, [_p, ctypes.POINTER(ResizeDesc), _p]),
    "sdx_concat_channels": (_i, [_p, _i64, _i, ctypes.POINTER(_i), ctypes.POINTER(_u64), _u64, _p]),
    "sdx_image_to_tensor": (_i, [_p, ctypes.POINTER(ImageDesc), _p]),
    "sdx_image_conv": (_i, [_p, ctypes.POINTER(ImageConvDesc), _p]),
    "sdx_convt_chain": (_i, [_p, ctypes.POINTER(ConvtChainDesc), _p]),
    "sdx_concat_nearest": (_i, [_p, _i, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_u64), _u64,
                                _p]),
    "sdx_binary": (_i, [_p, _i64, _i, _i, _u64, _u64, _u64, _p]),
    "sdx_act": (_i, [_p, _i64, _i, _u64, _u64, _p]),
    "sdx_convert": (_i, [_p, _i, _i, _i64, _i, _i, _i, _i, _u64, _u64, _p]),
    "sdx_convert_pad": (_i, [_p, _i, _i, _i, _i64, _i, _i, _i, _i, _u64, _u64, _p]),
    "sdx_layernorm": (_i, [_p, _i64, _i, _f, _u64, _u64, _u64, _u64, _p]),
    "sdx_softmax": (_i, [_p, _i64, _i, _i, _u64, _u64, _p]),
    "sdx_attention": (_i, [_p, _i, _i, _i, _i, _f, _u64, _u64, _p]),
    "sdx_binary_bcast": (_i, [_p, ctypes.POINTER(BcastDesc), _p]),
    "sdx_safe_div": (_i, [_p, ctypes.POINTER(SafeDivDesc), _p]),
    "sdx_channel_shift": (_i, [_p, ctypes.POINTER(ShiftDesc), _p]),
    "sdx_uphead": (_i, [_p, ctypes.POINTER(UpHeadDesc), _p]),
    "sdx_matmul": (_i, [_p, ctypes.POINTER(MatMulDesc), _p]),
    "sdx_gemm_argmax_scratch_bytes": (_sz, [_i, _i]),
    "sdx_gemm_argmax": (_i, [_p, ctypes.POINTER(GemmArgmaxDesc), _p]),
    "sdx_dw_pw_supported": (_i, [ctypes.POINTER(DwPwDesc)]),
    "sdx_dw_pw": (_i, [_p, ctypes.POINTER(DwPwDesc), _p]),
    "sdx_desc_size": (_sz, [_i]),
    "sdx_session_create": (_i, [_p, _sz, ctypes.POINTER(_p)]),
    "sdx_session_arena": (_i, [_p, ctypes.POINTER(_u64), ctypes.POINTER(_sz)]),
    "sdx_session_add_node": (_i, [_p, _i, _p, _sz]),
    "sdx_session_set_io": (_i, [_p, _u64, _sz, _u64, _sz]),
    "sdx_session_build": (_i, [_p, _i]),
    "sdx_session_stream": (_i, [_p, ctypes.POINTER(_p)]),
    "sdx_session_enqueue": (_i, [_p]),
    "sdx_session_submit": (_i, [_p, _p, _p]),
    "sdx_session_wait": (_i, [_p, _i]),
    "sdx_session_run": (_i, [_p, _p, _p, _i]),
    "sdx_session_node_count": (_i, [_p, ctypes.POINTER(_i)]),
    "sdx_session_enqueue_node": (_i, [_p, _i]),
    "sdx_session_destroy": (_i, [_p]),
}

EXPORTS = tuple(_SIGS)

_lib = None


class SdxError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"sdx {STATUS.get(code, code)}: {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    """The loaded libsdxcuda (raises when the in-tree build is missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libsdxcuda.so is not built ({LIB_PATH}); run python -m simdonnx_b200.build")
        so = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(so, name)
            fn.restype = res
            fn.argtypes = args
        _lib = so
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().sdx_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != SDX_OK:
        raise SdxError(rc, last_error())


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
