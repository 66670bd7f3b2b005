"""CudaGraphModel / CudaInferenceSession: lower an ExecPlan onto libsdxcuda and run it.

The reference's Vulkan backend is the template (VkGraphModel, src/Backends/Vulkan/VkGraph.cs:44-155,
:472-1112; VkInferenceSession, src/Backends/Vulkan/VkSession.cs:63-143, :282-337, :535-556):
  * backend-side rewrites that change no numerics class (cuda_rewrite): fp32 -> fp16 boundary
    conversion where a tensor-core conv reads a graph input; the squeeze-excitation product x*s
    folded into the load of the depthwise convs that consume it; a channel Concat of
    nearest-upsampled tensors becomes one ConcatNearest node that writes whole output pixels;
    producers of any other channel Concat write straight into their slice of its output; the image
    session's u8 -> fp32 normalisation is fused into the stem conv that reads it (ImageConv);
  * one device arena (int64 byte offsets, plan.plan_arena) + a per-model const store of packed
    weights; every node becomes one sdx_* descriptor over device pointers arena + offset;
  * the node list is validated once eagerly and captured into one CUDA graph.
"""
from __future__ import annotations

import copy
import ctypes

import numpy as np
import torch

from . import _native as N
from . import backend as B
from .plan import ExecPlan, Node, conv_out
from .rewrites import fold_conv_batchnorm, lower_batchnorm

_DT = {"f16": N.F16, "f32": N.F32}
_NP = {"f16": np.float16, "f32": np.float32, "i32": np.int32, "u8": np.uint8}
_LAY = {"nhwc": N.NHWC, "nchw": N.NCHW, "raw": N.NHWC}


def _nhwc_shape(v):
    s = v.shape
    return (s[0], s[2], s[3], s[1]) if v.layout == "nchw" else s


def _small_stem_pool(P: ExecPlan, n) -> bool:
    """Conv + 2x2/2 max pool that the fused small-stem kernel takes (GraphCompiler.GpuSmallConv,
    src/Engine/GraphCompiler.cs:28-32, with the pool fused only for such convs, :897-898)."""
    xv = P.values[n.ins[0]]
    ic = _nhwc_shape(xv)[3]
    W = P.values[n.ins[1]].const
    oc = W.shape[0]
    return (n.p.group == 1 and ic < 8 and oc % 8 == 0 and oc <= 128 and oc * ic * W.shape[2] * W.shape[3] <= 4096 and
            tuple(n.p.strides) == (1, 1) and not n.p.add and P.values[n.outs[0]].layout == "nhwc")


# The fused depthwise -> pointwise node (sdx_dw_pw) in the session rewrite: measured slower on B200
# than the two separate kernels for the det shapes (its depthwise warps cannot keep the pointwise
# epilogue fed), so the rewrite leaves the pairs unfused; sdx_dw_pw stays available and tested.
DW_PW_FUSION = False


def cuda_rewrite(plan: ExecPlan) -> ExecPlan:
    # the reference's load-time BatchNorm rewrites come first (FoldConvBatchNorm, EmitBatchNorm)
    plan = lower_batchnorm(fold_conv_batchnorm(plan))
    P = copy.copy(plan)
    P.values = {k: copy.copy(v) for k, v in plan.values.items()}
    P.nodes = [Node(n.op, list(n.ins), list(n.outs), copy.copy(n.p), n.name) for n in plan.nodes]
    P.inputs = list(plan.inputs or [plan.input])

    # 0. conv + fused 2x2/2 max pool (ConvP.Pool, src/Engine/ExecPlan.cs:63-64) -> conv into an arena
    #    value, then MaxPool (+relu): max of fp16-rounded values == fp16 rounding of the max, so the
    #    result equals the fused kernel's. Small stems keep the pool in their epilogue (the fused
    #    direct kernel); the wider convs that reach here go through the tensor cores.
    out_nodes = []
    for n in P.nodes:
        if n.op == "Conv" and n.p.pool is not None and not _small_stem_pool(P, n):
            pool = n.p.pool
            yv = P.values[n.outs[0]]
            nb, ih, iw, _ = _nhwc_shape(P.values[n.ins[0]])
            oc = yv.shape[3]
            k, st, pd = n.p.kernel, n.p.strides, n.p.pads
            ch, cw = conv_out(ih, k[0], st[0], pd[0], pd[2]), conv_out(iw, k[1], st[1], pd[1], pd[3])
            full = P.add_value(n.outs[0] + ".prepool", (nb, ch, cw, oc), yv.dtype, "nhwc")
            conv = Node("Conv", list(n.ins), [full], copy.copy(n.p), n.name)
            conv.p.pool = None
            out_nodes.append(conv)
            out_nodes.append(Node("MaxPool", [full], list(n.outs), pool, n.name + ".pool"))
            continue
        out_nodes.append(n)
    P.nodes = out_nodes

    # 1. fp32 NHWC graph input read by a tensor-core conv -> explicit conversion to fp16; an fp32
    #    input with fewer than 8 channels (an RGB image) read by a stride-1 k x k conv with 8 or more
    #    outputs -> conversion to fp16 NHWC zero-padded to 8 channels, the weights padded to match, so
    #    that the conv runs on the tensor cores instead of the CUDA-core direct kernel
    out_nodes = []
    for n in P.nodes:
        if n.op == "Conv":
            xv = P.values[n.ins[0]]
            nb, ih, iw, cin = _nhwc_shape(xv)
            W = P.values[n.ins[1]].const
            if xv.dtype == "f32" and xv.layout == "nhwc" and cin % 8 == 0 and n.p.group == 1 and n.p.strides == (1, 1):
                h = P.add_value(n.ins[0] + ".f16", xv.shape, "f16", "nhwc")
                out_nodes.append(Node("Convert", [n.ins[0]], [h], None, h))
                n.ins[0] = h
            elif (xv.dtype == "f32" and cin < 8 and n.p.group == 1 and tuple(n.p.strides) == (1, 1) and
                  n.p.pool is None and W.shape[0] >= 8 and tuple(n.p.kernel) != (1, 1) and
                  getattr(n.p, "in_scale", None) is None):
                h = P.add_value(n.ins[0] + ".f16x8", (nb, ih, iw, 8), "f16", "nhwc")
                out_nodes.append(Node("Convert", [n.ins[0]], [h], None, h))
                n.ins[0] = h
                wpad = np.zeros((W.shape[0], 8) + W.shape[2:], np.float32)
                wpad[:, :cin] = W
                n.ins[1] = P.add_const(n.ins[1] + "__pad8", wpad)
        out_nodes.append(n)
    P.nodes = out_nodes

    # 2. SE product x * s folded into the convs that consume it: depthwise convs scale their staged
    #    weights; 1x1 tensor-core convs get per-image scaled weights (sdx_conv_desc.in_scale; the
    #    scratch is added in the last step, after the rewrites that replace conv nodes)
    keep = []
    for n in P.nodes:
        if n.op == "Elementwise" and n.p.op == "mul" and n.p.act == "none":
            x, s = n.ins
            xs, ss = P.values[x].shape, P.values[s].shape
            cons = P.consumers(n.outs[0])
            if (len(ss) == 2 and len(xs) == 4 and ss == (xs[0], xs[3]) and cons and n.outs[0] != P.output and
                    P.values[s].dtype == "f32" and
                    all(c.op == "Conv" and c.ins[0] == n.outs[0] and
                        (c.p.group > 1 or _scaled_rows_bytes(P, c, x) > 0) for c in cons)):
                for c in cons:
                    c.ins[0] = x
                    c.p.in_scale = s
                continue
        keep.append(n)
    P.nodes = keep

    # 3. channel concat of nearest-upsampled inputs -> one ConcatNearest node that writes whole
    #    output pixels (the upsampled 24-channel slices alone would be partial-sector writes)
    prods = {o: m for m in P.nodes for o in m.outs}
    drop = set()
    out_nodes = []
    for n in P.nodes:
        if n.op == "Concat" and P.values[n.outs[0]].dtype == "f16" and len(P.shape(n.outs[0])) == 4:
            nb, oh, ow, _ = P.shape(n.outs[0])
            srcs, scales, resized, ok = [], [], [], True
            for v in n.ins:
                vs = P.shape(v)
                m = prods.get(v)
                if P.values[v].dtype != "f16" or len(vs) != 4 or vs[3] % 8 != 0:
                    ok = False
                    break
                if (m is not None and m.op == "ResizeNearest" and len(m.ins) == 1 and len(P.consumers(v)) == 1 and
                        m.p.scales[0] == m.p.scales[1] and v != P.output):
                    src = m.ins[0]
                    ss = P.shape(src)
                    f = m.p.scales[0]
                    if ss[1] * f != oh or ss[2] * f != ow or P.values[src].dtype != "f16":
                        ok = False
                        break
                    srcs.append(src)
                    scales.append(f)
                    resized.append(m)
                elif vs[1:3] == (oh, ow):
                    srcs.append(v)
                    scales.append(1)
                else:
                    ok = False
                    break
            if ok and resized and len(srcs) <= 8:
                drop.update(id(m) for m in resized)
                out_nodes.append(Node("ConcatNearest", srcs, list(n.outs), tuple(scales), n.name))
                continue
        out_nodes.append(n)
    P.nodes = [n for n in out_nodes if id(n) not in drop]

    # 4. channel concat: producers write into their slice. An input qualifies when a conv (or a
    #    nearest resize) produces it and its other readers are pools, which read the slice in place
    #    (sdx_pool_desc.x_pix_stride); the concat node stays for the other inputs only (their
    #    pointers; an in-place input is passed as 0)
    keep = []
    for n in P.nodes:
        if n.op == "Concat" and P.values[n.outs[0]].dtype == "f16" and not P.values[n.outs[0]].alias:
            prods = {o: m for m in P.nodes for o in m.outs}
            inplace = []
            for v in n.ins:
                m = prods.get(v)
                inplace.append(m is not None and (m.op == "ResizeNearest" or (m.op == "Conv" and m.p.group == 1)) and
                               v != P.output and
                               P.values[v].dtype == "f16" and P.shape(v)[3] % 8 == 0 and not P.values[v].alias and
                               n.ins.count(v) == 1 and
                               all(c is n or c.op in ("MaxPool", "AvgPool") for c in P.consumers(v)))
            off = 0
            for v, ok in zip(n.ins, inplace):
                if ok:
                    P.values[v].alias = (n.outs[0], off)
                off += P.shape(v)[3]
            if all(inplace):
                continue
            n.p = tuple(inplace)  # the lowering skips these inputs
        keep.append(n)
    P.nodes = keep

    # 5. FPN top-down add: ResizeNearest(x, scale 2, add = a conv's output that nothing else reads) ->
    #    the conv with x as a nearest-upsampled residual (sdx_conv_desc.add_up = 2), placed where the
    #    resize was; the conv's activation must be none (the add comes before it); add_relu -> relu
    prods = {o: m for m in P.nodes for o in m.outs}
    fused = {}
    for n in P.nodes:
        if n.op == "ResizeNearest" and len(n.ins) == 2 and tuple(n.p.scales) == (2, 2):
            x, a = n.ins
            m = prods.get(a)
            if m is None or m.op != "Conv" or len(P.consumers(a)) != 1 or a == P.output:
                continue
            xv, av = P.values[x], P.values[a]
            if (m.p.add or m.p.pool is not None or m.p.act != "none" or m.p.group != 1 or av.alias or
                    m.p.strides != (1, 1) or av.dtype != "f16" or xv.dtype != "f16" or av.layout != "nhwc" or
                    P.values[m.ins[0]].dtype != "f16" or len(av.shape) != 4 or av.shape[1] % 2 or av.shape[2] % 2 or
                    xv.shape != (av.shape[0], av.shape[1] // 2, av.shape[2] // 2, av.shape[3]) or
                    P.values[n.outs[0]].alias or av.shape[3] % 8):
                continue
            c = Node("Conv", list(m.ins), list(n.outs), copy.copy(m.p), m.name)
            c.p.add = x
            c.p.add_up = 2
            c.p.act = "relu" if n.p.add_relu else "none"
            fused[id(n)] = c
            fused[id(m)] = None
    if fused:
        P.nodes = [fused.get(id(n), n) for n in P.nodes if fused.get(id(n), n) is not None]

    # 6. ConvTranspose 2x2 (8, 16 or 24 outputs) whose output only a 2x2 ConvTranspose to one channel reads
    #    -> one ConvTChain node (the intermediate stays in registers, fp32)
    out_nodes = []
    drop = set()
    prods = {o: m for m in P.nodes for o in m.outs}
    for n in P.nodes:
        if n.op == "ConvTranspose":
            m = prods.get(n.ins[0])
            if m is not None and m.op == "ConvTranspose" and len(P.consumers(n.ins[0])) == 1 and n.ins[0] != P.output:
                W1, W2 = P.values[m.ins[1]].const, P.values[n.ins[1]].const
                ic1, oc1, kh1, kw1 = W1.shape
                ic2, oc2, kh2, kw2 = W2.shape
                xv = P.values[m.ins[0]]
                if (oc1 in (8, 16, 24) and (kh1, kw1) == (2, 2) and (kh2, kw2) == (2, 2) and oc2 == 1 and ic2 == oc1 and
                        ic1 % 8 == 0 and xv.dtype == "f16" and len(xv.shape) == 4):
                    drop.add(id(m))
                    out_nodes.append(Node("ConvTChain", [m.ins[0], m.ins[1], n.ins[1]], list(n.outs), (m.p, n.p),
                                          n.name))
                    continue
        out_nodes.append(n)
    P.nodes = [n for n in out_nodes if id(n) not in drop]

    # 7. image-session normalisation + the stem conv that alone reads its fp32 tensor -> ImageConv
    #    (the tensor is never written); the shape is the fused kernel's (sdx_image_conv)
    out_nodes = []
    drop = set()
    prods = {o: m for m in P.nodes for o in m.outs}
    for n in P.nodes:
        if n.op == "Conv" and not n.p.add and n.p.pool is None and n.p.group == 1:
            m = prods.get(n.ins[0])
            xv, yv = P.values[n.ins[0]], P.values[n.outs[0]]
            if (m is not None and m.op == "ImageToTensor" and len(P.consumers(n.ins[0])) == 1 and
                    xv.layout == "nchw" and xv.dtype == "f32" and n.ins[0] not in P.inputs and
                    n.p.kernel == (3, 3) and n.p.strides == (2, 2) and xv.shape[1] == 3 and
                    P.values[n.ins[1]].const.shape[0] == 16 and yv.dtype == "f16" and yv.layout == "nhwc" and
                    not yv.alias and P.values[m.ins[0]].shape[3] in (3, 4)):
                drop.add(id(m))
                out_nodes.append(Node("ImageConv", [m.ins[0]] + list(n.ins[1:]), list(n.outs),
                                      (m.p, n.p, xv.shape[2], xv.shape[3]), n.name))
                continue
        out_nodes.append(n)
    P.nodes = [n for n in out_nodes if id(n) not in drop]

    # 8. SE gate whose input is the output of a 1x1 tensor-core conv (fp16 TMA-store epilogue) -> the
    #    conv also writes the 32-pixel channel sums of its output (sdx_conv_desc.gap_sums, fp32
    #    [nb * h * w / 32, c]) and the gate reduces those instead of re-reading the tensor
    prods = {o: m for m in P.nodes for o in m.outs}
    for n in P.nodes:
        if n.op != "ChannelGate" or len(n.ins) != 3:
            continue
        m = prods.get(n.ins[0])
        if m is None or m.op != "Conv" or len(m.outs) != 1:
            continue
        xv, yv = P.values[m.ins[0]], P.values[m.outs[0]]
        W = P.values[m.ins[1]].const
        addv = P.values[m.p.add] if m.p.add else None
        if not (m.p.group == 1 and m.p.pool is None and tuple(m.p.kernel) == (1, 1) and
                tuple(m.p.strides) == (1, 1) and not any(m.p.pads) and getattr(m.p, "in_scale", None) is None and
                xv.dtype == "f16" and xv.layout == "nhwc" and len(xv.shape) == 4 and xv.shape[3] % 8 == 0 and
                yv.dtype == "f16" and yv.layout == "nhwc" and (W.shape[0] in (16, 32, 64) or W.shape[0] % 128 == 0) and
                (addv is None or (addv.dtype == "f16" and addv.layout == "nhwc" and not addv.alias))):
            continue
        if yv.alias and (P.shape(yv.alias[0])[3] % 8 or yv.alias[1] % 8):
            continue
        nb, h, w, c = yv.shape
        if (h * w) % 32 or c != W.shape[0]:
            continue
        sums = P.add_value(m.outs[0] + ".gapsums", (nb * h * w // 32, c), "f32", "raw")
        m.outs.append(sums)
        n.ins.append(sums)

    # 9. depthwise 3x3 (stride 1) whose output only a 1x1 tensor-core conv reads -> one DwPw node
    #    (sdx_dw_pw: the depthwise output is built tile by tile in shared memory, never stored); off
    #    while DW_PW_FUSION is False
    prods = {o: m for m in P.nodes for o in m.outs}
    fused, drop = {}, set()
    for n in (P.nodes if DW_PW_FUSION else []):
        if n.op != "Conv" or n.p.group != 1 or getattr(n.p, "in_scale", None) is not None:
            continue
        d = prods.get(n.ins[0])
        if (d is None or d.op != "Conv" or d.p.group == 1 or len(P.consumers(n.ins[0])) != 1 or
                n.ins[0] == P.output or P.values[n.ins[0]].alias or d.p.add or n.p.add or n.p.pool is not None or
                getattr(n.p, "add_up", 0) or P.values[n.outs[0]].alias):
            continue
        if not _dw_pw_ok(P, d, n):
            continue
        outs = list(n.outs)
        oh, ow = P.values[d.outs[0]].shape[1:3]
        if len(outs) > 1 and (ow % 32 or oh % 4):
            # the fused form's channel sums need whole 32-pixel runs per tile row: the gate reads the
            # tensor instead (step 8's sums dropped)
            sums = outs.pop()
            for g in P.consumers(sums):
                g.ins.remove(sums)
            del P.values[sums]
        fused[id(n)] = Node("DwPw", [d.ins[0], d.ins[1], n.ins[1]], outs, (d.p, n.p, (oh, ow)), n.name)
        drop.add(id(d))
    if fused:
        for n in P.nodes:
            if id(n) in drop:
                del P.values[n.outs[0]]  # the depthwise output is never stored
        P.nodes = [fused.get(id(n), n) for n in P.nodes if id(n) not in drop]

    # 10. scratch of the per-image scaled weights of the 1x1 convs that read x * s (step 2): an extra
    #    output of the conv, live for that node only
    for n in P.nodes:
        if n.op == "Conv" and n.p.group == 1 and getattr(n.p, "in_scale", None) is not None:
            nbytes = _scaled_rows_bytes(P, n, n.ins[0])
            assert nbytes > 0, n.name
            w = P.add_value(n.name + ".wscaled", (nbytes,), "u8", "raw")
            n.outs.append(w)
            n.p.w_scaled = w
    return P


def _dw_pw_descs(P: ExecPlan, x: str, dp, pp, oc: int, mid_hw: tuple, out: str):
    """(depthwise desc, 1x1 desc) of a depthwise conv (params dp) over `x` feeding a 1x1 conv (params pp,
    oc outputs) that writes `out`; shape and layout fields only."""
    nb, ih, iw, c = _nhwc_shape(P.values[x])
    oh, ow = mid_hw
    k = dp.kernel
    dwd = B.conv_desc(nb, ih, iw, c, c, k[0], k[1], stride=dp.strides, pads=dp.pads, group=c, act=dp.act)
    if getattr(dp, "in_scale", None) is not None:
        dwd.in_scale = 1  # set: the support query reads whether it is
    yslice = P.values[out].alias
    pwd = B.conv_desc(nb, oh, ow, c, oc, 1, 1, act=pp.act,
                      y_pix_stride=P.shape(yslice[0])[3] if yslice else 0, y_ch_off=yslice[1] if yslice else 0)
    return dwd, pwd


def _dw_pw_ok(P: ExecPlan, d: Node, n: Node) -> bool:
    xv, mv, yv = P.values[d.ins[0]], P.values[d.outs[0]], P.values[n.outs[0]]
    if xv.dtype != "f16" or xv.layout != "nhwc" or mv.dtype != "f16" or yv.dtype != "f16" or yv.layout != "nhwc":
        return False
    oc = P.values[n.ins[1]].const.shape[0]
    dwd, pwd = _dw_pw_descs(P, d.ins[0], d.p, n.p, oc, mv.shape[1:3], n.outs[0])
    return B.dw_pw_supported(dwd, pwd)


def _scaled_rows_bytes(P: ExecPlan, c: Node, x: str) -> int:
    """Scratch bytes if conv `c`, reading x * s, runs as a 1x1 tensor-core conv with per-image
    scaled weights (sdx_conv_scaled_weights_bytes), else 0."""
    if (c.op != "Conv" or c.p.group != 1 or tuple(c.p.kernel) != (1, 1) or tuple(c.p.strides) != (1, 1) or
            any(c.p.pads) or c.p.pool is not None):
        return 0
    xv, yv = P.values[x], P.values[c.outs[0]]
    if xv.dtype != "f16" or xv.layout != "nhwc" or yv.layout != "nhwc" or len(xv.shape) != 4:
        return 0
    nb, ih, iw, ic = xv.shape
    oc = P.values[c.ins[1]].const.shape[0]
    d = B.conv_desc(nb, ih, iw, ic, oc, 1, 1, y_dtype=torch.float16 if yv.dtype == "f16" else torch.float32)
    d.in_scale = 1  # set: the query only reads whether it is
    return B.conv_scaled_weights_bytes(d)


class CudaInferenceSession:
    """One compiled plan on one GPU: arena + const store + a graph-captured node list."""

    def __init__(self, plan: ExecPlan, device: int = 0, use_graph: bool = True, keep_all: bool = False):
        self.be = B.CudaBackend.get(device)
        self.device = torch.device("cuda", device)
        self.src_plan = plan
        self.plan = P = cuda_rewrite(plan)
        P.plan_arena(keep_all=keep_all)
        self._consts = {}
        self._scratch_bytes = 0
        for n in P.nodes:
            if n.op == "ChannelGate":
                nn, h, w, c = P.shape(n.ins[0])
                self._scratch_bytes = max(self._scratch_bytes, int(N.lib().sdx_channel_gate_scratch_bytes(nn, h * w, c)))
            if n.op == "Gemm" and getattr(n.p, "ctc", False):
                Wb = P.values[n.ins[1]].const
                k, nn = (Wb.shape[1], Wb.shape[0]) if n.p.trans_b else Wb.shape
                m = int(np.prod(P.shape(n.ins[0]))) // k
                self._scratch_bytes = max(self._scratch_bytes, int(N.lib().sdx_gemm_argmax_scratch_bytes(m, nn)))
        total = P.arena_bytes + self._scratch_bytes + 256
        h = ctypes.c_void_p()
        with torch.cuda.device(device):
            N.call("sdx_session_create", self.be.ctx, total, ctypes.byref(h))
        self.h = h
        base = ctypes.c_uint64()
        N.call("sdx_session_arena", h, ctypes.byref(base), None)
        self.base = base.value
        self.scratch = self.base + (P.arena_bytes + 255) // 256 * 256
        with torch.cuda.device(device):
            for n in P.nodes:
                kind, desc = self._lower(n)
                N.call("sdx_session_add_node", h, kind, ctypes.byref(desc), ctypes.sizeof(desc))
            ins = P.inputs
            self.in_off = P.offsets[ins[0]]
            self.in_bytes = max(P.offsets[v] + P.values[v].nbytes for v in ins) - self.in_off
            self.out_off = P.offsets[P.output]
            self.out_bytes = P.values[P.output].nbytes
            N.call("sdx_session_set_io", h, self.base + self.in_off, self.in_bytes, self.base + self.out_off,
                   self.out_bytes)
            torch.cuda.synchronize()
            N.call("sdx_session_build", h, int(use_graph))
        st = ctypes.c_void_p()
        N.call("sdx_session_stream", h, ctypes.byref(st))
        self.stream_ptr = st.value
        self.stream = torch.cuda.ExternalStream(st.value, device=self.device)
        self._pin_in = self._pin_out = None

    # ------------------------------------------------------------------ lowering
    def ptr(self, v: str) -> int:
        return self.base + self.plan.offsets[v]

    def _const_dev(self, key, make):
        t = self._consts.get(key)
        if t is None:
            t = self._consts[key] = make()
        return t

    def _f32(self, name):
        if name is None:
            return 0
        return B.ptr(self._const_dev(name, lambda: torch.from_numpy(self.plan.values[name].const).to(self.device)))

    def _zeros(self, n):
        return B.ptr(self._const_dev(("zeros", n), lambda: torch.zeros(n, dtype=torch.float32, device=self.device)))

    def _lower(self, n):
        P = self.plan
        op, p = n.op, n.p
        if op == "Conv":
            xv, yv = P.values[n.ins[0]], P.values[n.outs[0]]
            nb, ih, iw, ic = _nhwc_shape(xv)
            W = P.values[n.ins[1]].const
            oc = W.shape[0]
            yslice = yv.alias
            addv = P.values[p.add] if p.add else None
            d = B.conv_desc(nb, ih, iw, ic, oc, p.kernel[0], p.kernel[1], stride=p.strides, pads=p.pads,
                            group=p.group, act=p.act, x_dtype=torch.float16 if xv.dtype == "f16" else torch.float32,
                            x_layout=_LAY[xv.layout], y_dtype=torch.float16 if yv.dtype == "f16" else torch.float32,
                            y_layout=_LAY[yv.layout],
                            add_dtype=torch.float16 if (addv is None or addv.dtype == "f16") else torch.float32,
                            add_layout=_LAY[addv.layout] if addv else N.NHWC,
                            pool=p.pool is not None, pool_relu=bool(p.pool and p.pool.fuse_relu),
                            y_pix_stride=P.shape(yslice[0])[3] if yslice else 0, y_ch_off=yslice[1] if yslice else 0)
            d.add_up = getattr(p, "add_up", 0)  # a layout field: set before packing (the fold depends on it)
            scale = getattr(p, "in_scale", None)
            d.in_scale = self.ptr(scale) if scale else 0  # so is whether in_scale is set
            wt = self._const_dev(("convw", n.name), lambda: B.pack_conv(d, W, self.device))
            d.x = self.ptr(n.ins[0])
            d.w = B.ptr(wt)
            d.bias = self._f32(p.bias) if p.bias else (self._zeros(oc) if p.group > 1 else 0)
            d.add = self.ptr(p.add) if p.add else 0
            d.y = self.ptr(n.outs[0])
            wsc = getattr(p, "w_scaled", None)
            sums = [o for o in n.outs[1:] if o != wsc]
            d.gap_sums = self.ptr(sums[0]) if sums else 0
            d.w_scaled = self.ptr(wsc) if wsc else 0
            return N.OP_CONV, d
        if op == "DwPw":
            pd, pp, mid_hw = p
            Wd, Wp = P.values[n.ins[1]].const, P.values[n.ins[2]].const
            dwd, pwd = _dw_pw_descs(P, n.ins[0], pd, pp, Wp.shape[0], mid_hw, n.outs[0])
            wd = self._const_dev(("dww", n.name), lambda: B.pack_conv(dwd, Wd, self.device))
            wp = self._const_dev(("pww", n.name), lambda: B.pack_conv(pwd, Wp, self.device))
            d = N.DwPwDesc()
            d.dw, d.pw = dwd, pwd
            d.dw.x, d.dw.w = self.ptr(n.ins[0]), B.ptr(wd)
            d.dw.bias = self._f32(pd.bias) if pd.bias else self._zeros(dwd.oc)
            scale = getattr(pd, "in_scale", None)
            d.dw.in_scale = self.ptr(scale) if scale else 0
            d.pw.w = B.ptr(wp)
            d.pw.bias = self._f32(pp.bias) if pp.bias else 0
            d.pw.y = self.ptr(n.outs[0])
            d.pw.gap_sums = self.ptr(n.outs[1]) if len(n.outs) > 1 else 0
            return N.OP_DW_PW, d
        if op == "ConvTranspose":
            xv, yv = P.values[n.ins[0]], P.values[n.outs[0]]
            nb, ih, iw, ic = xv.shape
            W = P.values[n.ins[1]].const
            _, oc, kh, kw = W.shape
            d = N.ConvtDesc()
            d.batch, d.ih, d.iw, d.ic, d.oc, d.kh, d.kw = nb, ih, iw, ic, oc, kh, kw
            d.act, d.y_dtype = N.ACT[p.act], _DT[yv.dtype]
            if oc >= 8:
                wt = self._const_dev(("convtw", n.name), lambda: B.pack_convt(W, self.device))
            else:
                wt = self._const_dev(("convtw", n.name), lambda: torch.from_numpy(W).to(self.device))
            d.x, d.w, d.y = self.ptr(n.ins[0]), B.ptr(wt), self.ptr(n.outs[0])
            d.bias = self._f32(p.bias)
            return N.OP_CONVT, d
        if op == "ChannelGate":
            nb, h, w, c = P.shape(n.ins[0])
            W1, W2 = P.values[n.ins[1]].const, P.values[n.ins[2]].const
            d = N.GateDesc()
            d.batch, d.hw, d.c, d.r = nb, h * w, c, W1.shape[0]
            d.act1_relu, d.hard = int(p.act1 == "relu"), int(p.hard)
            d.alpha, d.beta, d.offset = p.alpha, p.beta, p.offset
            d.x, d.w1, d.w2 = self.ptr(n.ins[0]), self._f32(n.ins[1]), self._f32(n.ins[2])
            d.b1, d.b2 = self._f32(p.b1), self._f32(p.b2)
            d.s, d.partial = self.ptr(n.outs[0]), self.scratch
            d.sums = self.ptr(n.ins[3]) if len(n.ins) > 3 else 0
            return N.OP_CHANNEL_GATE, d
        if op == "Elementwise":
            a, b = n.ins
            sa, sb = P.shape(a), P.shape(b)
            va, vb, vy = P.values[a], P.values[b], P.values[n.outs[0]]
            f16 = va.dtype == "f16" and vb.dtype == "f16" and vy.dtype == "f16"
            d = N.MiscDesc()
            d.op, d.relu = N.EW[p.op], int(p.act == "relu")
            if sa == sb and f16 and p.act in ("none", "relu") and int(np.prod(sa)) % 8 == 0:
                d.n = int(np.prod(sa))
                d.a, d.b, d.y = self.ptr(a), self.ptr(b), self.ptr(n.outs[0])
                return N.OP_BINARY, d
            if (len(sa) == 4 and sb == (sa[0], sa[3]) and va.dtype == "f16" and vy.dtype == "f16" and vb.dtype == "f32"
                    and p.act in ("none", "relu") and not vb.is_const):
                nb, c = sa[0], sa[-1]
                d.batch, d.c, d.pixels = nb, c, int(np.prod(sa)) // (nb * c)
                d.x, d.b, d.y = self.ptr(a), self.ptr(b), self.ptr(n.outs[0])
                return N.OP_CHANNEL_BROADCAST, d
            # numpy broadcast (Ops.Elementwise's general case); the plan's [N, C] gate vector is
            # [N, 1, 1, C] against an NHWC tensor
            if len(sb) == 2 and len(sa) == 4 and sb == (sa[0], sa[3]):
                sb = (sa[0], 1, 1, sa[3])
            if len(sa) == 2 and len(sb) == 4 and sa == (sb[0], sb[3]):
                sa = (sb[0], 1, 1, sb[3])
            out = np.broadcast_shapes(sa, sb)
            r = len(out)
            full = lambda s: [1] * (r - len(s)) + list(s)
            bd = N.BcastDesc()
            bd.rank = r
            for i, (o, x, z) in enumerate(zip(out, full(sa), full(sb))):
                bd.out_shape[i], bd.a_shape[i], bd.b_shape[i] = o, x, z
            bd.op, bd.act = N.EW[p.op], N.ACT[p.act]
            bd.a_dtype, bd.b_dtype, bd.y_dtype = _DT[va.dtype], _DT[vb.dtype], _DT[vy.dtype]
            bd.a = self._f32(a) if va.is_const else self.ptr(a)
            bd.b = self._f32(b) if vb.is_const else self.ptr(b)
            bd.y = self.ptr(n.outs[0])
            return N.OP_BINARY_BCAST, bd
        if op == "SafeDiv":
            va = P.values[n.ins[0]]
            d = N.SafeDivDesc()
            d.n, d.eps, d.lo, d.hi, d.dtype = int(np.prod(va.shape)), p.eps, p.lo, p.hi, _DT[va.dtype]
            d.a, d.b, d.y = self.ptr(n.ins[0]), self.ptr(n.ins[1]), self.ptr(n.outs[0])
            return N.OP_SAFE_DIV, d
        if op == "ChannelShift":
            nb, h, w, c = P.shape(n.ins[0])
            d = N.ShiftDesc()
            d.batch, d.h, d.w, d.c, d.axis, d.ngroups = nb, h, w, c, p.axis, len(p.group_ends)
            for i, (e, o) in enumerate(zip(p.group_ends, p.offsets)):
                d.group_ends[i], d.offsets[i] = e, o
            d.dtype, d.x, d.y = _DT[P.values[n.ins[0]].dtype], self.ptr(n.ins[0]), self.ptr(n.outs[0])
            return N.OP_CHANNEL_SHIFT, d
        if op == "UpHead":
            x, skip, wv = n.ins
            nb, ih, iw, c = P.shape(x)
            _, oh, ow, oc = P.shape(n.outs[0])
            W = P.values[wv].const.reshape(oc, c)
            d = N.UpHeadDesc()
            d.batch, d.ih, d.iw, d.c, d.oh, d.ow, d.oc = nb, ih, iw, c, oh, ow, oc
            d.scale_h, d.scale_w = p.scales
            d.resize_relu, d.skip_relu, d.act = int(p.resize_relu), int(p.skip_relu), N.ACT[p.act]
            d.x_dtype, d.skip_dtype = _DT[P.values[x].dtype], _DT[P.values[skip].dtype]
            d.y_dtype = _DT[P.values[n.outs[0]].dtype]
            wt = self._const_dev(("uphead", n.name), lambda: torch.from_numpy(np.ascontiguousarray(W)).to(self.device))
            d.x, d.skip, d.w, d.bias, d.y = self.ptr(x), self.ptr(skip), B.ptr(wt), self._f32(p.bias), self.ptr(n.outs[0])
            return N.OP_UPHEAD, d
        if op == "MatMul":
            a, b = n.ins
            sa, sb = P.shape(a), P.shape(b)
            r = max(len(sa), len(sb))
            d = N.MatMulDesc()
            d.rank = r
            for i, (x, z) in enumerate(zip([1] * (r - len(sa)) + list(sa), [1] * (r - len(sb)) + list(sb))):
                d.a_shape[i], d.b_shape[i] = x, z
            d.a_dtype, d.b_dtype = _DT[P.values[a].dtype], _DT[P.values[b].dtype]
            d.y_dtype = _DT[P.values[n.outs[0]].dtype]
            d.a, d.b, d.y = self.ptr(a), self.ptr(b), self.ptr(n.outs[0])
            return N.OP_MATMUL, d
        if op == "ResizeNearest":
            x = n.ins[0]
            nb, ih, iw, c = P.shape(x)
            yv = P.values[n.outs[0]]
            d = N.ResizeDesc()
            d.batch, d.ih, d.iw, d.c = nb, ih, iw, c
            d.oh, d.ow = yv.shape[1], yv.shape[2]
            d.add_relu = int(p.add_relu)
            d.y_pix_stride = P.shape(yv.alias[0])[3] if yv.alias else c
            d.y_ch_off = yv.alias[1] if yv.alias else 0
            d.x = self.ptr(x)
            d.add = self.ptr(n.ins[1]) if len(n.ins) > 1 else 0
            d.y = self.ptr(n.outs[0])
            return N.OP_RESIZE_NEAREST, d
        if op == "ImageToTensor":
            img, yv = P.values[n.ins[0]], P.values[n.outs[0]]
            nb, ih, iw, bpp = img.shape
            d = N.ImageDesc()
            d.batch, d.ih, d.iw, d.bpp, d.swap_rb = nb, ih, iw, bpp, int(p.swap_rb)
            if yv.layout == "nchw":
                d.oh, d.ow, d.y_nhwc_f16 = yv.shape[2], yv.shape[3], 0
            else:
                d.oh, d.ow, d.y_nhwc_f16 = yv.shape[1], yv.shape[2], 1
            d.pad_t, d.pad_l = p.pads
            d.stride, d.image_bytes = iw * bpp, ih * iw * bpp
            d.src, d.lut, d.y = self.ptr(n.ins[0]), self._f32(p.lut), self.ptr(n.outs[0])
            return N.OP_IMAGE, d
        if op == "ConvTChain":
            p1, p2 = p
            xv, yv = P.values[n.ins[0]], P.values[n.outs[0]]
            nb, ih, iw, ic = xv.shape
            W1, W2 = P.values[n.ins[1]].const, P.values[n.ins[2]].const
            _, oc1, kh, kw = W1.shape
            d = N.ConvtChainDesc()
            f = d.first
            f.batch, f.ih, f.iw, f.ic, f.oc, f.kh, f.kw = nb, ih, iw, ic, oc1, kh, kw
            f.act, f.y_dtype = N.ACT[p1.act], N.F16
            w1 = self._const_dev(("convtw", n.name + ".1"), lambda: B.pack_convt(W1, self.device))
            w2 = self._const_dev(("convtw", n.name + ".2"), lambda: torch.from_numpy(W2).to(self.device))
            f.x, f.w, f.bias, f.y = self.ptr(n.ins[0]), B.ptr(w1), self._f32(p1.bias), 0
            d.oc2, d.kh2, d.kw2, d.act2, d.y_dtype = 1, 2, 2, N.ACT[p2.act], _DT[yv.dtype]
            d.w2 = B.ptr(w2)
            d.bias2 = self._f32(p2.bias) if p2.bias else self._zeros(1)
            d.y = self.ptr(n.outs[0])
            if not p1.bias:
                f.bias = self._zeros(kh * kw * oc1)
            return N.OP_CONVT_CHAIN, d
        if op == "ImageConv":
            ip, cp, th, tw = p
            img = P.values[n.ins[0]]
            nb, ih, iw, bpp = img.shape
            W = P.values[n.ins[1]].const
            d = N.ImageConvDesc()
            im = d.image
            im.batch, im.ih, im.iw, im.bpp, im.swap_rb = nb, ih, iw, bpp, int(ip.swap_rb)
            im.oh, im.ow, im.y_nhwc_f16 = th, tw, 0
            im.pad_t, im.pad_l = ip.pads
            im.stride, im.image_bytes = iw * bpp, ih * iw * bpp
            im.src, im.lut, im.y = self.ptr(n.ins[0]), self._f32(ip.lut), 0
            cd = B.conv_desc(nb, th, tw, 3, W.shape[0], cp.kernel[0], cp.kernel[1], stride=cp.strides, pads=cp.pads,
                             act=cp.act, x_dtype=torch.float32, x_layout=N.NCHW)
            wt = self._const_dev(("convw", n.name), lambda: B.pack_conv(cd, W, self.device))
            cd.x, cd.w, cd.y = 0, B.ptr(wt), self.ptr(n.outs[0])
            cd.bias = self._f32(cp.bias) if cp.bias else 0
            d.conv = cd
            return N.OP_IMAGE_CONV, d
        if op == "ConcatNearest":
            nb, oh, ow, _ = P.shape(n.outs[0])
            d = N.MiscDesc()
            d.batch, d.rows, d.n = nb, oh, ow
            d.nin = len(n.ins)
            for i, v in enumerate(n.ins):
                d.counts[i] = P.shape(v)[-1]
                d.aux[i] = int(p[i])
                d.ins[i] = self.ptr(v)
            d.y = self.ptr(n.outs[0])
            return N.OP_CONCAT_NEAREST, d
        if op == "Concat":
            d = N.MiscDesc()
            first = P.shape(n.ins[0])
            d.pixels = int(np.prod(first[:-1]))
            d.nin = len(n.ins)
            inplace = p if isinstance(p, tuple) else (False,) * len(n.ins)
            for i, v in enumerate(n.ins):
                d.counts[i] = P.shape(v)[-1]
                d.ins[i] = 0 if inplace[i] else self.ptr(v)  # 0: written in place by its producer
            d.y = self.ptr(n.outs[0])
            return N.OP_CONCAT, d
        if op in ("MaxPool", "AvgPool"):
            nb, ih, iw, c = P.shape(n.ins[0])
            _, oh, ow, _ = P.shape(n.outs[0])
            d = N.PoolDesc()
            d.batch, d.ih, d.iw, d.c, d.oh, d.ow = nb, ih, iw, c, oh, ow
            d.kh, d.kw = p.kernel
            d.sh, d.sw = p.strides
            d.pad_t, d.pad_l = p.pads[0], p.pads[1]
            d.is_avg, d.relu, d.count_include_pad = int(op == "AvgPool"), int(p.fuse_relu), int(p.count_include_pad)
            d.x, d.y = self.ptr(n.ins[0]), self.ptr(n.outs[0])
            xs = P.values[n.ins[0]].alias  # the input is a channel slice of a concat (written in place)
            if xs:
                d.x_pix_stride, d.x_ch_off = P.shape(xs[0])[3], xs[1]
            return N.OP_POOL, d
        if op == "Gemm" and getattr(p, "ctc", False):
            # CTC head: indices (int32 [rows]) then probabilities (fp32 [rows]) in the output value
            a = n.ins[0]
            Wb = P.values[n.ins[1]].const
            k, nn = (Wb.shape[1], Wb.shape[0]) if p.trans_b else Wb.shape
            m = int(np.prod(P.shape(a))) // k
            d = N.GemmArgmaxDesc()
            g = d.gemm
            g.m, g.k, g.n, g.lda = m, k, nn, k
            g.act, g.y_dtype, g.add_dtype = N.ACT["none"], N.F32, N.F16
            wt = self._const_dev(("gemmw", n.name), lambda: B.pack_gemm(Wb, p.trans_b, self.device))
            g.a, g.w, g.bias = self.ptr(a), B.ptr(wt), self._f32(p.bias)
            d.indices = self.ptr(n.outs[0])
            d.probs = self.ptr(n.outs[0]) + 4 * m
            d.scratch = self.scratch
            return N.OP_GEMM_ARGMAX, d
        if op == "Gemm":
            a = n.ins[0]
            Wb = P.values[n.ins[1]].const
            k, nn = (Wb.shape[1], Wb.shape[0]) if p.trans_b else Wb.shape
            m = int(np.prod(P.shape(a))) // k
            yv = P.values[n.outs[0]]
            d = N.GemmDesc()
            d.m, d.k, d.n, d.lda = m, k, nn, k
            d.act, d.y_dtype = N.ACT[p.act], _DT[yv.dtype]
            d.add_dtype = _DT[P.values[p.add].dtype] if p.add else N.F16
            d.ldy, d.ldadd = nn, nn
            wt = self._const_dev(("gemmw", n.name), lambda: B.pack_gemm(Wb, p.trans_b, self.device))
            d.a, d.w, d.y = self.ptr(a), B.ptr(wt), self.ptr(n.outs[0])
            d.bias = self._f32(p.bias)
            d.add = self.ptr(p.add) if p.add else 0
            return N.OP_GEMM, d
        if op == "Convert":
            xv, yv = P.values[n.ins[0]], P.values[n.outs[0]]
            nb, h, w, c = _nhwc_shape(xv)
            c_out = _nhwc_shape(yv)[3]
            d = N.MiscDesc()
            d.batch, d.c, d.pixels = nb, c, h * w
            d.aux[0] = c_out if c_out != c else 0  # zero-padded channels
            d.x_dtype, d.x_layout, d.y_dtype, d.y_layout = _DT[xv.dtype], _LAY[xv.layout], _DT[yv.dtype], _LAY[yv.layout]
            d.x, d.y = self.ptr(n.ins[0]), self.ptr(n.outs[0])
            return N.OP_CONVERT, d
        if op == "LayerNorm":
            c = P.shape(n.ins[0])[-1]
            d = N.MiscDesc()
            d.rows, d.c, d.eps = int(np.prod(P.shape(n.ins[0]))) // c, c, p.eps
            d.x, d.w, d.bias, d.y = self.ptr(n.ins[0]), self._f32(n.ins[1]), self._f32(n.ins[2]), self.ptr(n.outs[0])
            return N.OP_LAYERNORM, d
        if op == "Softmax":
            c = P.shape(n.ins[0])[-1]
            d = N.MiscDesc()
            d.rows, d.c, d.y_dtype = int(np.prod(P.shape(n.ins[0]))) // c, c, _DT[P.values[n.outs[0]].dtype]
            d.x, d.y = self.ptr(n.ins[0]), self.ptr(n.outs[0])
            return N.OP_SOFTMAX, d
        if op == "Attention":
            nb, t, _ = P.shape(n.ins[0])
            d = N.MiscDesc()
            d.batch, d.t, d.heads, d.d, d.scale = nb, t, p.heads, p.head_dim, p.scale
            d.x, d.y = self.ptr(n.ins[0]), self.ptr(n.outs[0])
            return N.OP_ATTENTION, d
        if op == "Act":
            d = N.MiscDesc()
            d.n, d.act = int(np.prod(P.shape(n.ins[0]))), N.ACT[p]
            d.x, d.y = self.ptr(n.ins[0]), self.ptr(n.outs[0])
            return N.OP_ACT, d
        raise NotImplementedError(f"no CUDA lowering for {op}")

    # ------------------------------------------------------------------ running
    def node_count(self) -> int:
        c = ctypes.c_int()
        N.call("sdx_session_node_count", self.h, ctypes.byref(c))
        return c.value

    def enqueue(self) -> None:
        """Device-resident run on the session stream (inputs already in the arena)."""
        N.call("sdx_session_enqueue", self.h)

    def write_inputs(self, feeds: dict) -> None:
        """Copy inputs into the arena (synchronous): numpy arrays from the host, or torch tensors
        already on this device (plan.feeds_dev)."""
        for name in self.plan.inputs:
            dt = self.plan.values[name].dtype
            f = feeds[name]
            if isinstance(f, torch.Tensor):
                t = f.to(self.device).contiguous()
                want = {"u8": torch.uint8, "f16": torch.float16}.get(dt, torch.float32)
                if t.dtype != want:
                    t = t.to(want)
                if tuple(t.shape) != tuple(self.plan.values[name].shape):
                    raise ValueError(f"input {name}: shape {tuple(t.shape)}, plan {self.plan.values[name].shape}")
            else:
                a = np.ascontiguousarray(f, np.uint8 if dt == "u8" else np.float32)
                t = torch.from_numpy(a).to(self.device)
                if dt == "f16":
                    t = t.half()
            torch.cuda.synchronize(self.device)
            N.call("sdx_memcpy_dtod_async", self.be.ctx, self.ptr(name), B.ptr(t), t.numel() * t.element_size(),
                   ctypes.c_void_p(self.stream_ptr))
            N.call("sdx_stream_sync", self.be.ctx, ctypes.c_void_p(self.stream_ptr), 0)

    def read(self, name: str) -> np.ndarray:
        """A value's arena contents as fp32 (dense values only)."""
        v = self.plan.values[name]
        dt = _NP[v.dtype]
        out = np.empty(v.shape, dt)
        N.call("sdx_stream_sync", self.be.ctx, ctypes.c_void_p(self.stream_ptr), 0)
        N.call("sdx_memcpy_dtoh_async", self.be.ctx, out.ctypes.data_as(ctypes.c_void_p), self.ptr(name), out.nbytes,
               ctypes.c_void_p(self.stream_ptr))
        N.call("sdx_stream_sync", self.be.ctx, ctypes.c_void_p(self.stream_ptr), 0)
        return out if v.dtype == "i32" else out.astype(np.float32)

    def pinned_io(self):
        """Pinned host staging buffers (input region, output) for end-to-end runs."""
        if self._pin_in is None:
            self._pin_in = torch.empty(self.in_bytes, dtype=torch.uint8).pin_memory()
            self._pin_out = torch.empty(self.out_bytes, dtype=torch.uint8).pin_memory()
        return self._pin_in, self._pin_out

    def stage_inputs(self, feeds: dict) -> None:
        pin_in, _ = self.pinned_io()
        buf = pin_in.numpy()
        for name in self.plan.inputs:
            dt = self.plan.values[name].dtype
            a = np.ascontiguousarray(feeds[name], np.uint8 if dt == "u8" else np.float32)
            if dt == "f16":
                a = a.astype(np.float16)
            off = self.plan.offsets[name] - self.in_off
            buf[off:off + a.nbytes] = a.view(np.uint8).ravel()

    def run(self, feeds: dict | None = None, timeout_ms: int = 0, copy: bool = True) -> np.ndarray:
        """End-to-end: pinned host input -> device, graph, device -> pinned host output, wait.
        copy=False returns a view of the pinned output buffer (valid until the next run)."""
        pin_in, pin_out = self.pinned_io()
        if feeds is not None:
            self.stage_inputs(feeds)
        N.call("sdx_session_run", self.h, ctypes.c_void_p(pin_in.data_ptr()), ctypes.c_void_p(pin_out.data_ptr()),
               timeout_ms)
        return self._output_view(pin_out, copy)

    def _output_view(self, pin_out, copy: bool) -> np.ndarray:
        ov = self.plan.values[self.plan.output]
        dt = _NP[ov.dtype]
        y = pin_out.numpy().view(dt).reshape(ov.shape)
        if ov.dtype == "i32":
            return y.copy() if copy else y
        return y.astype(np.float32) if (copy or dt != np.float32) else y

    def submit(self, pin_in: torch.Tensor, pin_out: torch.Tensor) -> None:
        """Pipelined end-to-end run (sdx_session_submit): returns at once; the pinned buffers must
        stay untouched until wait()."""
        N.call("sdx_session_submit", self.h, ctypes.c_void_p(pin_in.data_ptr()), ctypes.c_void_p(pin_out.data_ptr()))

    def wait(self, timeout_ms: int = 0) -> None:
        N.call("sdx_session_wait", self.h, timeout_ms)

    def close(self) -> None:
        if getattr(self, "h", None):
            N.call("sdx_session_destroy", self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
