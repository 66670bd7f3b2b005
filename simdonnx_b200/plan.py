"""The reference's lowered plan, restated: ExecOp nodes with their fused parameter records over
named values, plus an arena planner with int64 byte offsets.

Mirrors src/Engine/ExecPlan.cs: ExecOp (:4-40), ConvP (:50-65), PoolP (:67-74), EwP (:76-80),
LnP (:82-85), GemmP (:87-93), ConvTP (:108-114), ResizeNearestP (:116-121), ChannelGateP (:151-158),
AttentionP (:160-174), CValue (:202-220), ExecNode (:235-276), ExecPlan (:279-317). Plans here are
built with the fusions of the reference's GraphCompiler already applied (Conv+BN+act, conv
residual, ChannelGate, FuseResizeAdd, ConvT bias, LayerNorm, Attention on GPU plans), for NHWC
storage (LayoutPlanner): 4-D activations are stored [N, H, W, C].
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

ACTS = ("none", "relu", "sigmoid", "gelu", "hardswish", "swish")


@dataclass
class PoolP:
    kernel: tuple
    strides: tuple
    pads: tuple = (0, 0, 0, 0)
    fuse_relu: bool = False
    count_include_pad: bool = False


@dataclass
class ConvP:
    kernel: tuple
    strides: tuple = (1, 1)
    pads: tuple = (0, 0, 0, 0)  # top, left, bottom, right
    group: int = 1
    act: str = "none"
    bias: str | None = None      # BiasValue
    add: str | None = None       # AddValue (residual, added before the activation)
    pool: PoolP | None = None    # fused 2x2/2 max pool (NHWC plans)


@dataclass
class ConvTP:
    kernel: tuple
    bias: str | None = None
    act: str = "none"


@dataclass
class GemmP:
    trans_b: bool = False
    bias: str | None = None
    act: str = "none"
    add: str | None = None       # residual folded into the Gemm epilogue (GPU plans)
    ctc: bool = False            # CTC head (CtcProjection.ArgMax): output i32 [2, rows] = per row the
                                 # index of the first maximum, then its softmax probability (fp32 bits)


@dataclass
class EwP:
    op: str                      # add | sub | mul | div
    act: str = "none"


@dataclass
class ResizeNearestP:
    scales: tuple                # (sh, sw)
    add_relu: bool = False       # optional addend in ins[1]: out = resize(x) + [relu](add)


@dataclass
class ChannelGateP:
    b1: str | None = None
    b2: str | None = None
    act1: str = "relu"
    hard: bool = True
    alpha: float = 0.2
    beta: float = 0.5
    offset: float = 0.0


@dataclass
class LnP:
    eps: float = 1e-5


@dataclass
class AttentionP:
    heads: int
    head_dim: int
    scale: float


@dataclass
class ImageP:
    """Image-session preprocessing (VkImageSession / img2nhwc.comp): u8 pixels -> lut -> tensor."""
    lut: str                     # const fp32 [3, 256]
    bpp: int = 3
    swap_rb: bool = False
    pads: tuple = (0, 0)         # image position (top, left) inside the tensor; replicate padding


@dataclass
class BatchNormP:
    """Inference BatchNormalization before the load-time rewrite (OnnxRewrites.FoldConvBatchNorm,
    src/Onnx/OnnxRewrites.cs:71-111, or GraphCompiler.EmitBatchNorm, src/Engine/GraphCompiler.cs:1896-1922):
    names of the fp32 [C] constants and epsilon."""
    gamma: str
    beta: str
    mean: str
    var: str
    eps: float = 1e-5


@dataclass
class SafeDivP:
    """SafeDivOp (src/Engine/Fusions/SafeDivOp.cs:9-13): out = clamp(a / max(b, eps), lo, hi)."""
    eps: float
    lo: float
    hi: float


@dataclass
class ShiftP:
    """ChannelShiftOp (src/Engine/Fusions/ChannelShiftOp.cs:9-14): per channel group a zero-filled
    shift along H (axis 2) or W (axis 3)."""
    axis: int
    group_ends: tuple
    offsets: tuple


@dataclass
class UpHeadP:
    """UpHeadOp (src/Engine/Fusions/UpHeadOp.cs:16-30): bilinear resize of ins[0] by scales (h, w),
    [relu], + [relu](ins[1]), 1x1 conv ins[2] ([oc, c, 1, 1]) + bias, act."""
    scales: tuple
    resize_relu: bool = False
    skip_relu: bool = False
    act: str = "none"
    bias: str | None = None


@dataclass
class Value:
    name: str
    shape: tuple
    dtype: str = "f16"           # storage type on the CUDA path: f16 activations, f32 graph I/O and gates
    layout: str = "nhwc"         # physical layout of rank-4 values
    const: np.ndarray | None = None
    alias: tuple | None = None   # (wider value, channel offset): stored as a channel slice of it

    @property
    def is_const(self) -> bool:
        return self.const is not None

    @property
    def nbytes(self) -> int:
        return int(np.prod(self.shape)) * {"f16": 2, "u8": 1}.get(self.dtype, 4)  # f32, i32: 4


@dataclass
class Node:
    op: str                      # ExecOp name: Conv, ConvTranspose, Gemm, MaxPool, AvgPool, ChannelGate, ...
    ins: list
    outs: list
    p: object = None
    name: str = ""


@dataclass
class ExecPlan:
    values: dict = field(default_factory=dict)
    nodes: list = field(default_factory=list)
    input: str = ""
    output: str = ""
    inputs: list = field(default_factory=list)     # every graph input, back to back at the arena start
    feeds: dict = field(default_factory=dict)      # input name -> callable making its seeded data
    feeds_dev: dict = field(default_factory=dict)  # input name -> callable(device): the same data as a
                                                   # torch tensor made on that device (large batches)
    offsets: dict = field(default_factory=dict)   # value -> arena byte offset (int64)
    arena_bytes: int = 0

    # ---- building
    def add_value(self, name, shape, dtype="f16", layout="nhwc", const=None) -> str:
        assert name not in self.values, name
        self.values[name] = Value(name, tuple(int(s) for s in shape), dtype, layout, const)
        return name

    def add_const(self, name, array) -> str:
        a = np.ascontiguousarray(array, np.float32)
        return self.add_value(name, a.shape, "f32", "raw", a)

    def add_node(self, op, ins, outs, p=None, name="") -> Node:
        n = Node(op, list(ins), list(outs), p, name or outs[0])
        self.nodes.append(n)
        return n

    def shape(self, v) -> tuple:
        return self.values[v].shape

    def consumers(self, v) -> list:
        out = []
        for n in self.nodes:
            refs = list(n.ins) + _param_refs(n.p)
            if v in refs:
                out.append(n)
        return out

    # ---- arena (PlanArena, src/Engine/GraphCompiler.cs:1336-1474, with int64 byte offsets)
    def plan_arena(self, align: int = 256, keep_all: bool = False) -> int:
        """Lifetime packing of every non-constant value: first fit in a free list, the graph input
        first and live for the whole run (:1371-1382), the output live to the end. With keep_all
        every value keeps its own region (debug runs that read back each node's output)."""
        acts = [v for v in self.values.values() if not v.is_const]
        last_use = {}
        for i, n in enumerate(self.nodes):
            for v in list(n.ins) + _param_refs(n.p) + list(n.outs):
                if v in self.values and not self.values[v].is_const:
                    last_use[v] = i
        last_use[self.input] = len(self.nodes)
        last_use[self.output] = len(self.nodes)
        sizes = {v.name: (v.nbytes + align - 1) // align * align for v in acts}
        for v in acts:  # a value aliased into a wider tensor lives as long as that tensor
            if getattr(v, "alias", None):
                last_use[v.alias[0]] = max(last_use.get(v.alias[0], -1), last_use.get(v.name, -1))
        offsets = {}
        live = []  # (start, end, name)
        top = 0

        def alloc(name):
            nonlocal top
            size = sizes[name]
            live.sort()
            cur = 0
            for s, e, _ in live:
                if s - cur >= size:
                    break
                cur = max(cur, e)
            offsets[name] = cur
            live.append((cur, cur + size, name))
            top = max(top, cur + size)

        ins = self.inputs or [self.input]
        for v in ins:
            alloc(v)
            last_use[v] = len(self.nodes)
        for i, n in enumerate(self.nodes):
            for v in n.outs:
                tgt = self.values[v].alias[0] if getattr(self.values[v], "alias", None) else v
                if tgt not in offsets:
                    alloc(tgt)
                if tgt != v:
                    last_use[tgt] = max(last_use.get(tgt, -1), last_use.get(v, -1), i)
            if not keep_all:
                live[:] = [(s, e, nm) for (s, e, nm) in live if last_use.get(nm, -1) > i]
        for v in acts:  # values no node produces or reads (none in a pruned plan)
            if v.name not in offsets and not getattr(v, "alias", None):
                alloc(v.name)
        for v in acts:  # aliases: the target's offset, the channel offset applies per pixel
            if getattr(v, "alias", None):
                offsets[v.name] = offsets[v.alias[0]]
        self.offsets = offsets
        self.arena_bytes = top
        return top


def _param_refs(p) -> list:
    """Value ids read through op params (ExecNode.ParamRefs, src/Engine/ExecPlan.cs:246-262)."""
    if isinstance(p, tuple):  # fused nodes carry the params of the nodes they replace
        return [v for q in p for v in _param_refs(q)]
    refs = []
    for attr in ("bias", "add", "b1", "b2", "in_scale", "gamma", "beta", "mean", "var"):
        v = getattr(p, attr, None)
        if isinstance(v, str):
            refs.append(v)
    return refs


def conv_out(i: int, k: int, s: int, p0: int, p1: int) -> int:
    """ONNX conv output size (src/Engine/GraphCompiler.cs:1790-1794)."""
    return (i + p0 + p1 - k) // s + 1
