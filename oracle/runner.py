"""CPU executor of an ExecPlan over the oracle kernels -- TEST INFRASTRUCTURE ONLY.

Restates the reference's InferenceSession node loop for NHWC plans (src/Engine/Session.cs:88-112,
ExecNhwc :322-427, generic ops :148-318): every node runs the oracle's restatement of the
reference CPU kernel, fp32 end to end. Packed weights are cached per node like the reference's
CpuKernels.Cache (src/Engine/CpuKernels.cs:16-40).
"""
from __future__ import annotations

import numpy as np

import oracle as O


def fold_batchnorm(plan):
    """The reference's load-time BatchNorm handling, restated (independently of the product's
    rewrite): OnnxRewrites.FoldConvBatchNorm (src/Onnx/OnnxRewrites.cs:71-111) folds a BatchNorm
    into the Conv it alone reads (no activation, pool or residual in between; conv output not a
    graph output): scale = gamma / sqrt(var + eps), w *= scale, b = (b - mean) * scale + beta, fp32.
    Every other BatchNorm stays and runs as x * s + t (GraphCompiler.EmitBatchNorm,
    src/Engine/GraphCompiler.cs:1896-1922)."""
    import copy
    if not any(n.op == "BatchNorm" for n in plan.nodes):
        return plan
    P = copy.copy(plan)
    P.values = dict(plan.values)
    nodes = [copy.copy(n) for n in plan.nodes]
    for n in nodes:
        n.ins, n.outs, n.p = list(n.ins), list(n.outs), copy.copy(n.p)
    prod = {o: m for m in nodes for o in m.outs}
    uses = {}
    for m in nodes:
        for v in m.ins:
            uses[v] = uses.get(v, 0) + 1
        for attr in ("bias", "add", "b1", "b2", "in_scale"):
            v = getattr(m.p, attr, None)
            if isinstance(v, str):
                uses[v] = uses.get(v, 0) + 1
    keep = []
    for n in nodes:
        if n.op == "BatchNorm":
            c = prod.get(n.ins[0])
            if (c is not None and c.op == "Conv" and uses.get(n.ins[0], 0) == 1 and n.ins[0] != P.output and
                    c.p.pool is None and not c.p.add and c.p.act == "none"):
                g, be = P.values[n.p.gamma].const, P.values[n.p.beta].const
                mu, var = P.values[n.p.mean].const, P.values[n.p.var].const
                scale = (g / np.sqrt(var + np.float32(n.p.eps), dtype=np.float32)).astype(np.float32)
                w = P.values[c.ins[1]].const
                b0 = P.values[c.p.bias].const if c.p.bias else np.zeros(w.shape[0], np.float32)
                wn, bn_ = "oracle.bnfold." + c.name + ".w", "oracle.bnfold." + c.name + ".b"
                P.values[wn] = copy.copy(P.values[c.ins[1]])
                P.values[wn].const = (w * scale.reshape(-1, 1, 1, 1)).astype(np.float32)
                P.values[bn_] = copy.copy(P.values[c.ins[1]])
                P.values[bn_].const = ((b0 - mu) * scale + be).astype(np.float32)
                P.values[bn_].shape = (w.shape[0],)
                c.ins[1] = wn
                c.p.bias = bn_
                c.outs[0] = n.outs[0]
                continue
        keep.append(n)
    P.nodes = keep
    return P


class OracleSession:
    def __init__(self, plan, keep_all: bool = False):
        plan = fold_batchnorm(plan)
        self.plan = plan
        self.keep_all = keep_all
        self._packs = {}

    def _conv_plan(self, n):
        kp = self._packs.get(n.name)
        if kp is None:
            p = n.p
            w = self.plan.values[n.ins[1]].const
            b = self.plan.values[p.bias].const if p.bias else None
            kp = O.ConvPlan(w, b, group=p.group, strides=p.strides)
            self._packs[n.name] = kp
        return kp

    def _gemm_plan(self, n):
        kp = self._packs.get(n.name)
        if kp is None:
            w = self.plan.values[n.ins[1]].const
            b = self.plan.values[n.p.bias].const if n.p.bias else None
            kp = O.GemmPlan(w, b, trans_b=n.p.trans_b)
            self._packs[n.name] = kp
        return kp

    def run(self, feeds: dict) -> dict:
        P = self.plan
        env = {}
        for name, v in P.values.items():
            if v.is_const:
                env[name] = v.const
        for name in (P.inputs or [P.input]):
            a = np.ascontiguousarray(feeds[name], np.uint8 if P.values[name].dtype == "u8" else np.float32)
            assert a.shape == P.values[name].shape, (name, a.shape)
            env[name] = a
        for n in P.nodes:
            out = self._exec(n, env)
            for o, val in zip(n.outs, out if isinstance(out, tuple) else (out,)):
                # the plan's shapes are authoritative ([N, 1, W, C] and [N, W, C] name the same rows)
                v = P.values[o]
                if v.layout != "nchw" and val.shape != v.shape and val.size == int(np.prod(v.shape)):
                    val = val.reshape(v.shape)
                env[o] = val
        return env if self.keep_all else {P.output: env[P.output]}

    def _nhwc(self, name, env):
        v = self.plan.values[name]
        a = env[name]
        if v.layout == "nchw":  # boundary relayout into the NHWC plan
            a = np.ascontiguousarray(a.transpose(0, 2, 3, 1))
        return a

    def _exec(self, n, env):
        P = self.plan
        op, p = n.op, n.p
        if op == "Conv":
            x = self._nhwc(n.ins[0], env)
            kp = self._conv_plan(n)
            add = self._nhwc(p.add, env) if p.add else None
            if p.pool is not None:
                return O.conv_pool(x, kp, pads=p.pads, act=p.act, pool_relu=p.pool.fuse_relu)
            return O.conv(x, kp, strides=p.strides, pads=p.pads, act=p.act, add=add)
        if op == "ConvTranspose":
            w = P.values[n.ins[1]].const
            b = P.values[p.bias].const if p.bias else None
            return O.convt(env[n.ins[0]], w, b, act=p.act)
        if op == "ChannelGate":
            x = env[n.ins[0]]
            return O.channel_gate(x, P.values[n.ins[1]].const, P.values[p.b1].const if p.b1 else None,
                                  P.values[n.ins[2]].const, P.values[p.b2].const if p.b2 else None,
                                  act1_relu=p.act1 == "relu", hard=p.hard, alpha=p.alpha, beta=p.beta, offset=p.offset)
        if op == "Elementwise":
            a, b = env[n.ins[0]], env[n.ins[1]]
            relu = p.act == "relu"
            if a.shape == b.shape:
                y = O.binary(a, b, p.op, relu)
            elif b.ndim == 2 and a.ndim == 4 and b.shape == (a.shape[0], a.shape[3]):
                y = O.channel_broadcast(a, b, p.op, relu=relu)
            else:
                # numpy broadcast (Ops.Elementwise's general case)
                return O.binary_bcast(a, b, p.op, p.act)
            if p.act not in ("none", "relu"):
                y = O.act(y, p.act)
            return y
        if op == "BatchNorm":
            # not folded: x * s + t (GraphCompiler.EmitBatchNorm), two fp32 elementwise passes
            g, be = P.values[p.gamma].const, P.values[p.beta].const
            mu, var = P.values[p.mean].const, P.values[p.var].const
            s = (g / np.sqrt(var + np.float32(p.eps), dtype=np.float32)).astype(np.float32)
            t = (be - mu * s).astype(np.float32)
            return O.binary_bcast(O.binary_bcast(env[n.ins[0]], s, "mul"), t, "add")
        if op == "SafeDiv":
            return O.safe_div(env[n.ins[0]], env[n.ins[1]], p.eps, p.lo, p.hi)
        if op == "ChannelShift":
            return O.channel_shift(env[n.ins[0]], p.axis, p.group_ends, p.offsets)
        if op == "UpHead":
            oc = P.values[n.outs[0]].shape[3]
            w = P.values[n.ins[2]].const.reshape(oc, -1)
            b = P.values[p.bias].const if p.bias else None
            return O.uphead(env[n.ins[0]], env[n.ins[1]], w, b, p.scales[0], p.scales[1], p.resize_relu, p.skip_relu,
                            p.act)
        if op == "MatMul":
            return O.matmul_bcast(env[n.ins[0]], env[n.ins[1]])
        if op == "ResizeNearest":
            add = env[n.ins[1]] if len(n.ins) > 1 else None
            return O.resize_nearest(env[n.ins[0]], p.scales, add=add, add_relu=p.add_relu)
        if op == "Concat":
            return O.concat_channels([env[v] for v in n.ins])
        if op == "MaxPool":
            return O.maxpool(env[n.ins[0]], p.kernel, p.strides, p.pads, relu=p.fuse_relu)
        if op == "AvgPool":
            return O.avgpool(env[n.ins[0]], p.kernel, p.strides, p.pads, p.count_include_pad)
        if op == "Gemm" and getattr(p, "ctc", False):
            # CtcProjection.ArgMax: the projection, then the per-row UpdateArgMax walk; packed as the
            # plan's [2, rows] int32 value (indices, then probabilities' fp32 bits)
            a = env[n.ins[0]]
            logits = O.gemm(a.reshape(-1, a.shape[-1]), self._gemm_plan(n))
            idx, prob = O.ctc_argmax(logits)
            return np.stack([idx.astype(np.int32), prob.astype(np.float32).view(np.int32)])
        if op == "Gemm":
            y = O.gemm(env[n.ins[0]], self._gemm_plan(n), act=p.act)
            if p.add:
                y = O.binary(y, env[p.add], "add")
            return y
        if op == "LayerNorm":
            return O.layernorm(env[n.ins[0]], P.values[n.ins[1]].const, P.values[n.ins[2]].const, p.eps)
        if op == "Softmax":
            return O.softmax(env[n.ins[0]])
        if op == "Attention":
            # CPU plans run the unfused MatMul -> scale -> Softmax -> MatMul (attention is fused on GPU
            # plans only, src/Engine/GraphCompiler.cs:614-770)
            qkv = env[n.ins[0]]
            nb, t = qkv.shape[0], qkv.shape[1]
            q, k, v = (np.ascontiguousarray(qkv.reshape(nb, t, 3, p.heads, p.head_dim)[:, :, i].transpose(0, 2, 1, 3))
                       for i in range(3))
            s = O.matmul(q, np.ascontiguousarray(k.transpose(0, 1, 3, 2)))
            s = O.binary(s, np.full(s.shape, p.scale, np.float32), "mul")
            y = O.matmul(O.softmax(s), v)
            return np.ascontiguousarray(y.transpose(0, 2, 1, 3)).reshape(nb, t, p.heads * p.head_dim)
        if op == "Act":
            return O.act(env[n.ins[0]], p)
        if op == "ImageToTensor":
            # img2nhwc.comp (src/Backends/Vulkan/Shaders/img2nhwc.comp:24-37): replicate padding,
            # byte -> lut[c][byte], channel 0 from byte 2 when swapped; here fp32 NCHW
            img = env[n.ins[0]]
            lut = P.values[p.lut].const.reshape(3, 256)
            out = P.values[n.outs[0]]
            nb, _, oh, ow = out.shape
            ih, iw = img.shape[1], img.shape[2]
            sy = np.clip(np.arange(oh) - p.pads[0], 0, ih - 1)
            sx = np.clip(np.arange(ow) - p.pads[1], 0, iw - 1)
            px = img[:, sy][:, :, sx]
            order = (2, 1, 0) if p.swap_rb else (0, 1, 2)
            return np.stack([lut[c][px[..., order[c]]] for c in range(3)], axis=1).astype(np.float32)
        raise NotImplementedError(op)
