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
    # SE products folded into the depthwise convs that read them; tap products stay (two readers)
    fused = [n for n in P.nodes if n.op == "Conv" and getattr(n.p, "in_scale", None)]
    assert len(fused) == 8
    assert sum(n.op == "Elementwise" for n in P.nodes) == 4
    # the FPN concat is written in place by its four producers
    assert not any(n.op == "Concat" for n in P.nodes)
    assert sorted(P.values[v].alias[1] for v in ("fpn.p5u", "fpn.p4u", "fpn.p3u", "fpn.p2")) == [0, 24, 48, 72]


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
