"""Every batch size BASELINE.json lists, and the benchmarked det N=256, on the CUDA backend.

The oracle is too slow for whole batches of 640x640 images, so parity at a large batch is shown
through two size-independent properties (the reference's kernels are batch-native, every image
computed independently: src/Engine/Session.cs:339-342):
  * each checked image of the big batch is bit-identical to the same image run alone at N=1, whose
    parity against the oracle is checked by tests/test_gpu_graphs.py; and
  * at the benchmarked configuration (det, N=256) one image in the middle of the batch is also
    compared with the oracle directly (rel-L2 <= 2e-3, max-abs <= 1e-2 * max|ref|).
Inputs are seeded U[0,1) tensors of each config's input shape (numpy PCG64: the SplitMix64 stream
of simdonnx_b200.synth takes minutes at N=256 on the host).
"""
import numpy as np
import pytest

from tests.parity import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def _input(plan, seed):
    shape = plan.values[plan.input].shape
    return np.random.default_rng(seed).random(shape, dtype=np.float32)


def _batch_vs_single(builder, batch, idxs, seed):
    from simdonnx_b200.session import CudaInferenceSession
    big = builder(batch=batch)
    x = _input(big, seed)
    sb = CudaInferenceSession(big)
    out = sb.run({big.input: x})
    again = sb.run({big.input: x}, copy=False)
    assert np.array_equal(out, again), f"batch {batch}: two runs of the same input differ"
    sb.close()
    one = builder(batch=1)
    s1 = CudaInferenceSession(one)
    for i in idxs:
        o1 = s1.run({one.input: x[i:i + 1]})
        assert np.array_equal(o1[0], out[i]), f"image {i} of batch {batch} differs from its N=1 run"
    s1.close()
    return x, out


def test_det_benchmark_batch_256():
    """C5, the bench's exact session (det, N=256 per GPU): images 0, 137 and 255 bit-identical to
    their N=1 runs, and image 137 within the parity bar of the oracle."""
    from oracle.runner import OracleSession
    from simdonnx_b200 import configs
    x, out = _batch_vs_single(configs.build_det, 256, (0, 137, 255), seed=256)
    one = configs.build_det(batch=1)
    ref = OracleSession(one).run({one.input: x[137:138]})[one.output]
    assert_close(out[137:138], ref, "det N=256, image 137 vs oracle")


@pytest.mark.parametrize("batch,idxs", [(8, (0, 7)), (32, (0, 13, 31))])
def test_det_listed_batches(batch, idxs):
    from simdonnx_b200 import configs
    _batch_vs_single(configs.build_det, batch, idxs, seed=batch)


@pytest.mark.parametrize("batch,idxs", [(16, (0, 9, 15)), (64, (0, 41, 63))])
def test_rec_listed_batches(batch, idxs):
    from simdonnx_b200 import configs
    _batch_vs_single(configs.build_rec, batch, idxs, seed=100 + batch)


@pytest.mark.parametrize("batch,idxs", [(4, (0, 3)), (16, (0, 6, 15))])
def test_unet_listed_batches(batch, idxs):
    from simdonnx_b200 import configs
    _batch_vs_single(configs.build_unet, batch, idxs, seed=200 + batch)


def test_rec_batch_64_image_vs_oracle():
    """C3 at its largest listed batch: one image against the oracle (the CTC logits)."""
    from oracle.runner import OracleSession
    from simdonnx_b200 import configs
    from simdonnx_b200.session import CudaInferenceSession
    big = configs.build_rec(batch=64)
    x = _input(big, 7)
    s = CudaInferenceSession(big)
    out = s.run({big.input: x})
    s.close()
    one = configs.build_rec(batch=1)
    ref = OracleSession(one).run({one.input: x[50:51]})[one.output]
    assert_close(out[50:51], ref, "rec N=64, image 50 vs oracle")
