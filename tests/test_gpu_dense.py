"""Dense layer and the digits MLP on the B200 (examples/nn_kernels.py,
examples/digits_model.py).

* dyadic inputs make every product and sum exact, so the dense layer is
  compared bit for bit (tests/test_nn_kernels.py:37-61);
* the fused MLP in QPU rounding mode matches three emulated dense layers bit
  for bit (golden); in IEEE mode the logits stay inside the reference's
  propagated rounding bound (examples/digits_reference.py:14-55) and the
  predicted classes match exactly wherever the top-2 margin exceeds twice
  that bound.
"""

import numpy as np
import pytest

from conftest import golden_ids, goldens
from oracle import oracle as O
from piton_b200 import digits
from piton_b200 import workloads as W
from piton_b200.kernels import dense_layer_kernel, dense_tiles

pytestmark = pytest.mark.gpu
DENSE = goldens("dense_")
MLP = goldens("mlp_")


def run_dense(x, w, bias, relu, add_bias=True, tiles=None, qpu=False):
    m, k = x.shape
    n = w.shape[1]
    bm, bn, bk = tiles or dense_tiles(n)
    grid = ((m + bm - 1) // bm * ((n + bn - 1) // bn),)
    storage = np.full(m * n + 32, np.float32(-1234.5), dtype=np.float32)
    originals = [a.copy() for a in (x, w, bias)]
    dense_layer_kernel[grid](x, w, bias, storage, m, N=n, K=k, BLOCK_SIZE_M=bm, BLOCK_SIZE_N=bn, BLOCK_SIZE_K=bk,
                             GROUP_SIZE_M=1, ADD_BIAS=add_bias, RELU=relu, device="b200", qpu_rounding=qpu)
    for a, original in zip((x, w, bias), originals):
        np.testing.assert_array_equal(a.view(np.uint32), original.view(np.uint32))
    np.testing.assert_array_equal(storage[m * n:], np.float32(-1234.5))
    return storage[:m * n].reshape(m, n)


@pytest.mark.parametrize("g", DENSE, ids=golden_ids(DENSE))
@pytest.mark.parametrize("qpu", [False, True])
def test_dense_dyadic_bit_exact(cuda, g, qpu):
    m = g.meta
    y = run_dense(g["x"], g["w"], g["bias"], m["relu"], m["add_bias"], qpu=qpu)
    np.testing.assert_array_equal(y.view(np.uint32), g["out"].view(np.uint32))


def test_dense_network_64_128_64_16(cuda):
    rng = np.random.default_rng(340)
    x = rng.uniform(-1, 1, (3, 64)).astype(np.float32)
    reference = x.astype(np.float64)
    for index, (k, n) in enumerate(((64, 128), (128, 64), (64, 16))):
        w = rng.normal(0, 0.1, (k, n)).astype(np.float32)
        bias = rng.normal(0, 0.1, n).astype(np.float32)
        relu = index < 2
        x = run_dense(x, w, bias, relu=relu)
        reference = reference @ w.astype(np.float64) + bias.astype(np.float64)
        if relu:
            reference = np.maximum(reference, 0)
        np.testing.assert_allclose(x, reference, rtol=2e-4, atol=2e-5)
    np.testing.assert_array_equal(np.argmax(x[:, :10], axis=1), np.argmax(reference[:, :10], axis=1))


@pytest.mark.parametrize("g", MLP, ids=golden_ids(MLP))
def test_fused_mlp_qpu_mode_matches_emulator(cuda, g):
    model = {k: g[k] for k in ("w1", "b1", "w2", "b2", "w3", "b3")}
    logits, pred = digits.forward(g["images"], model, qpu_rounding=True, return_pred=True)
    np.testing.assert_array_equal(logits.view(np.uint32), g["logits"].view(np.uint32))
    np.testing.assert_array_equal(pred, np.argmax(g["logits"][:, :10], axis=1))


def test_fused_mlp_1797_images(cuda):
    images = W.digits_images(1797, 0)
    model = W.digits_model(0)
    logits, pred = digits.forward(images, model, return_pred=True)
    ref, bound = O.mlp_f64_with_bounds(images, model)
    assert np.all(np.abs(logits - ref) <= bound + 1e-12)
    oracle_logits = O.qpu_mlp(images, model, threads=8)
    top = np.sort(ref[:, :10], axis=1)
    clear = (top[:, -1] - top[:, -2]) > 2 * bound[:, :10].max(axis=1)
    np.testing.assert_array_equal(pred[clear], np.argmax(ref[clear, :10], axis=1))
    np.testing.assert_array_equal(pred[clear], np.argmax(oracle_logits[clear, :10], axis=1))
    assert clear.mean() > 0.9                       # the propagated bound is conservative
    # every image where the B200's argmax differs from the float64 one is a near tie inside the
    # propagated bound: the chosen class's exact logit is within the two classes' bounds of the top
    best = np.argmax(ref[:, :10], axis=1)
    idx = np.arange(len(pred))
    gap = ref[idx, best] - ref[idx, pred]
    assert np.all(gap <= bound[idx, best] + bound[idx, pred] + 1e-12), np.flatnonzero(
        gap > bound[idx, best] + bound[idx, pred])
    assert (pred == np.argmax(oracle_logits[:, :10], axis=1)).mean() > 0.995
    np.testing.assert_array_equal(logits[:, 10:], 0)


def test_mlp_ragged_batches(cuda):
    model = W.digits_model(1)
    for n in (1, 31, 33, 256):
        images = W.digits_images(n, n)
        logits = digits.forward(images, model, qpu_rounding=True)
        np.testing.assert_array_equal(logits.view(np.uint32), O.qpu_mlp(images, model).view(np.uint32))
