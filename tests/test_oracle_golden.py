"""The CPU oracle against the reference emulator's golden outputs (CPU only).

The fixtures under tests/golden were produced by running PIton's own strict
QPU emulator (tests/golden/make_golden.py).  The oracle restates the
emulator's arithmetic and must reproduce every fixture bit for bit; this pins
it before it checks the B200 kernels.
"""

import numpy as np
import pytest

from conftest import golden_ids, goldens, sha256
from oracle import oracle as O
from piton_b200 import workloads as W

ADD = goldens("add_")
SOFTMAX = goldens("softmax_")
MATMUL = goldens("matmul_")
DENSE = goldens("dense_")
MLP = goldens("mlp_")
ATTN = goldens("attn_")


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("g", ADD, ids=golden_ids(ADD))
def test_add(g):
    m = g.meta
    x, y = W.vector_add(m["n"], m["seed"])
    assert sha256(x) == m["sha_x"] and sha256(y) == m["sha_y"], "input recipe changed"
    out = O.qpu_add(x, y)
    assert sha256(out) == m["sha_out"]
    if "out" in g:
        np.testing.assert_array_equal(bits(out), bits(g["out"]))
    else:
        np.testing.assert_array_equal(bits(out[g["sample_idx"]]), bits(g["sample"]))


@pytest.mark.parametrize("g", SOFTMAX, ids=golden_ids(SOFTMAX))
def test_softmax(g):
    m = g.meta
    x = W.softmax_input(1823 if m["n"] == 781 else m["m"], m["n"], m["seed"])[:m["m"]]
    assert sha256(x) == m["sha_x"]
    y = O.qpu_softmax(x, m["block"])
    assert sha256(y) == m["sha_out"]


@pytest.mark.parametrize("g", MATMUL, ids=golden_ids(MATMUL))
def test_matmul(g):
    m = g.meta
    if m["M"] * m["N"] * m["K"] > 256 ** 3:
        pytest.skip("large fixtures are checked by test_matmul_large")
    a, b = W.matmul_inputs(m["M"], m["N"], m["K"], m["seed"])
    assert sha256(a) == m["sha_a"] and sha256(b) == m["sha_b"]
    c = O.qpu_matmul(a, b, threads=4)
    assert sha256(c) == m["sha_c"]


@pytest.mark.parametrize("g", [g for g in MATMUL if g.meta["M"] * g.meta["N"] * g.meta["K"] > 256 ** 3],
                         ids=golden_ids([g for g in MATMUL if g.meta["M"] * g.meta["N"] * g.meta["K"] > 256 ** 3]))
def test_matmul_large(g):
    m = g.meta
    a, b = W.matmul_inputs(m["M"], m["N"], m["K"], m["seed"])
    c = O.qpu_matmul(a, b, threads=8)
    np.testing.assert_array_equal(bits(c[g["rows"]]), bits(g["sample"]))
    assert sha256(c) == m["sha_c"]


@pytest.mark.parametrize("g", DENSE, ids=golden_ids(DENSE))
def test_dense_dyadic(g):
    m = g.meta
    y = O.qpu_dense(g["x"], g["w"], g["bias"], m["add_bias"], m["relu"])
    np.testing.assert_array_equal(bits(y), bits(g["out"]))
    # dyadic inputs: every product and sum is exact, so numpy agrees too
    ref = g["x"] @ g["w"]
    if m["add_bias"]:
        ref = ref + g["bias"]
    if m["relu"]:
        ref = np.maximum(ref, np.float32(0))
    np.testing.assert_array_equal(y, ref)


@pytest.mark.parametrize("g", MLP, ids=golden_ids(MLP))
def test_mlp(g):
    model = {k: g[k] for k in ("w1", "b1", "w2", "b2", "w3", "b3")}
    np.testing.assert_array_equal(g["images"], W.digits_images(g.meta["m"], g.meta["seed"]))
    y = O.qpu_mlp(g["images"], model)
    np.testing.assert_array_equal(bits(y), bits(g["logits"]))


@pytest.mark.parametrize("g", ATTN, ids=golden_ids(ATTN))
def test_attention(g):
    m = g.meta
    q, k, v = W.attention_inputs(m["heads"], m["n"], m["d"], m["seed"])
    o = O.qpu_attention(q, k, v, m["causal"], m["block"][0], m["block"][1])
    assert sha256(o) == m["sha_out"]
    if "out" in g:
        np.testing.assert_array_equal(bits(o), bits(g["out"]))
    else:
        np.testing.assert_array_equal(bits(o[:2]), bits(g["out_first_heads"]))


IDIV = goldens("idiv_")
LIFE = goldens("life_")
ELEM = goldens("elem_")


@pytest.mark.parametrize("g", IDIV, ids=golden_ids(IDIV))
def test_idiv(g):
    q, r = O.idiv_c(g["x"], g["y"], g.meta["signed"])
    np.testing.assert_array_equal(q, g["q"].view(np.uint32))
    np.testing.assert_array_equal(r, g["r"].view(np.uint32))


@pytest.mark.parametrize("g", LIFE, ids=golden_ids(LIFE))
def test_life(g):
    if g.meta["kernel"] == "bits":
        n_cols = g.meta["shape"][1]
        want = O.pack_bits(O.life_step(O.unpack_bits(g["src"], n_cols)))
        np.testing.assert_array_equal(want, g["dst"])
    else:
        np.testing.assert_array_equal(O.life_step(g["src"]), g["dst"])


@pytest.mark.parametrize("g", ELEM, ids=golden_ids(ELEM))
def test_elementwise_qpu(g):
    x, y = g["x"], g["y"]
    if g.meta["op"] == "elem_mul":
        got = O.qpu_binary("fmul", x, y)
    elif g.meta["op"] == "elem_fma":
        got = O.qpu_fma(x, y, 0.3)
    else:
        got = O.qpu_scaled_relu(x, 0.5)
    np.testing.assert_array_equal(bits(got), bits(g["out"]))


TGPT = goldens("tinygpt_emu_p")


@pytest.mark.parametrize("g", TGPT, ids=golden_ids(TGPT))
def test_tinygpt_host_model_against_reference_kernels(g):
    """The float64 TinyGPT host model against the model composed from the reference's own
    kernels on its emulator (dense_layer_kernel, attn_fwd_kernel, layernorm_kernel): the
    logits of every prompt prefix within 2e-5 (they are O(0.5); the emulator rounds toward
    zero), the same greedy token."""
    from oracle import tinygpt_ref
    from piton_b200 import tinygpt
    w = tinygpt.init_weights(g.meta["weight_seed"])
    prompt = g["prompt"]
    for p in range(1, len(prompt) + 1):
        _, logits, _ = tinygpt_ref.generate(w, prompt[None, :p], 0)
        np.testing.assert_allclose(logits[0], g["logits"][p - 1], rtol=0, atol=2e-5)
        assert int(np.argmax(logits[0])) == int(np.argmax(g["logits"][p - 1]))
