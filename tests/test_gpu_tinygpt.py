"""TinyGPT greedy decoding on the B200 against the float64 host model.

Parity is not pinned by the reference (it has no TinyGPT).  Tokens must match
the host model exactly up to the first step where the float64 top-2 logit
margin is below 1e-4 (a near tie, where fp32 rounding may pick the other
token); the last step's logits must agree within 2e-4 absolute (logits are
O(0.3)) for every sequence whose decode had no near tie.
"""

import numpy as np
import pytest

from oracle import tinygpt_ref
from piton_b200 import tinygpt

pytestmark = pytest.mark.gpu


def check(model, weights, prompts, new_tokens):
    toks, logits = model.generate(prompts, new_tokens, return_logits=True)
    ref, ref_logits, near = tinygpt_ref.generate(weights, prompts, new_tokens)
    plen = prompts.shape[1]
    for b in range(len(prompts)):
        upto = plen + new_tokens if near[b] < 0 else near[b] + 1
        np.testing.assert_array_equal(toks[b, :upto], ref[b, :upto], err_msg=f"sequence {b}")
    clean = near < 0
    assert clean.mean() > 0.9
    np.testing.assert_allclose(logits[clean], ref_logits[clean], rtol=0, atol=2e-4)
    return toks, near


@pytest.mark.parametrize("batch", [1, 5, 256])
def test_greedy_decode_matches_host_model(cuda, batch):
    w = tinygpt.init_weights(0)
    model = tinygpt.TinyGPT(w)
    prompts = tinygpt.random_prompts(batch, seed=batch)
    toks, _ = check(model, w, prompts, tinygpt.NEW_TOKENS)
    assert toks.shape == (batch, 80)


def test_prefill_only_logits_and_short_prompts(cuda):
    w = tinygpt.init_weights(3)
    model = tinygpt.TinyGPT(w)
    for plen, new in ((16, 0), (1, 5), (3, 1)):
        prompts = tinygpt.random_prompts(7, seed=plen, length=plen)
        toks, logits = model.generate(prompts, new, return_logits=True)
        ref, ref_logits, near = tinygpt_ref.generate(w, prompts, new)
        np.testing.assert_array_equal(toks[:, :plen], prompts)
        np.testing.assert_allclose(logits[near < 0], ref_logits[near < 0], rtol=0, atol=2e-4)


def test_context_overflow_is_rejected(cuda):
    model = tinygpt.TinyGPT(tinygpt.init_weights(0))
    with pytest.raises(ValueError):
        model.generate(tinygpt.random_prompts(2, length=100), 29)


def test_batch_rows_are_independent(cuda):
    # a sequence decodes the same alone and inside a batch (no cross-talk between CTAs / cache rows)
    w = tinygpt.init_weights(4)
    model = tinygpt.TinyGPT(w)
    prompts = tinygpt.random_prompts(9, seed=11)
    together = model.generate(prompts, 20)
    alone = np.concatenate([model.generate(prompts[i:i + 1], 20) for i in range(9)])
    np.testing.assert_array_equal(together, alone)


def test_logits_against_reference_kernels_on_the_emulator(cuda):
    """The B200 decode against TinyGPT composed from the reference's own kernels on its
    emulator (tests/golden/make_golden.py case_tinygpt): the logits after every prefix of the
    prompt within 5e-5, the same greedy token."""
    from conftest import goldens
    gs = goldens("tinygpt_emu_")
    assert gs
    for g in gs:
        model = tinygpt.TinyGPT(tinygpt.init_weights(g.meta["weight_seed"]))
        prompt = g["prompt"]
        for p in range(1, len(prompt) + 1):
            _, logits = model.generate(prompt[None, :p], 0, return_logits=True)
            np.testing.assert_allclose(logits[0], g["logits"][p - 1], rtol=0, atol=5e-5)
            assert int(np.argmax(logits[0])) == int(np.argmax(g["logits"][p - 1]))
