"""TinyGPT greedy decoding on the B200 against the float64 host model.

The reference has no TinyGPT; the host model is pinned to TinyGPT composed from
the reference's own kernels on its emulator (prefill and a 4-step greedy decode,
last test below).  Every generated token of every sequence is judged: the host
model is fed the B200's own tokens (teacher forcing), and at every step the
B200's choice must be the host model's argmax, or, only where the host's top-2
logits lie within TIE of each other (a near tie, where fp32 rounding may pick
the other token), a token whose host logit is within TIE of the maximum.  So
the decodes may part only at a near tie, and every step after it is still
checked on the B200's own path.  The B200's last logits must agree with the host
model's for the same tokens within LOGIT_ATOL (logits are O(0.3)).
"""

import numpy as np
import pytest

from oracle import tinygpt_ref
from piton_b200 import tinygpt

pytestmark = pytest.mark.gpu
LOGIT_ATOL = 5e-5
TIE = 2 * LOGIT_ATOL


def check(model, weights, prompts, new_tokens):
    toks, logits = model.generate(prompts, new_tokens, return_logits=True)
    plen = prompts.shape[1]
    np.testing.assert_array_equal(toks[:, :plen], prompts)
    lg = tinygpt_ref.teacher_forced_logits(weights, toks, plen)          # [B, new, 65]
    chosen = np.take_along_axis(lg, toks[:, plen:, None].astype(np.int64), 2)[..., 0]
    gap = lg.max(2) - chosen                                              # 0 where the argmax was taken
    top2 = np.sort(lg, 2)[..., -2:]
    clear = (top2[..., 1] - top2[..., 0]) >= TIE
    np.testing.assert_array_equal(toks[:, plen:][clear], lg.argmax(2)[clear])
    assert float(gap.max(initial=0.0)) <= TIE, float(gap.max())
    if new_tokens:
        np.testing.assert_allclose(logits, lg[:, -1], rtol=0, atol=LOGIT_ATOL)
    near = np.where((~clear).any(1), (~clear).argmax(1) + plen, -1)
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
        if new:
            check(model, w, prompts, new)
            continue
        toks, logits = model.generate(prompts, new, return_logits=True)
        _, ref_logits, _ = tinygpt_ref.generate(w, prompts, new)
        np.testing.assert_array_equal(toks[:, :plen], prompts)
        np.testing.assert_allclose(logits, ref_logits, rtol=0, atol=LOGIT_ATOL)


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
    gs = goldens("tinygpt_emu_p")
    assert gs
    for g in gs:
        model = tinygpt.TinyGPT(tinygpt.init_weights(g.meta["weight_seed"]))
        prompt = g["prompt"]
        for p in range(1, len(prompt) + 1):
            _, logits = model.generate(prompt[None, :p], 0, return_logits=True)
            np.testing.assert_allclose(logits[0], g["logits"][p - 1], rtol=0, atol=5e-5)
            assert int(np.argmax(logits[0])) == int(np.argmax(g["logits"][p - 1]))


def test_decode_against_reference_kernels_on_the_emulator(cuda):
    """The B200 greedy decode (KV cache, one position per step) against the same decode composed
    from the reference's kernels on its emulator (tests/golden/make_golden.py
    case_tinygpt_decode): a 16-token prompt and 4 greedy steps give the same tokens, and the logits
    that chose each token agree within LOGIT_ATOL."""
    from conftest import goldens
    gs = goldens("tinygpt_emu_decode_")
    assert gs
    for g in gs:
        model = tinygpt.TinyGPT(tinygpt.init_weights(g.meta["weight_seed"]))
        plen, new = g.meta["prompt_len"], g.meta["new_tokens"]
        toks = model.generate(g["prompt"][None], new)
        np.testing.assert_array_equal(toks[0, plen:], g["tokens"])
        for k in range(1, new + 1):
            _, logits = model.generate(g["prompt"][None], k, return_logits=True)
            np.testing.assert_allclose(logits[0], g["logits"][k - 1], rtol=0, atol=LOGIT_ATOL)


@pytest.mark.parametrize("kernel,batch", [("heads", 1), ("heads", 7), ("heads", 37), ("step", 12), ("cluster", 3)])
def test_every_decode_kernel_matches_host_model(cuda, monkeypatch, kernel, batch):
    """Each decode kernel, forced with PITON_B200_TINYGPT_KERNEL, judged step by step against the
    host model: the 16-CTA cluster kernel (small batches), the 4-CTA heads kernel (groups of up
    to 8 sequences per cluster, ragged last group) and the per-position step kernel."""
    monkeypatch.setenv("PITON_B200_TINYGPT_KERNEL", kernel)
    w = tinygpt.init_weights(1)
    model = tinygpt.TinyGPT(w)
    check(model, w, tinygpt.random_prompts(batch, seed=40 + batch), 24)


def test_unknown_decode_kernel_is_rejected(cuda, monkeypatch):
    monkeypatch.setenv("PITON_B200_TINYGPT_KERNEL", "bogus")
    model = tinygpt.TinyGPT(tinygpt.init_weights(0))
    with pytest.raises(ValueError):
        model.generate(tinygpt.random_prompts(2), 2)
