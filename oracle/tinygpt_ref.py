"""float64 numpy host model of TinyGPT (TEST INFRASTRUCTURE; the checker of the
B200 decode).

The reference has no TinyGPT (its pieces are dense_layer_kernel,
attn_fwd_kernel, softmax_kernel and a LayerNorm test kernel), so this model
follows the specification in piton_b200/tinygpt.py.  It is pinned at small size
against the same model composed from those reference kernels on the reference's
emulator (tests/golden/tinygpt_emu_*.npz, made by tests/golden/make_golden.py):
the logits of every prompt prefix agree within 2e-5.  It recomputes with a KV
cache exactly like the device kernel: per fed position, every layer, attention
over positions 0..pos.

Greedy decoding is compared token by token; when the float64 top-2 logit
margin at some step is below `tie_margin`, the B200's fp32 arithmetic may
legitimately pick the other token, so `generate` reports the first such step.
"""

from __future__ import annotations

import math

import numpy as np

VOCAB, D, L, H, CTX = 65, 128, 4, 4, 128
HD = D // H


def _ln(x, g, b):
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    return (x - m) / np.sqrt(v + 1e-5) * g + b


def _gelu(x):
    from scipy.special import erf
    return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))


def generate(weights: dict, prompts: np.ndarray, new_tokens: int, tie_margin: float = 1e-4):
    """Returns (tokens [B, P+new], last logits [B, 65], first_near_tie_step [B] (-1: none))."""
    return _decode(weights, np.asarray(prompts), new_tokens, tie_margin, None)


def teacher_forced_logits(weights: dict, tokens: np.ndarray, prompt_len: int) -> np.ndarray:
    """The logits this model gives for every generated step when it is fed `tokens` [B, T]
    (tokens a decode produced, the prompt in [:, :prompt_len]) instead of its own choices:
    [B, T - prompt_len, 65], entry t being the logits at position prompt_len - 1 + t, the ones
    that chose tokens[:, prompt_len + t].  Judges every step of another implementation's greedy
    decode, also after a near tie where the two decodes may part."""
    tokens = np.asarray(tokens)
    steps = []
    _decode(weights, tokens[:, :prompt_len], tokens.shape[1] - prompt_len, 0.0, tokens, steps)
    return np.stack(steps, 1) if steps else np.zeros((tokens.shape[0], 0, VOCAB))


def _decode(weights, prompts, new_tokens, tie_margin, forced, step_logits=None):
    W = {k: np.asarray(v, np.float64) for k, v in weights.items()}
    B, P = prompts.shape
    toks = np.zeros((B, P + new_tokens), np.int64)
    toks[:, :P] = prompts
    kc = np.zeros((L, B, CTX, D))
    vc = np.zeros((L, B, CTX, D))
    near = np.full(B, -1)
    logits = None
    steps = P + new_tokens - 1 if new_tokens > 0 else P
    for pos in range(steps):
        x = W["wte"][toks[:, pos]] + W["wpe"][pos]
        for l in range(L):
            p = f"h{l}."
            h = _ln(x, W[p + "ln1_g"], W[p + "ln1_b"])
            qkv = h @ W[p + "w_qkv"] + W[p + "b_qkv"]
            q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
            kc[l, :, pos] = k
            vc[l, :, pos] = v
            att = np.zeros((B, D))
            for hh in range(H):
                sl = slice(hh * HD, (hh + 1) * HD)
                s = np.einsum("bd,btd->bt", q[:, sl], kc[l, :, :pos + 1, sl]) / math.sqrt(HD)
                s = s - s.max(1, keepdims=True)
                e = np.exp(s)
                att[:, sl] = np.einsum("bt,btd->bd", e / e.sum(1, keepdims=True), vc[l, :, :pos + 1, sl])
            x = x + att @ W[p + "w_o"] + W[p + "b_o"]
            h = _ln(x, W[p + "ln2_g"], W[p + "ln2_b"])
            x = x + _gelu(h @ W[p + "w_fc"] + W[p + "b_fc"]) @ W[p + "w_pr"] + W[p + "b_pr"]
        h = _ln(x, W["lnf_g"], W["lnf_b"])
        logits = h @ W["wte"].T
        if pos + 1 >= P and pos + 1 < P + new_tokens:
            top2 = np.sort(logits, 1)[:, -2:]
            tie = (top2[:, 1] - top2[:, 0]) < tie_margin
            near = np.where((near < 0) & tie, pos + 1, near)
            toks[:, pos + 1] = np.argmax(logits, 1) if forced is None else forced[:, pos + 1]
            if step_logits is not None:
                step_logits.append(logits)
    return toks.astype(np.int32), logits, near
