"""TinyGPT: a character-level decoder generated greedily on the B200.

The reference has no such model (it has the pieces: dense layers, causal
attention, softmax, a LayerNorm test kernel); this module fixes its
specification from the benchmark configuration and runs it through the fused
``piton_b200_tinygpt_generate`` entry point:

* vocab 65, d_model 128, 4 layers, 4 heads (head dim 32), context 128;
* learned token and position embeddings; the output head is the token
  embedding transposed (tied);
* pre-LayerNorm blocks: x += attn(LN1(x)); x += proj(GELU(fc(LN2(x)))),
  LayerNorm with gain and bias (eps 1e-5, biased variance), exact (erf) GELU,
  4x MLP (128 -> 512 -> 128), causal softmax attention scaled by 1/sqrt(32);
* a final LayerNorm before the tied head; greedy decoding takes the first
  maximum of the 65 logits;
* initialisation from one seed: every matrix ~ N(0, 0.02) drawn in the order
  wte, wpe, then per layer w_qkv, w_o, w_fc, w_pr; biases 0; LayerNorm gains 1,
  biases 0.

Prompts are 16 tokens drawn uniformly from 0..64; 64 new tokens are generated.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from .runtime.cuda import _lib
from .runtime.cuda._lib import lib

VOCAB, D_MODEL, N_LAYER, N_HEAD, CTX = 65, 128, 4, 4, 128
FFN = 4 * D_MODEL
PROMPT_LEN, NEW_TOKENS = 16, 64

LAYER_TENSORS = [("ln1_g", (D_MODEL,)), ("ln1_b", (D_MODEL,)), ("w_qkv", (D_MODEL, 3 * D_MODEL)),
                 ("b_qkv", (3 * D_MODEL,)), ("w_o", (D_MODEL, D_MODEL)), ("b_o", (D_MODEL,)),
                 ("ln2_g", (D_MODEL,)), ("ln2_b", (D_MODEL,)), ("w_fc", (D_MODEL, FFN)), ("b_fc", (FFN,)),
                 ("w_pr", (FFN, D_MODEL)), ("b_pr", (D_MODEL,))]


def init_weights(seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    w = {"wte": rng.normal(0.0, 0.02, (VOCAB, D_MODEL)).astype(np.float32),
         "wpe": rng.normal(0.0, 0.02, (CTX, D_MODEL)).astype(np.float32)}
    for layer in range(N_LAYER):
        for name, shape in LAYER_TENSORS:
            key = f"h{layer}.{name}"
            if name.startswith("w_"):
                w[key] = rng.normal(0.0, 0.02, shape).astype(np.float32)
            elif name.endswith("_g"):
                w[key] = np.ones(shape, np.float32)
            else:
                w[key] = np.zeros(shape, np.float32)
    w["lnf_g"] = np.ones(D_MODEL, np.float32)
    w["lnf_b"] = np.zeros(D_MODEL, np.float32)
    return w


def pack(weights: dict) -> np.ndarray:
    """Weights in the packed layout libpiton_b200 reads (csrc/tinygpt.cu)."""
    parts = [weights["wte"], weights["wpe"]]
    for layer in range(N_LAYER):
        parts += [weights[f"h{layer}.{name}"] for name, _ in LAYER_TENSORS]
    parts += [weights["lnf_g"], weights["lnf_b"]]
    flat = np.concatenate([np.ascontiguousarray(p, np.float32).ravel() for p in parts])
    return flat


def random_prompts(batch: int, seed: int = 0, length: int = PROMPT_LEN) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(0, VOCAB, (batch, length)).astype(np.int32)


class TinyGPT:
    """Device-resident packed weights; ``generate`` runs the whole greedy decode on the GPU."""

    def __init__(self, weights: dict, device=None):
        import torch
        self.torch = torch
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        flat = pack(weights)
        expect = lib().piton_b200_tinygpt_weight_floats()
        if flat.size != expect:
            raise ValueError(f"packed weights have {flat.size} floats, the kernel expects {expect}")
        self.w = torch.from_numpy(flat).to(self.device)
        self._kv = None

    def kv_cache(self, batch: int):
        torch = self.torch
        need = N_LAYER * 2 * batch * CTX * D_MODEL
        if self._kv is None or self._kv.numel() < need:
            self._kv = torch.empty(need, dtype=torch.float32, device=self.device)
        return self._kv

    def generate_device(self, tokens, prompt_len: int, new_tokens: int, logits=None, stream=None,
                        graph: bool = False):
        """tokens: CUDA int32 [batch, 128] with the prompts in [:, :prompt_len]; fills
        [:, prompt_len:prompt_len + new_tokens] on the stream (asynchronous).  graph=True
        replays a CUDA graph of the decode's launches, captured by the library the first
        time these buffers and sizes are seen."""
        torch = self.torch
        if tokens.dtype != torch.int32 or tokens.dim() != 2 or tokens.shape[1] != CTX or not tokens.is_contiguous():
            raise ValueError("tokens must be a contiguous CUDA int32 tensor [batch, 128]")
        batch = tokens.shape[0]
        kv = self.kv_cache(batch)
        a = _lib.TinyGPTArgs(self.w.data_ptr(), kv.data_ptr(), tokens.data_ptr(),
                             logits.data_ptr() if logits is not None else 0, batch, prompt_len, new_tokens,
                             VOCAB, D_MODEL, N_LAYER, N_HEAD, CTX, _lib.CUDA_GRAPH if graph else 0)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        _lib.check(lib().piton_b200_tinygpt_generate(C.byref(a), C.c_void_p(s.cuda_stream)), "tinygpt")

    def generate(self, prompts: np.ndarray, new_tokens: int = NEW_TOKENS, return_logits: bool = False):
        """prompts: int [batch, prompt_len] -> int32 [batch, prompt_len + new_tokens] (and the
        logits of the last fed position)."""
        torch = self.torch
        prompts = np.asarray(prompts)
        if prompts.ndim != 2 or prompts.size and (prompts.min() < 0 or prompts.max() >= VOCAB):
            raise ValueError("prompts must be [batch, length] token ids in 0..64")
        batch, plen = prompts.shape
        buf = np.zeros((batch, CTX), np.int32)
        buf[:, :plen] = prompts
        t = torch.from_numpy(buf).to(self.device)
        logits = torch.empty(batch, VOCAB, dtype=torch.float32, device=self.device) if return_logits else None
        self.generate_device(t, plen, new_tokens, logits)
        out = t.cpu().numpy()[:, :plen + new_tokens]
        return (out, logits.cpu().numpy()) if return_logits else out
