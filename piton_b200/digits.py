"""The 64 -> 128 -> 64 -> 10 digits classifier on the B200.

The reference runs it as three ``dense_layer_kernel`` launches plus a host
argmax (examples/digits_model.py:120-139, tests/test_digits_model.py:119-131);
here one fused kernel (``piton_b200_mlp_f32``) normalises the uint8 images,
runs the three layers with bias and ReLU and takes the argmax of the first
ten logits.  The weights use the reference's model layout: w1 [64,128],
b1 [128], w2 [128,64], b2 [64], w3 [64,16], b3 [16] (six zero padding outputs).
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from .runtime.cuda import _lib
from .runtime.cuda._lib import lib

SHAPES = {"w1": (64, 128), "b1": (128,), "w2": (128, 64), "b2": (64,), "w3": (64, 16), "b3": (16,)}


class DigitsMLP:
    """Device-resident weights and the fused forward."""

    def __init__(self, model: dict, device=None):
        import torch
        self.torch = torch
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.w = {}
        for name, shape in SHAPES.items():
            a = np.ascontiguousarray(model[name], dtype=np.float32)
            if a.shape != shape:
                raise ValueError(f"{name}: shape {a.shape}, expected {shape}")
            self.w[name] = torch.from_numpy(a).to(self.device)

    def forward_device(self, images, logits, pred=None, qpu_rounding=False, n_classes=10):
        """images: CUDA uint8 [M,64] (raw 0..16) or float32 [M,64] in 0..1;
        logits: CUDA float32 [M,16]; pred: CUDA int32 [M] or None."""
        torch = self.torch
        M = images.shape[0]
        if images.shape != (M, 64) or logits.shape != (M, 16) or not images.is_contiguous():
            raise ValueError("images must be contiguous [M,64], logits [M,16]")
        if images.dtype not in (torch.uint8, torch.float32):
            raise TypeError("images must be uint8 intensities or float32")
        if pred is not None and (pred.dtype != torch.int32 or pred.numel() < M):
            raise ValueError("pred must be int32 [M]")
        w = self.w
        a = _lib.MlpArgs(images.data_ptr(), w["w1"].data_ptr(), w["b1"].data_ptr(), w["w2"].data_ptr(),
                         w["b2"].data_ptr(), w["w3"].data_ptr(), w["b3"].data_ptr(), logits.data_ptr(),
                         pred.data_ptr() if pred is not None else 0, M, int(images.dtype == torch.uint8),
                         n_classes, _lib.QPU_ROUNDING if qpu_rounding else 0, 0)
        stream = C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(lib().piton_b200_mlp_f32(C.byref(a), stream), "mlp")

    def __call__(self, images, qpu_rounding=False, return_pred=False):
        torch = self.torch
        images = np.asarray(images)
        if np.issubdtype(images.dtype, np.integer):
            if images.size and (images.min() < 0 or images.max() > 16):
                raise ValueError("raw digit pixels must be in 0..16")
            t = torch.from_numpy(np.ascontiguousarray(images, dtype=np.uint8)).to(self.device)
        else:
            t = torch.from_numpy(np.ascontiguousarray(images, dtype=np.float32)).to(self.device)
        M = images.shape[0]
        logits = torch.empty(M, 16, dtype=torch.float32, device=self.device)
        pred = torch.empty(M, dtype=torch.int32, device=self.device)
        self.forward_device(t, logits, pred, qpu_rounding)
        out = logits.cpu().numpy()
        return (out, pred.cpu().numpy()) if return_pred else out


def forward(images, model, qpu_rounding=False, return_pred=False):
    """All 16 logits (and optionally the predicted class) for [M,64] images."""
    return DigitsMLP(model)(images, qpu_rounding=qpu_rounding, return_pred=return_pred)


def predict(images, model):
    return forward(images, model, return_pred=True)[1]
