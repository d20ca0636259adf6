"""Resampling / concatenation tensor ops and the operand-staged direct
convolutions (test infrastructure only: the checker of the GPU kernels).

* downsample2x -- rdv/shaders/tensors/downsample2x_tensor_op.h:1-45:
  ((x00 + x01) + x10) + x11, times 0.25, every step rounded to float32;
* upsample2x -- rdv/shaders/tensors/upsample2x_tensor_op.h:1-33 (copy);
* concat -- rdv/shaders/tensors/concat_tensor_op.h:1-35 (copy);
  the three are pinned bit for bit to the reference's own shader functions
  by tests/golden/resample.npz (tests/golden/make_golden.py);
* conv2d_staged -- the reference's tensor-core direct convolutions
  (Conv2DTensorOpFast / Simple / Simple3x3 / Window3x3, rdv/domain/nn.py:608-999):
  x and w rounded to float16 (or bfloat16), products and sums in float64,
  + bias. Their parity is against this restatement within BASELINE's
  float16 tolerance: the reference's cooperative-matrix accumulation order
  is not specified.
"""
from __future__ import annotations

import numpy as np

from .mlp import stage
from .winograd import conv2d_direct


def downsample2x(x: np.ndarray, h: int, w: int) -> np.ndarray:
    """x [h*w, c] float32 -> [(h/2)*(w/2), c]."""
    c = x.shape[1]
    r = np.asarray(x, dtype=np.float32).reshape(h, w, c)
    s = (r[0::2, 0::2] + r[0::2, 1::2]).astype(np.float32)
    s = (s + r[1::2, 0::2]).astype(np.float32)
    s = (s + r[1::2, 1::2]).astype(np.float32)
    return (s * np.float32(0.25)).astype(np.float32).reshape(-1, c)


def upsample2x(x: np.ndarray, h: int, w: int) -> np.ndarray:
    """x [h*w, c] -> [(2h)*(2w), c], nearest neighbour."""
    c = x.shape[1]
    r = np.asarray(x, dtype=np.float32).reshape(h, w, c)
    return np.repeat(np.repeat(r, 2, axis=0), 2, axis=1).reshape(-1, c)


def concat(x1: np.ndarray, x2: np.ndarray) -> np.ndarray:
    return np.concatenate([np.asarray(x1, dtype=np.float32), np.asarray(x2, dtype=np.float32)], axis=1)


def conv2d_staged(x_hw_c: np.ndarray, w_hwio: np.ndarray, bias, h: int, w: int, math: str = "f16") -> np.ndarray:
    """x [h*w, cin] -> [h*w, cout]; operands staged to `math`, float64 sums."""
    cin = x_hw_c.shape[1]
    xs = stage(np.asarray(x_hw_c, dtype=np.float32), math).reshape(1, h, w, cin)
    ws = stage(np.asarray(w_hwio, dtype=np.float32), math)
    return conv2d_direct(xs, ws, bias).reshape(h * w, -1)
