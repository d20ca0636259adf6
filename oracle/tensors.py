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


def tensor_sampler(t: np.ndarray, x: np.ndarray, clamp: bool = True, aligned: bool = False,
                   linear: bool = True) -> np.ndarray:
    """TensorSampler (rdv/shaders/samplers/tensor_sampler.h, IN = 1..3)
    restated in float32, vectorised over points: t [D0, .., D(IN-1), OUT],
    x [n, IN] -> [n, OUT]. Dimension d is addressed by x[:, IN-1-d]; corner
    weights and the innermost mix(l, r, a) = l (1 - a) + r a in the
    reference's order, out-of-range corners clamped or dropped."""
    t = np.asarray(t, dtype=np.float32)
    x = np.asarray(x, dtype=np.float32)
    IN = t.ndim - 1
    dims = t.shape[:IN]
    one, half = np.float32(1.0), np.float32(0.5)
    ac = np.float32(1.0 if aligned else 0.0)
    lo, alpha, lo_in, hi_in, clo, chi = [], [], [], [], [], []
    for d in range(IN):
        g = np.float32(dims[d])
        idx = ((x[:, IN - 1 - d] * (g - ac) + g) * half - half).astype(np.float32)
        l = np.floor(idx).astype(np.int64)
        h = l + 1
        lo.append(l)
        alpha.append((idx - l.astype(np.float32)).astype(np.float32))
        lo_in.append(clamp | ((l >= 0) & (l < dims[d])))
        hi_in.append(clamp | ((h >= 0) & (h < dims[d])))
        clo.append(np.clip(l, 0, dims[d] - 1))
        chi.append(np.clip(h, 0, dims[d] - 1))
    n = x.shape[0]
    out_dim = t.shape[-1]
    if not linear:
        idx = [lo[d] + (alpha[d] >= half) for d in range(IN)]
        inside = np.ones(n, dtype=bool)
        for d in range(IN):
            inside &= (idx[d] >= 0) & (idx[d] < dims[d])
            idx[d] = np.clip(idx[d], 0, dims[d] - 1)
        y = t[tuple(idx)]
        if not clamp:
            y = np.where(inside[:, None], y, np.float32(0.0))
        return y.astype(np.float32)

    def pair(outer_idx, left_ok, right_ok, rest, y):
        L = IN - 1
        left = t[tuple(outer_idx + [clo[L]])]
        right = t[tuple(outer_idx + [chi[L]])]
        a = alpha[L][:, None]
        r = rest[:, None]
        both = (left * (one - a) + right * a).astype(np.float32)
        add = np.where((left_ok & right_ok)[:, None], (r * both).astype(np.float32),
                       np.where(left_ok[:, None], ((r * (one - a)).astype(np.float32) * left).astype(np.float32),
                                np.where(right_ok[:, None], ((r * a).astype(np.float32) * right).astype(np.float32),
                                         np.float32(0.0))))
        return (y + add).astype(np.float32)

    y = np.zeros((n, out_dim), dtype=np.float32)
    if IN == 1:
        return pair([], lo_in[0], hi_in[0], np.ones(n, np.float32), y)
    if IN == 2:
        y = pair([clo[0]], lo_in[0] & lo_in[1], lo_in[0] & hi_in[1], (one - alpha[0]).astype(np.float32), y)
        return pair([chi[0]], hi_in[0] & lo_in[1], hi_in[0] & hi_in[1], alpha[0], y)
    a0, a1 = alpha[0], alpha[1]
    y = pair([clo[0], clo[1]], lo_in[0] & lo_in[1] & lo_in[2], lo_in[0] & lo_in[1] & hi_in[2],
             ((one - a0) * (one - a1)).astype(np.float32), y)
    y = pair([clo[0], chi[1]], lo_in[0] & hi_in[1] & lo_in[2], lo_in[0] & hi_in[1] & hi_in[2],
             ((one - a0) * a1).astype(np.float32), y)
    y = pair([chi[0], chi[1]], hi_in[0] & hi_in[1] & lo_in[2], hi_in[0] & hi_in[1] & hi_in[2],
             (a0 * a1).astype(np.float32), y)
    return pair([chi[0], clo[1]], hi_in[0] & lo_in[1] & lo_in[2], hi_in[0] & lo_in[1] & hi_in[2],
                (a0 * (one - a1)).astype(np.float32), y)


def grid_sampler(t: np.ndarray, x: np.ndarray, clamp: bool = True, aligned: bool = False,
                 linear: bool = True) -> np.ndarray:
    """GridSampler (rdv/shaders/samplers/grid_sampler.h) over a dense grid
    t [D0, .., D(IN-1), OUT], restated in float32 and vectorised over
    points x [n, IN] -> [n, OUT]. Dimension i takes coordinate x[:, IN-1-i]:
    t_i = x * 0.5 + 0.5; pos = aligned ? t_i (D - 1) : t_i D - 0.5;
    voxel = floor(pos); alpha = pos - voxel. Linear: the 2^IN corners in
    bit-mask order (bit i: +1 along dimension i), weight the product over i
    ascending (from 1) of alpha_i or 1 - alpha_i, out += w * value, corners
    outside skipped unless clamp (clamped then). Nearest: voxel +
    (alpha >= 0.5), outside -> 0 unless clamp."""
    t = np.asarray(t, dtype=np.float32)
    x = np.asarray(x, dtype=np.float32)
    IN = t.ndim - 1
    dims = t.shape[:IN]
    half, one = np.float32(0.5), np.float32(1.0)
    voxel, alpha = [], []
    for i in range(IN):
        ti = (x[:, IN - 1 - i] * half + half).astype(np.float32)
        if aligned:
            pos = (ti * np.float32(dims[i] - 1)).astype(np.float32)
        else:
            pos = ((ti * np.float32(dims[i])).astype(np.float32) - half).astype(np.float32)
        fv = np.floor(pos)
        voxel.append(fv.astype(np.int64))
        alpha.append((pos - fv).astype(np.float32))
    n = x.shape[0]
    out = np.zeros((n, t.shape[-1]), dtype=np.float32)
    if not linear:
        idx, inside = [], np.ones(n, dtype=bool)
        for i in range(IN):
            c = voxel[i] + (alpha[i] >= half)
            if clamp:
                c = np.clip(c, 0, dims[i] - 1)
            inside &= (c >= 0) & (c < dims[i])
            idx.append(np.clip(c, 0, dims[i] - 1))
        y = t[tuple(idx)]
        return (y if clamp else np.where(inside[:, None], y, np.float32(0.0))).astype(np.float32)
    for bits in range(1 << IN):
        idx, inside = [], np.ones(n, dtype=bool)
        w = np.ones(n, dtype=np.float32)
        for i in range(IN):
            up = (bits >> i) & 1
            c = voxel[i] + up
            if clamp:
                c = np.clip(c, 0, dims[i] - 1)
            inside &= (c >= 0) & (c < dims[i])
            idx.append(np.clip(c, 0, dims[i] - 1))
            w = (w * (alpha[i] if up else (one - alpha[i]))).astype(np.float32)
        v = t[tuple(idx)]
        add = (w[:, None] * v).astype(np.float32)
        if not clamp:
            add = np.where(inside[:, None], add, np.float32(0.0))
        out = (out + add).astype(np.float32)
    return out
