"""Winograd 3x3 convolution oracle (test infrastructure only).

Follows the reference operator Conv2DTensorOpWinograd3x3
(rdv/domain/nn.py:1002-1087):

* filter transform ``U = G g G^T`` in fp32, stored float16 as
  ``[positions][CIN][COUT]`` (nn.py:522-538, G at nn.py:522);
* input transform ``V = B^T d B`` of each zero-padded 4x4 patch in fp32,
  staged float16 (conv2d_tensor_op_winograd3x3.h:59-78, :123-137);
* one CIN-reduction GEMM per domain position with fp32 accumulation
  (:140-161);
* inverse transform ``Y = A^T M A`` in fp32 plus bias (:80-93, :164-174).

F(4x4, 3x3) is a B200 extension (the reference has only F(2x2, 3x3)); its
matrices come from the Toom-Cook construction below, with the same float16
staging of U and V.

Tensors are NHWC; weights ``[3, 3, CIN, COUT]`` (channels-last, the
reference TensorOp layout, nn.py:1060-1061).
"""
from __future__ import annotations

import numpy as np

from .mlp import stage

# F(2x2, 3x3): rows of the reference's own scalar transforms.
G_F23 = np.array([[1, 0, 0], [0.5, 0.5, 0.5], [0.5, -0.5, 0.5], [0, 0, 1]], dtype=np.float64)
BT_F23 = np.array([[1, 0, -1, 0], [0, 1, 1, 0], [0, -1, 1, 0], [0, 1, 0, -1]], dtype=np.float64)
AT_F23 = np.array([[1, 1, 1, 0], [0, 1, -1, -1]], dtype=np.float64)

def toom_cook_matrices(points, m: int, r: int = 3):
    """A^T [m, a], G [a, r], B^T [a, a] of the Toom-Cook construction for
    F(m, r) with a = m + r - 1 evaluation points: the given a-1 finite points
    plus the point at infinity (Lavin & Gray, arXiv:1509.09308, section 4;
    Toom 1963 / Cook 1966). G carries the Lagrange normalisation 1/N_j."""
    a = m + r - 1
    f = np.asarray(points, dtype=np.float64)
    assert f.shape == (a - 1,)
    AT = np.zeros((m, a))
    for j in range(a - 1):
        AT[:, j] = f[j] ** np.arange(m)
    AT[m - 1, a - 1] = 1.0
    G = np.zeros((a, r))
    for j in range(a - 1):
        nj = np.prod([f[j] - f[l] for l in range(a - 1) if l != j])
        G[j, :] = f[j] ** np.arange(r) / nj
    G[a - 1, r - 1] = 1.0
    BT = np.zeros((a, a))
    poly = np.poly(f)  # coefficients of prod (x - f_l), highest power first
    for j in range(a - 1):
        q, _ = np.polydiv(poly, np.array([1.0, -f[j]]))
        BT[j, :a - 1] = q[::-1]
    BT[a - 1, :] = poly[::-1]
    return AT, G, BT


# F(4x4, 3x3) on the points {0, 1, -1, 2, -1/2, inf}: with float16 staging of
# U and V this set keeps the error ~3x lower than the textbook
# {0, 1, -1, 2, -2, inf} (measured on BASELINE config-3-like data), in line
# with the point-selection analysis of Barabasz et al., "Error analysis and
# improving the accuracy of Winograd convolution for deep neural networks"
# (arXiv:1803.10986).
F43_POINTS = (0.0, 1.0, -1.0, 2.0, -0.5)
AT_F43, G_F43, BT_F43 = toom_cook_matrices(F43_POINTS, 4)

VARIANTS = {
    "F2x2": dict(m=2, a=4, G=G_F23, BT=BT_F23, AT=AT_F23),
    "F4x4": dict(m=4, a=6, G=G_F43, BT=BT_F43, AT=AT_F43),
}


def winograd_fwd_f23(d: np.ndarray) -> np.ndarray:
    """Restates _winograd_fwd (conv2d_tensor_op_winograd3x3.h:59-78) on a
    [..., 16] array in float32, same operation order."""
    d = np.asarray(d, dtype=np.float32).reshape(-1, 4, 4)
    m = np.empty_like(d)
    d0, d1, d2, d3 = d[:, 0, :], d[:, 1, :], d[:, 2, :], d[:, 3, :]
    m[:, 0, :] = d0 - d2
    m[:, 1, :] = d1 + d2
    m[:, 2, :] = d2 - d1
    m[:, 3, :] = d1 - d3
    V = np.empty_like(d)
    m0, m1, m2, m3 = m[:, :, 0], m[:, :, 1], m[:, :, 2], m[:, :, 3]
    V[:, :, 0] = m0 - m2
    V[:, :, 1] = m1 + m2
    V[:, :, 2] = m2 - m1
    V[:, :, 3] = m1 - m3
    return V.reshape(-1, 16)


def winograd_inv_f23(M: np.ndarray) -> np.ndarray:
    """Restates _winograd_inv (conv2d_tensor_op_winograd3x3.h:80-93) on a
    [..., 16] array in float32, same operation order."""
    M = np.asarray(M, dtype=np.float32).reshape(-1, 4, 4)
    t = np.empty((M.shape[0], 2, 4), dtype=np.float32)
    t[:, 0, :] = M[:, 0, :] + M[:, 1, :] + M[:, 2, :]
    t[:, 1, :] = M[:, 1, :] - M[:, 2, :] - M[:, 3, :]
    Y = np.empty((M.shape[0], 2, 2), dtype=np.float32)
    Y[:, :, 0] = t[:, :, 0] + t[:, :, 1] + t[:, :, 2]
    Y[:, :, 1] = t[:, :, 1] - t[:, :, 2] - t[:, :, 3]
    return Y.reshape(-1, 4)


def filter_transform(w_33io: np.ndarray, variant: str = "F2x2", staged: bool | None = None) -> np.ndarray:
    """U = G g G^T per (cin, cout) filter, computed in float32 like the
    reference's torch code (nn.py:533-538), with layout [a*a, CIN, COUT];
    float16-staged (as float32 values) when `staged`, by default for F2x2
    only (the F4x4 extension keeps U fp32)."""
    if staged is None:
        staged = variant == "F2x2"
    v = VARIANTS[variant]
    w = np.asarray(w_33io, dtype=np.float32)
    g = np.transpose(w, (2, 3, 0, 1))  # [CIN, COUT, 3, 3]
    G = v["G"].astype(np.float32)
    U = G @ g @ G.T  # [CIN, COUT, a, a]
    a = v["a"]
    cin, cout = g.shape[0], g.shape[1]
    U = np.ascontiguousarray(U.reshape(cin, cout, a * a).transpose(2, 0, 1))
    return stage(U, "f16") if staged else U.astype(np.float32)


def conv3x3_direct(x_nhwc: np.ndarray, w_33io: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """'same' (pad 1, stride 1) 3x3 cross-correlation in float64 -- the
    direct convolution the reference's Conv2DTensorOp computes
    (conv2d_tensor_op.h:21-87: acc = bias; acc += x[h+kh-1, w+kw-1, k] *
    w[kh, kw, k, c])."""
    x = np.asarray(x_nhwc, dtype=np.float64)
    w = np.asarray(w_33io, dtype=np.float64)
    n, H, W, cin = x.shape
    xp = np.zeros((n, H + 2, W + 2, cin), dtype=np.float64)
    xp[:, 1:H + 1, 1:W + 1, :] = x
    y = np.zeros((n, H, W, w.shape[3]), dtype=np.float64) + np.asarray(bias, dtype=np.float64)
    for kh in range(3):
        for kw in range(3):
            y += np.einsum("nhwc,cd->nhwd", xp[:, kh:kh + H, kw:kw + W, :], w[kh, kw])
    return y


def conv2d_direct(x_nhwc: np.ndarray, w_hwio: np.ndarray, bias) -> np.ndarray:
    """'same' (padding KH//2, KW//2), stride-1 KHxKW cross-correlation in
    float64, the general form of Conv2DTensorOp (conv2d_tensor_op.h:21-87:
    pad_h = KH / 2, ih = h + kh - pad_h)."""
    x = np.asarray(x_nhwc, dtype=np.float64)
    w = np.asarray(w_hwio, dtype=np.float64)
    n, H, W, cin = x.shape
    KH, KW, _, cout = w.shape
    ph, pw = KH // 2, KW // 2
    xp = np.zeros((n, H + KH - 1, W + KW - 1, cin), dtype=np.float64)
    xp[:, ph:ph + H, pw:pw + W, :] = x
    y = np.zeros((n, H, W, cout), dtype=np.float64)
    if bias is not None:
        y += np.asarray(bias, dtype=np.float64)
    for kh in range(KH):
        for kw in range(KW):
            y += np.einsum("nhwc,cd->nhwd", xp[:, kh:kh + H, kw:kw + W, :], w[kh, kw])
    return y


def conv3x3_winograd(x_nhwc: np.ndarray, w_33io: np.ndarray, bias: np.ndarray,
                     variant: str = "F2x2", staged: bool = True) -> np.ndarray:
    """Winograd convolution with the reference's precision recipe: U and V
    staged float16 when `staged` (F2x2: V from the reference's fp32 transform
    in its operation order; F4x4: B^T d B in float64, then float32, then
    float16), per-position GEMM and inverse transform in float64, + bias.
    H and W must be multiples of the output tile size m."""
    v = VARIANTS[variant]
    m, a = v["m"], v["a"]
    x = np.asarray(x_nhwc, dtype=np.float32)
    n, H, W, cin = x.shape
    cout = w_33io.shape[3]
    assert H % m == 0 and W % m == 0
    th, tw = H // m, W // m
    # zero-padded input: tile (i, j) covers rows i*m-1 .. i*m+a-2
    pad_hi_h = (th - 1) * m + a - 1 - H
    pad_hi_w = (tw - 1) * m + a - 1 - W
    xp = np.zeros((n, H + 1 + pad_hi_h, W + 1 + pad_hi_w, cin), dtype=np.float64)
    xp[:, 1:H + 1, 1:W + 1, :] = x
    # gather tiles: [n, th, tw, a, a, cin]
    idx_h = (np.arange(th) * m)[:, None] + np.arange(a)[None, :]
    idx_w = (np.arange(tw) * m)[:, None] + np.arange(a)[None, :]
    d = xp[:, idx_h][:, :, :, idx_w]  # n, th, a, tw, a, cin
    d = d.transpose(0, 1, 3, 2, 4, 5)  # n, th, tw, a, a, cin
    BT = v["BT"]
    if staged and variant == "F2x2":
        # the reference's own fp32 transform, in its operation order
        # (_winograd_fwd, conv2d_tensor_op_winograd3x3.h:59-78), then float16
        dc = np.ascontiguousarray(d.astype(np.float32).transpose(0, 1, 2, 5, 3, 4)).reshape(-1, 16)
        V = winograd_fwd_f23(dc).reshape(n, th, tw, cin, 4, 4).transpose(0, 1, 2, 4, 5, 3)
        V = stage(np.ascontiguousarray(V), "f16").astype(np.float64)
    else:
        V = np.einsum("ij,nxyjkc,lk->nxyilc", BT, d, BT)  # B^T d B
        if staged:
            V = stage(V.astype(np.float32), "f16").astype(np.float64)
    if staged:
        U = filter_transform(w_33io, variant, staged=True).astype(np.float64)  # [a*a, cin, cout]
    else:
        g = np.transpose(np.asarray(w_33io, dtype=np.float64), (2, 3, 0, 1))
        U = (v["G"] @ g @ v["G"].T).reshape(cin, cout, a * a).transpose(2, 0, 1)
    U = U.reshape(a, a, cin, cout)
    M = np.einsum("nxyijc,ijcd->nxyijd", V, U)
    AT = v["AT"]
    Y = np.einsum("pi,nxyijd,qj->nxypqd", AT, M, AT)  # n, th, tw, m, m, cout
    Y = Y.transpose(0, 1, 3, 2, 4, 5).reshape(n, H, W, cout)
    return Y + np.asarray(bias, dtype=np.float64)


def conv3x3_winograd_f23_ordered(x_nhwc: np.ndarray, u16: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """Conv2DTensorOpWinograd3x3.forward in the reference's own fp32
    operation order (conv2d_tensor_op_winograd3x3.h:95-177), for the
    reference's shapes (H and W even): per 2x2 tile the zero-padded 4x4
    patch of every input channel, V = _winograd_fwd(patch) in fp32 staged
    float16 (:123-137); per domain position p an fp32 accumulator from 0
    with the float16 products V[c] * U[p][c][o] added in ascending c
    (:140-161; each product is exact in fp32, each sum rounded); the 16
    sums through _winograd_inv in fp32, then + bias (:164-174).

    `u16` is the float16 filter image [16][CIN][COUT] (any float dtype
    holding float16 values). Returns float32 NHWC."""
    x = np.asarray(x_nhwc, dtype=np.float32)
    n, H, W, cin = x.shape
    assert H % 2 == 0 and W % 2 == 0
    U = np.asarray(u16, dtype=np.float32).reshape(16, cin, -1)
    cout = U.shape[2]
    th, tw = H // 2, W // 2
    xp = np.zeros((n, H + 2, W + 2, cin), dtype=np.float32)
    xp[:, 1:H + 1, 1:W + 1, :] = x
    idx_h = (np.arange(th) * 2)[:, None] + np.arange(4)[None, :]
    idx_w = (np.arange(tw) * 2)[:, None] + np.arange(4)[None, :]
    d = xp[:, idx_h][:, :, :, idx_w]                        # n, th, 4, tw, 4, cin
    d = np.ascontiguousarray(d.transpose(0, 1, 3, 5, 2, 4))  # n, th, tw, cin, 4, 4
    V = winograd_fwd_f23(d.reshape(-1, 16)).reshape(n * th * tw, cin, 16)
    V = stage(V, "f16")
    M = np.zeros((n * th * tw, 16, cout), dtype=np.float32)
    for c in range(cin):
        # M[t, p, o] += V[t, c, p] * U[p, c, o], one fp32 rounding per term
        M += V[:, c, :, None] * U[None, :, c, :]
    Mt = np.ascontiguousarray(M.transpose(0, 2, 1)).reshape(-1, 16)   # (tile, o) rows of 16 positions
    Y = winograd_inv_f23(Mt).reshape(n, th, tw, cout, 2, 2)
    Y = Y + np.asarray(bias, dtype=np.float32)[None, None, None, :, None, None]
    return np.ascontiguousarray(Y.transpose(0, 1, 4, 2, 5, 3)).reshape(n, H, W, cout)
