"""Volume ray-march oracle (test infrastructure only).

Pieces restated from the reference:

* pinhole rays -- rdv/shaders/rendering/cameras.h:1-20 with the defaults of
  rdv/domain/rendering.py:24-42 (aspect = W/H, fov = pi/4, no jitter);
* implicit [-1, 1]^3 box slab test -- rdv/shaders/libraries/math_library.h:48-57;
* object-space transform, miss rule and entry clamp --
  rdv/shaders/volumes/raymarching_transmittance.h:1-21 (x <- L (x - O),
  w <- L w with L the inverse of the node's 3x3 part, O its origin);
* fixed-step absorption -- rdv/shaders/volumes/raymarching_transmittance_trait.h:1-14
  (``transmittance_rm``);
* the MLP as a LinearFast chain (float16 staging, fp32 accumulate), see
  oracle/mlp.py.

The emission-absorption compositing of BASELINE config 4 (128 uniform samples,
softplus density, sigmoid colour, front-to-back alpha compositing, RGBA with
A = 1 - T) has no counterpart in the reference; it follows BASELINE.json's
config text and its parity is unpinned.
"""
from __future__ import annotations

import math

import numpy as np

from .mlp import stage


def orbit_pose(frame: int, n_frames: int = 8, radius: float = 3.0, height: float = 0.5) -> np.ndarray:
    """Camera k of the orbit around the unit cube: origin (r cos t, h, r sin t),
    target 0, up +y, as [9] float32 (origin | target | up, the layout
    Cameras expects, rendering.py:37)."""
    t = 2.0 * math.pi * frame / n_frames
    return np.array([radius * math.cos(t), height, radius * math.sin(t), 0, 0, 0, 0, 1, 0], dtype=np.float32)


def _normalize(v):
    return v / np.sqrt(np.sum(v * v, axis=-1, keepdims=True))


def camera_rays(pose9, width: int, height: int, aspect: float | None = None, fov: float | None = None,
                row_begin: int = 0, row_end: int | None = None, jitter_seeds=None, camera_index: int = 0):
    """cameras.h:1-20 for every pixel (rows row_begin..row_end) -> origins
    [R, 3], unit directions [R, 3], float32 arithmetic. With jitter_seeds
    (pixel_jitter, cameras.h:7) the sub-pixel point is (random(), random())
    of the pixel's generator -- the seeds spawned by its flat index
    (camera_index * height + row) * width + column -- instead of the centre."""
    if aspect is None:
        aspect = width / height
    if fov is None:
        fov = math.pi / 4
    row_end = height if row_end is None else row_end
    pose = np.asarray(pose9, dtype=np.float32).reshape(3, 3)
    o, t, n = pose[0], pose[1], pose[2]
    ys, xs = np.meshgrid(np.arange(row_begin, row_end, dtype=np.float32),
                         np.arange(width, dtype=np.float32), indexing="ij")
    if jitter_seeds is None:
        jx = jy = np.float32(0.5)
    else:
        flat = ((camera_index * height + ys.astype(np.int64)) * width + xs.astype(np.int64)).reshape(-1)
        st = random_spawn(jitter_seeds, flat)
        jx = random_draw(st).reshape(xs.shape)
        jy = random_draw(st).reshape(xs.shape)
    px = (xs + jx) / np.float32(width) * np.float32(2.0) - np.float32(1.0)
    py = (ys + jy) / np.float32(height) * np.float32(2.0) - np.float32(1.0)
    sx = px * np.float32(aspect)
    sy = py
    sz = np.float32(1.0 / math.tan(np.float32(fov) * 0.5))
    zaxis = _normalize(t - o)
    xaxis = _normalize(np.cross(n, zaxis))
    yaxis = np.cross(zaxis, xaxis)
    w = xaxis[None, None, :] * sx[..., None] + yaxis[None, None, :] * sy[..., None] + zaxis * sz
    w = _normalize(w).astype(np.float32).reshape(-1, 3)
    origins = np.broadcast_to(o, w.shape).astype(np.float32)
    return origins, w


def ray_box(x: np.ndarray, w: np.ndarray):
    """math_library.h:48-57: slab test against [-1, 1]^3."""
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.float32(1.0) / w
        xc = -x * inv
        s = np.abs(inv)
        tmin = np.max(xc - s, axis=-1)
        tmax = np.min(xc + s, axis=-1)
    return tmin.astype(np.float32), tmax.astype(np.float32)


def softplus(v):
    return np.maximum(v, 0.0) + np.log1p(np.exp(-np.abs(v)))


def sigmoid(v):
    return 1.0 / (1.0 + np.exp(-v))


def mlp_eval(points: np.ndarray, layers) -> np.ndarray:
    """LinearFast chain in float64 on staged operands (see mlp.mlp_forward_f64)."""
    a = points.astype(np.float32)
    for l in layers:
        xs = stage(a, l["math"]).astype(np.float64)
        ws = stage(l["W"], l["math"]).astype(np.float64)
        out = xs @ ws.T + l["b"].astype(np.float64)
        if l["relu"]:
            out = np.maximum(out, 0.0)
        a = out.astype(np.float32)
    return a.astype(np.float64)


def render_emission_absorption(pose9, width: int, height: int, n_samples: int, layers,
                               aspect: float | None = None, fov: float | None = None,
                               row_begin: int = 0, row_end: int | None = None) -> np.ndarray:
    """RGBA [rows, width, 4] float64."""
    row_end = height if row_end is None else row_end
    o, w = camera_rays(pose9, width, height, aspect, fov, row_begin, row_end)
    tmin, tmax = ray_box(o, w)
    hit = ~((tmax <= 0) | (tmin > tmax))
    tmin = np.maximum(tmin, np.float32(0.0))
    rgba = np.zeros((o.shape[0], 4), dtype=np.float64)
    idx = np.nonzero(hit)[0]
    if idx.size:
        oh, wh = o[idx], w[idx]
        t0, t1 = tmin[idx], tmax[idx]
        dt = (t1 - t0) / np.float32(n_samples)
        i = np.arange(n_samples, dtype=np.float32)
        ts = t0[:, None] + (i[None, :] + np.float32(0.5)) * dt[:, None]
        pts = oh[:, None, :] + ts[..., None] * wh[:, None, :]
        out = mlp_eval(pts.reshape(-1, 3).astype(np.float32), layers).reshape(idx.size, n_samples, -1)
        sigma = softplus(out[..., 0])
        rgb = sigmoid(out[..., 1:4])
        tau = sigma * dt.astype(np.float64)[:, None]
        alpha = 1.0 - np.exp(-tau)
        # T_i = prod_{j<i} (1 - alpha_j) = exp(-sum_{j<i} tau_j)
        excl = np.concatenate([np.zeros((idx.size, 1)), np.cumsum(tau, axis=1)[:, :-1]], axis=1)
        T = np.exp(-excl)
        wgt = T * alpha
        rgba[idx, :3] = np.sum(wgt[..., None] * rgb, axis=1)
        rgba[idx, 3] = 1.0 - np.exp(-np.sum(tau, axis=1))
    return rgba.reshape(row_end - row_begin, width, 4)


def transmittance_rm(x, w, d, step_size, density_scale, extinction, safety_cap: int = 4096, counts=None):
    """raymarching_transmittance_trait.h:1-14 vectorised over rays:
    tau accumulates extinction(x) * scale * step while d > 0 (at most
    safety_cap steps); any ray whose tau exceeds 16 returns 0, else exp(-tau).
    `extinction` maps [R, 3] float32 positions to [R] float32. `counts`, if
    given ([R] int64), receives each ray's number of extinction evaluations."""
    x = np.array(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    d = np.array(d, dtype=np.float32)
    tau = np.zeros(x.shape[0], dtype=np.float32)
    dead = np.zeros(x.shape[0], dtype=bool)  # returned 0 early
    step = np.float32(step_size)
    scale = np.float32(density_scale)
    for _ in range(safety_cap):
        live = (d > 0) & ~dead
        if not live.any():
            break
        ext = extinction(x[live]).astype(np.float32) * scale
        if counts is not None:
            counts[live] += 1
        tau[live] = tau[live] + ext * step
        over = np.zeros_like(live)
        over[live] = tau[live] > 16
        dead |= over
        d[live] = d[live] - step
        x[live] = x[live] + step * w[live]
    out = np.exp(-tau.astype(np.float64)).astype(np.float32)
    out[dead] = 0.0
    return out


def object_space(origins, dirs, transform=None):
    """raymarching_transmittance.h:4-9: x <- L (x - O), w <- L w, where
    transform is the node's mat4x3 (12 floats, column-major: three columns of
    the 3x3 part, then the origin O) and L the 3x3 inverse (formed in float64,
    rounded to float32). Each component is ((L_i0 v_0 + L_i1 v_1) + L_i2 v_2)
    with every product and sum rounded to float32."""
    o = np.asarray(origins, dtype=np.float32)
    w = np.asarray(dirs, dtype=np.float32)
    if transform is None:
        return o.copy(), w.copy()
    t = np.asarray(transform, dtype=np.float64).reshape(-1)
    M = t[:9].reshape(3, 3).T  # M[row, col]; the flat layout is column-major
    O = t[9:12].astype(np.float32)
    L = np.linalg.inv(M).astype(np.float32)

    def apply(v):
        out = np.empty_like(v)
        for i in range(3):
            acc = (L[i, 0] * v[:, 0]).astype(np.float32) + (L[i, 1] * v[:, 1]).astype(np.float32)
            out[:, i] = acc.astype(np.float32) + (L[i, 2] * v[:, 2]).astype(np.float32)
        return out

    return apply((o - O).astype(np.float32)), apply(w)


def raymarching_transmittance(origins, dirs, step_size, density_scale, extinction, transform=None,
                              return_evaluations: bool = False):
    """RaymarchingTransmittance.forward (raymarching_transmittance.h:1-21):
    object-space transform, slab test, miss -> 1, entry clamp, then
    transmittance_rm over d = tMax - tMin. With return_evaluations, also the
    total number of extinction evaluations."""
    o, w = object_space(origins, dirs, transform)
    tmin, tmax = ray_box(o, w)
    miss = (tmax <= 0) | (tmin > tmax)
    tmin = np.maximum(tmin, np.float32(0.0))
    x = o + w * tmin[:, None]
    d = tmax - tmin
    out = np.ones(o.shape[0], dtype=np.float32)
    hit = ~miss
    counts = np.zeros(int(hit.sum()), dtype=np.int64)
    if hit.any():
        out[hit] = transmittance_rm(x[hit], w[hit], d[hit], step_size, density_scale, extinction, counts=counts)
    if return_evaluations:
        return out, int(counts.sum())
    return out


def mlp_extinction(layers, input_relu: bool = False):
    """extinction(x) of a Linear / LinearFast chain 3 -> ... -> 1 (layers as
    mlp_eval): [R, 3] float32 -> [R] float32."""
    def ext(p):
        a = np.maximum(p, np.float32(0.0)) if input_relu else p
        return mlp_eval(np.asarray(a, dtype=np.float32), layers)[:, 0].astype(np.float32)
    return ext


# ---------------------------------------------------------------------------
# Ratio tracking (RatiotrackingTransmittance, rdv/domain/volumes.py:144-170)
# ---------------------------------------------------------------------------
# The reference's generator (rdv/shaders/libraries/random_library.h:7-44):
# three Tausworthe components and one LCG, combined by XOR; random() keeps
# the low 23 bits as the mantissa of a float in [1, 2) and subtracts 1. Each
# invocation starts from the dispatch's seeds spawned by its index
# (random_library.h:256-268, index = gl_GlobalInvocationID.x for a Map
# dispatch, i.e. the row). States are [R, 4] uint32 arrays.
_TAUS = ((13, 19, 12, 4294967294), (2, 25, 4, 4294967288), (3, 11, 17, 4294967280))


def random_step(state: np.ndarray) -> None:
    """random_step (random_library.h:13-19), in place."""
    for c, (s1, s2, s3, m) in enumerate(_TAUS):
        z = state[:, c]
        b = ((z << np.uint32(s1)) ^ z) >> np.uint32(s2)
        state[:, c] = ((z & np.uint32(m)) << np.uint32(s3)) ^ b
    state[:, 3] = state[:, 3] * np.uint32(1664525) + np.uint32(1013904223)


def random_spawn(seeds, index: np.ndarray) -> np.ndarray:
    """random_spawn (random_library.h:44-49) of the dispatch seeds for each
    invocation index: the per-thread initial state."""
    s = np.asarray(seeds, dtype=np.uint32).reshape(4)
    i = np.asarray(index, dtype=np.int64).astype(np.uint32)  # two's complement, as GLSL's int -> uint
    with np.errstate(over="ignore"):
        st = np.stack([s[0] ^ (i ^ np.uint32(17)), s[1] ^ (i * np.uint32(123111171)), s[2] ^ (i + np.uint32(11)),
                       s[3] ^ (i ^ (s[0] + np.uint32(13) * s[1]))], axis=1).astype(np.uint32)
    random_step(st)
    return st


def random_draw(state: np.ndarray) -> np.ndarray:
    """random() (random_library.h:27-34) for every row of state, in place."""
    random_step(state)
    v = state[:, 0] ^ state[:, 1] ^ state[:, 2] ^ state[:, 3]
    return ((v & np.uint32(0x007FFFFF)) | np.uint32(0x3F800000)).view(np.float32) - np.float32(1.0)


def voxel_majorant(grid: np.ndarray, x: np.ndarray, w: np.ndarray):
    """VoxelMajorantField.forward (rdv/shaders/volumes/voxel_majorant_field.h):
    grid [D, H, W] (z, y, x) float32; x, w [R, 3] object space. Returns the
    cell's majorant and the distance along w to the cell's exit."""
    dims = np.array([grid.shape[2], grid.shape[1], grid.shape[0]], dtype=np.int64)
    f = dims.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        pos = (x * np.float32(0.5) + np.float32(0.5)) * f
        cell = np.clip(np.trunc(pos).astype(np.int64), 0, dims - 1)
        vs = np.float32(2.0) / f
        bmin = cell.astype(np.float32) * vs - np.float32(1.0)
        bmax = bmin + vs
        t0 = (bmin - x) / w
        t1 = (bmax - x) / w
        # GLSL max(a, b) = a < b ? b : a, min(a, b) = b < a ? b : a
        texit = np.where(t0 < t1, t1, t0)
        dist = np.where(texit[:, 1] < texit[:, 0], texit[:, 1], texit[:, 0])
        dist = np.where(texit[:, 2] < dist, texit[:, 2], dist)
    value = grid[cell[:, 2], cell[:, 1], cell[:, 0]]
    return value.astype(np.float32), dist.astype(np.float32)


def _log_f32(v: np.ndarray) -> np.ndarray:
    """float32 log, correctly rounded (evaluated in float64)."""
    return np.log(v.astype(np.float64)).astype(np.float32)


def transmittance_rt(x, w, d, density_scale, extinction, majorant, state, counts=None):
    """transmittance_rt (rdv/shaders/volumes/ratiotracking_transmittance_trait.h)
    vectorised over rays in lock step, every operation in float32:

        T = 1; for (safety < 1024 while d > 0):
            maj = max(majorant(x, w, dist), 1e-12); dist = max(dist, 1e-6)
            dt = min(dist, -log(1 - random()) / (maj * density_scale))
            d -= dt; x += dt w
            dt >= dist -> next iteration (left the majorant's cell)
            d <= 0 -> return T
            T *= 1 - extinction(x) / maj
            T < 0.05: random() >= T -> return 0, else T = 1 (Russian roulette)
        return T

    `state` ([R, 4] uint32, each ray's generator) advances in place.
    `majorant(x, w)` returns (value, distance); `extinction` maps [n, 3] to [n]."""
    x = np.array(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    d = np.array(d, dtype=np.float32)
    n = x.shape[0]
    T = np.ones(n, dtype=np.float32)
    out = np.ones(n, dtype=np.float32)
    running = np.ones(n, dtype=bool)
    ds = np.float32(density_scale)
    for _ in range(1024):
        ended = running & ~(d > 0)   # the loop condition failed: return T
        out[ended] = T[ended]
        running &= ~ended
        act = np.nonzero(running)[0]
        if act.size == 0:
            break
        maj, dist = majorant(x[act], w[act])
        maj = np.where(maj < np.float32(1e-12), np.float32(1e-12), maj).astype(np.float32)
        dist = np.where(dist < np.float32(1e-6), np.float32(1e-6), dist).astype(np.float32)
        st = state[act]
        u = random_draw(st)
        with np.errstate(divide="ignore"):
            q = (-_log_f32(np.float32(1.0) - u)) / (maj * ds)
        dt = np.where(q < dist, q, dist).astype(np.float32)
        d[act] = d[act] - dt
        x[act] = x[act] + dt[:, None] * w[act]
        moved_out = dt >= dist
        reached = ~moved_out & (d[act] <= 0)
        done = act[reached]
        out[done] = T[done]
        running[done] = False
        coll = ~moved_out & ~reached
        ci = act[coll]
        if ci.size:
            sigma = np.asarray(extinction(x[ci]), dtype=np.float32)
            if counts is not None:
                counts[ci] += 1
            T[ci] = T[ci] * (np.float32(1.0) - sigma / maj[coll])
            low = T[ci] < np.float32(0.05)
            if low.any():
                li = np.nonzero(coll)[0][low]   # positions inside act
                sub = st[li]
                u2 = random_draw(sub)
                st[li] = sub
                rays = act[li]
                killed = u2 >= T[rays]
                out[rays[killed]] = 0.0
                running[rays[killed]] = False
                T[rays[~killed]] = 1.0
        state[act] = st
    out[running] = T[running]
    return out


def ratiotracking_transmittance(origins, dirs, density_scale, extinction, grid, seeds, transform=None,
                                index=None, return_evaluations: bool = False, draws_before: int = 0):
    """RatiotrackingTransmittance.forward
    (rdv/shaders/volumes/ratiotracking_transmittance.h): object space, slab
    test, miss -> 1, entry clamp, then transmittance_rt over d = tMax - tMin
    with ray r's generator spawned from `seeds` by index[r] (default r) and
    a VoxelMajorantField over `grid` [D, H, W]. draws_before: draws of each
    ray's generator already taken in the same invocation (2 after a jittered
    camera, cameras.h:7)."""
    o, w = object_space(origins, dirs, transform)
    tmin, tmax = ray_box(o, w)
    miss = (tmax <= 0) | (tmin > tmax)
    tmin = np.maximum(tmin, np.float32(0.0))
    x = o + w * tmin[:, None]
    d = tmax - tmin
    n = o.shape[0]
    out = np.ones(n, dtype=np.float32)
    idx = np.arange(n) if index is None else np.asarray(index)
    hit = np.nonzero(~miss)[0]
    counts = np.zeros(hit.size, dtype=np.int64)
    g = np.asarray(grid, dtype=np.float32)
    if g.ndim == 4:
        g = g[..., 0]
    if hit.size:
        state = random_spawn(seeds, idx[hit])
        for _ in range(draws_before):
            random_step(state)
        out[hit] = transmittance_rt(x[hit], w[hit], d[hit], density_scale, extinction,
                                    lambda xx, ww: voxel_majorant(g, xx, ww), state, counts=counts)
    if return_evaluations:
        return out, int(counts.sum())
    return out


# ---------------------------------------------------------------------------
# PBVR (rdv/domain/volumes.py:257-326, rdv/shaders/volumes/pbvr.h)
# ---------------------------------------------------------------------------
_PI = np.float32(3.14159265358979323846)
_INV_PI = np.float32(0.31830988618379067153776752674503)


def _glsl_min(a, b):
    """GLSL min(a, b) = b < a ? b : a (elementwise, float32)."""
    return np.where(b < a, b, a).astype(np.float32)


def _glsl_max(a, b):
    """GLSL max(a, b) = a < b ? b : a (elementwise, float32)."""
    return np.where(a < b, b, a).astype(np.float32)


def _f32(fn, v):
    """A float32 math function, correctly rounded (evaluated in float64)."""
    return fn(np.asarray(v, dtype=np.float64)).astype(np.float32)


def sphere_majorant(grid: np.ndarray, x: np.ndarray, w: np.ndarray):
    """SphereMajorantField.forward (rdv/shaders/volumes/sphere_majorant_field.h):
    grid [D, H, W, 2] (z, y, x; majorant, radius in voxels) float32; x, w
    [R, 3] object space. Returns the cell's majorant and the distance along
    w to the exit of the box of half-width radius voxels around the cell's
    centre, at least 1e-6."""
    dims = np.array([grid.shape[2], grid.shape[1], grid.shape[0]], dtype=np.int64)
    f = dims.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        pos = (x * np.float32(0.5) + np.float32(0.5)) * f
        cell = np.clip(np.trunc(pos).astype(np.int64), 0, dims - 1)
        value = grid[cell[:, 2], cell[:, 1], cell[:, 0]]
        maj = value[:, 0].astype(np.float32)
        radius = value[:, 1].astype(np.float32)
        vs = np.float32(2.0) / f
        center = (cell.astype(np.float32) + np.float32(0.5)) * vs - np.float32(1.0)
        half = radius[:, None] * vs
        t0 = ((center - half) - x) / w
        t1 = ((center + half) - x) / w
        texit = _glsl_max(t0, t1)
        dist = _glsl_min(_glsl_min(texit[:, 0], texit[:, 1]), texit[:, 2])
        dist = _glsl_max(dist, np.float32(1e-6))
    return maj, dist


def dir2xr(w: np.ndarray) -> np.ndarray:
    """dir2xr (rdv/shaders/libraries/math_library.h:265-276) in float32:
    (atan(w.x, w.z) / pi, asin(clamp(w.y, -1, 1)) * 2 / pi), w.x += 1e-7
    where w.x = w.z = 0 (and += 0 elsewhere, which turns -0 into +0)."""
    w = np.asarray(w, dtype=np.float32)
    nudge = np.where((w[:, 0] == 0) & (w[:, 2] == 0), np.float32(1e-7), np.float32(0.0))
    wx = (w[:, 0] + nudge).astype(np.float32)
    beta = _f32(np.arcsin, np.clip(w[:, 1], np.float32(-1.0), np.float32(1.0)))
    alpha = np.arctan2(wx.astype(np.float64), w[:, 2].astype(np.float64)).astype(np.float32)
    return np.stack([alpha * _INV_PI, beta * (np.float32(2.0) * _INV_PI)], axis=1).astype(np.float32)


def constant_environment(rgb):
    """A Constant map's environment: the same RGB for every direction."""
    c = np.asarray(rgb, dtype=np.float32).reshape(1, 3)
    return lambda w: np.repeat(c, w.shape[0], axis=0)


def equirect_environment(image, clamp: bool = True, aligned: bool = False, linear: bool = True):
    """XRProject() >> TensorSampler(image [H, W, 3]): dir2xr, then the 2-D
    sampler (oracle/tensors.py tensor_sampler)."""
    from .tensors import tensor_sampler
    img = np.asarray(image, dtype=np.float32)
    return lambda w: tensor_sampler(img, dir2xr(w), clamp=clamp, aligned=aligned, linear=linear)


def ortho_basis(n: np.ndarray):
    """create_ortho_basis (math_library.h:323-330), float32, [R, 3] -> (T, B)."""
    one = np.float32(1.0)
    sign = np.where(n[:, 2] >= 0, one, -one).astype(np.float32)
    a = (-one / (sign + n[:, 2])).astype(np.float32)
    b = ((n[:, 0] * n[:, 1]) * a).astype(np.float32)
    T = np.stack([one + ((sign * n[:, 0]) * n[:, 0]) * a, sign * b, -sign * n[:, 0]], axis=1)
    B = np.stack([b, sign + (n[:, 1] * n[:, 1]) * a, -n[:, 1]], axis=1)
    return T.astype(np.float32), B.astype(np.float32)


def hg_phase_sample(w: np.ndarray, g: float, state: np.ndarray) -> np.ndarray:
    """hg_phase_sample (rdv/shaders/libraries/random_library.h:224-239) in
    float32: two draws (azimuth phi, then xi), the inverted Henyey-Greenstein
    CDF (uniform cosine when |g| < 0.001), the direction around w in
    create_ortho_basis' frame. `state` advances in place."""
    one, two = np.float32(1.0), np.float32(2.0)
    g = np.float32(g)
    phi = (random_draw(state) * two) * _PI
    xi = random_draw(state)
    g2 = g * g
    with np.errstate(divide="ignore", invalid="ignore"):
        t = (one - g2) / ((one - g) + (two * g) * xi)
        invertcdf = (np.float32(0.5) / g) * ((one + g2) - t * t)
    cos_t = ((two * xi) - one) if abs(float(g)) < 0.001 else invertcdf
    cos_t = np.asarray(cos_t, dtype=np.float32)
    sin_t = np.sqrt(np.maximum(np.float32(0.0), one - cos_t * cos_t)).astype(np.float32)
    t0, t1 = ortho_basis(w)
    s0 = (sin_t * _f32(np.sin, phi))[:, None]
    s1 = (sin_t * _f32(np.cos, phi))[:, None]
    return ((s0 * t0 + s1 * t1) + cos_t[:, None] * w).astype(np.float32)


def _inverse3(transform):
    if transform is None:
        return np.eye(3, dtype=np.float32)
    t = np.asarray(transform, dtype=np.float64).reshape(-1)
    return np.linalg.inv(t[:9].reshape(3, 3).T).astype(np.float32)


def _apply3(L, v):
    out = np.empty_like(v)
    for i in range(3):
        acc = (L[i, 0] * v[:, 0]).astype(np.float32) + (L[i, 1] * v[:, 1]).astype(np.float32)
        out[:, i] = acc.astype(np.float32) + (L[i, 2] * v[:, 2]).astype(np.float32)
    return out


def slab_exit(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """tMax of ray_box_intersection (math_library.h:48-57) from x along w,
    min(min(c.x, c.y), c.z) with GLSL min, c = -x / w + |1 / w|."""
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.float32(1.0) / w
        c = (-x * inv + np.abs(inv)).astype(np.float32)
    return _glsl_min(_glsl_min(c[:, 0], c[:, 1]), c[:, 2])


def pbvr(origins, dirs, extinction, environment, majorant, seeds, transform=None, albedo=(1.0, 1.0, 1.0),
         g: float = 0.0, max_bounces: int = 32, index=None, draws_before: int = 0,
         return_evaluations: bool = False, safety_cap: int = 8192):
    """PBVR.forward (rdv/shaders/volumes/pbvr.h:21-110) vectorised over rays
    in lock step, every operation in float32:

        x, wo <- object space; miss -> environment(w)
        x <- entry point; d = tMax - tMin; W = 1; bounces = 0
        for (safety < 8192 while d > 0):
            maj = max(majorant(x, wo, max_step), 1e-12); max_step = max(max_step, 1e-6)
            dt = -log(1 - random()) / maj; step = min(dt, min(max_step, d))
            x += step wo; d -= step
            step < dt: d <= 0 -> escaped (break), else continue
            random() >= extinction(x) / maj -> continue (null collision)
            W *= albedo; max(W) < 1e-4 -> 0; bounces >= max_bounces -> 0
            w <- hg_phase_sample(w, g); wo <- L w; d <- slab exit from x; bounces++
        escaped -> W * environment(w), else 0

    `majorant(x, wo)` returns (value, distance) -- voxel_majorant or
    sphere_majorant; `environment(w)` maps [n, 3] -> [n, 3]. The reference's
    local_majorant (volumes/majorant_field_precode.h) is absent from its
    checkout; it is taken as the field's (majorant, distance) with the
    distance floored at 1e-6, the floor ratiotracking_transmittance_trait.h:14
    applies (pbvr.h:60-61 names local_majorant's own epsilon)."""
    o, w_obj = object_space(origins, dirs, transform)
    w_world = np.asarray(dirs, dtype=np.float32).copy()
    L = _inverse3(transform)
    tmin, tmax = ray_box(o, w_obj)
    miss = (tmax <= 0) | (tmin > tmax)
    tmin = np.maximum(tmin, np.float32(0.0))
    n = o.shape[0]
    out = np.zeros((n, 3), dtype=np.float32)
    if miss.any():
        out[miss] = environment(w_world[miss])
    hit = np.nonzero(~miss)[0]
    evals = 0
    if hit.size:
        idx = np.arange(n) if index is None else np.asarray(index)
        state = random_spawn(seeds, idx[hit])
        for _ in range(draws_before):
            random_step(state)
        x = (o[hit] + w_obj[hit] * tmin[hit, None]).astype(np.float32)
        wo = w_obj[hit].copy()
        w = w_world[hit].copy()
        d = (tmax[hit] - tmin[hit]).astype(np.float32)
        m = hit.size
        W = np.ones((m, 3), dtype=np.float32)
        bounces = np.zeros(m, dtype=np.int64)
        running = np.ones(m, dtype=bool)
        escaped = np.zeros(m, dtype=bool)
        alb = np.asarray(albedo, dtype=np.float32).reshape(1, 3)
        for _ in range(safety_cap):
            running &= d > 0
            act = np.nonzero(running)[0]
            if act.size == 0:
                break
            maj, max_step = majorant(x[act], wo[act])
            maj = _glsl_max(maj.astype(np.float32), np.float32(1e-12))
            max_step = _glsl_max(max_step.astype(np.float32), np.float32(1e-6))
            st = state[act]
            u = random_draw(st)
            with np.errstate(divide="ignore", over="ignore"):
                dt = ((-_log_f32(np.float32(1.0) - u)) / maj).astype(np.float32)
            step = _glsl_min(dt, _glsl_min(max_step.astype(np.float32), d[act]))
            x[act] = (x[act] + step[:, None] * wo[act]).astype(np.float32)
            d[act] = (d[act] - step).astype(np.float32)
            free = step < dt
            esc = free & (d[act] <= 0)
            escaped[act[esc]] = True
            running[act[esc]] = False
            coll = np.nonzero(~free)[0]          # positions inside act
            if coll.size:
                ci = act[coll]
                sigma = np.asarray(extinction(x[ci]), dtype=np.float32)
                evals += ci.size
                sub = st[coll]
                u2 = random_draw(sub)
                real = ~(u2 >= (sigma / maj[coll]).astype(np.float32))
                if real.any():
                    rp = coll[real]                  # positions inside act
                    ri = act[rp]
                    W[ri] = (W[ri] * alb).astype(np.float32)
                    wmax = _glsl_max(_glsl_max(W[ri, 0], W[ri, 1]), W[ri, 2])
                    stop = (wmax < np.float32(1e-4)) | (bounces[ri] >= max_bounces)
                    running[ri[stop]] = False
                    go = ~stop
                    if go.any():
                        gi = ri[go]
                        s2 = sub[real][go]
                        w[gi] = hg_phase_sample(w[gi], g, s2)
                        wo[gi] = _apply3(L, w[gi])
                        d[gi] = slab_exit(x[gi], wo[gi])
                        bounces[gi] += 1
                        tmp = sub[real]
                        tmp[go] = s2
                        sub[real] = tmp
                st[coll] = sub
            state[act] = st
        if escaped.any():
            e = np.nonzero(escaped)[0]
            out[hit[e]] = (W[e] * environment(w[e])).astype(np.float32)
    if return_evaluations:
        return out, evals
    return out


def hg_phase_eval(cos_t: np.ndarray, g: float) -> np.ndarray:
    """hg_phase_eval (random_library.h:241-249) in float32:
    (0.25 / pi) (1 - g^2) / (1 + g^2 - 2 g cos)^1.5, or 0.25 / pi when
    |g| < 0.001."""
    cos_t = np.asarray(cos_t, dtype=np.float32)
    g = np.float32(g)
    quarter_pi = np.float32(np.float32(0.25) / _PI)
    if abs(float(g)) < 0.001:
        return np.full(cos_t.shape, quarter_pi, dtype=np.float32)
    g2 = g * g
    base = ((np.float32(1.0) + g2) - (np.float32(2.0) * g) * cos_t).astype(np.float32)
    powed = np.power(base.astype(np.float64), 1.5).astype(np.float32)
    return ((quarter_pi * (np.float32(1.0) - g2)) / powed).astype(np.float32)


def normalize3(v) -> np.ndarray:
    """v / sqrt((x x + y y) + z z) in float32."""
    v = np.asarray(v, dtype=np.float32).reshape(3)
    sq = np.float32(np.float32(v[0] * v[0] + v[1] * v[1]) + v[2] * v[2])
    return (v / np.float32(np.sqrt(np.float64(sq)))).astype(np.float32)


def xr_env_sample(densities: np.ndarray, levels: int, environment, state: np.ndarray):
    """XREnvironmentSampler.forward (rdv/shaders/rendering/
    xr_environment_sampler.h) in float32 for every row of `state` (advanced
    in place): one draw walks the quadtree (rescaled to [0, 1) per level),
    prob the product of the chosen children's probabilities; two more draws
    place the direction uniformly in solid angle inside the leaf pixel
    (usc2dir, math_library.h:256-263). Returns (directions [R, 3],
    environment / pdf [R, 3])."""
    f32 = np.float32
    dens = np.asarray(densities, dtype=np.float32)
    n = state.shape[0]
    node = np.zeros(n, dtype=np.int64)
    u0 = np.zeros(n, f32); u1 = np.ones(n, f32); v0 = np.zeros(n, f32); v1 = np.ones(n, f32)
    prob = np.ones(n, f32)
    sel = random_draw(state)
    for _ in range(levels):
        cdf = dens[node[:, None] * 4 + np.arange(4)[None, :]]
        child = np.full(n, 3, dtype=np.int64)
        lo = np.zeros(n, f32)
        hi = cdf[:, 3].copy()
        decided = np.zeros(n, dtype=bool)
        for c in range(3):
            take = ~decided & (sel < cdf[:, c])
            child[take] = c
            hi[take] = cdf[take, c]
            decided |= take
            lo = np.where(decided, lo, cdf[:, c]).astype(f32)
        span = (hi - lo).astype(f32)
        prob = (prob * _glsl_max(f32(0.0), span)).astype(f32)
        q = ((sel - lo) / _glsl_max(f32(1e-9), span)).astype(f32)
        sel = _glsl_min(_glsl_max(q, f32(0.0)), f32(1.0))
        umed = ((u0 + u1) * f32(0.5)).astype(f32)
        vmed = ((v0 + v1) * f32(0.5)).astype(f32)
        even = child % 2 == 0
        u1 = np.where(even, umed, u1); u0 = np.where(even, u0, umed)
        top = child // 2 == 0
        v1 = np.where(top, vmed, v1); v0 = np.where(top, v0, vmed)
        node = node * 4 + 1 + child
    pi_, half_pi = _PI, np.float32(1.5707963267948966)
    a0 = ((u0 * f32(2.0) - f32(1.0)) * pi_).astype(f32)
    a1 = ((u1 * f32(2.0) - f32(1.0)) * pi_).astype(f32)
    b0 = ((v0 * f32(2.0) - f32(1.0)) * half_pi).astype(f32)
    b1 = ((v1 * f32(2.0) - f32(1.0)) * half_pi).astype(f32)
    sb0, sb1 = _f32(np.sin, b0), _f32(np.sin, b1)
    solid = ((a1 - a0) * (sb1 - sb0)).astype(f32)
    pdf = (prob / _glsl_max(f32(1e-9), solid)).astype(f32)
    weight = (f32(1.0) / _glsl_max(f32(1e-9), pdf)).astype(f32)
    ta = random_draw(state)
    alpha = ((a0 * (f32(1.0) - ta)) + (a1 * ta)).astype(f32)
    ts = random_draw(state)
    sv = ((sb0 * (f32(1.0) - ts)) + (sb1 * ts)).astype(f32)
    beta = _f32(np.arcsin, np.clip(sv, f32(-1.0), f32(1.0)))
    rr = _f32(np.cos, beta)
    d = np.stack([_f32(np.sin, alpha) * rr, _f32(np.sin, beta), _f32(np.cos, alpha) * rr], axis=1).astype(f32)
    env = np.asarray(environment(d), dtype=np.float32)
    return d, (env * weight[:, None]).astype(f32)


def xr_quadtree(density: np.ndarray, levels: int) -> np.ndarray:
    """The quadtree of rdv/domain/rendering.py:175-278 from an already
    resampled, channel-summed density [2^levels, 2^levels] (float32): row
    solid-angle weights sin(beta1) - sin(beta0), normalisation, the mass
    pyramid, per node (Morton order) the cumulative child probabilities
    (0.25 each under an empty parent), the last forced to 1 -- in float64
    here, so the GPU build agrees within float32 rounding."""
    res = 1 << levels
    d = np.maximum(np.asarray(density, dtype=np.float64), 0.0)
    v0 = np.arange(res) / res
    v1 = (np.arange(res) + 1) / res
    w = np.sin((v1 * 2 - 1) * np.pi / 2) - np.sin((v0 * 2 - 1) * np.pi / 2)
    d = np.maximum(d * w[:, None], 0.0)
    d = d / max(d.sum(), 1e-12)
    pyr = [d]
    for _ in range(levels):
        g = pyr[-1]
        pyr.append(g.reshape(g.shape[0] // 2, 2, g.shape[1] // 2, 2).sum(axis=(1, 3)))
    pyr.reverse()

    def morton(t, dd):
        if dd == 0:
            return t.reshape(1)
        order = [a for i in range(dd) for a in (i, dd + i)]
        return t.reshape([2] * (2 * dd)).transpose(order).reshape(-1)

    out = []
    for dd in range(levels):
        parent = morton(pyr[dd], dd)
        kids = morton(pyr[dd + 1], dd + 1).reshape(-1, 4)
        p = np.where(parent[:, None] > 1e-12, kids / np.maximum(parent, 1e-12)[:, None], 0.25)
        cum = np.cumsum(p, axis=1)
        cum[:, 3] = 1.0
        out.append(cum.reshape(-1))
    return np.concatenate(out)


def pbvrt(origins, dirs, extinction, majorant, seeds, albedo, light_direction, light_intensity=(1.0, 1.0, 1.0),
          environment=None, transform=None, density_scale: float = 1.0, g: float = 0.0, max_bounces: int = 32,
          variant: str = "pbvrt", index=None, draws_before: int = 0, return_evaluations: bool = False,
          env_densities=None, env_levels: int = 0):
    """PBVRT.forward (rdv/shaders/volumes/pbvrt.h:21-149) and, with
    variant="nee", PBVR_NEE.forward (pbvr_nee.h), vectorised over rays, each
    ray a state machine of the main path and its shadow ray run in lock step,
    every operation in float32:

        object space; miss (tMax <= 0 or tMin >= tMax) -> 0 (PBVRT: alpha 1)
        x <- entry at max(0, tMin) + 1e-5; d = tMax - tMin; W = 1
        for (safety < 16384):
            maj = majorant(x, wo, dist) + 1e-5; dist <= 1e-5 -> 1e-5
            dt = min(min(d, dist), -log(1 - random()) / (density_scale maj))
            x += dt wo; d -= dt; dt >= dist -> continue; d <= 1e-7 -> break
            random() >= extinction(x) / maj -> continue
            ++bounces > max_bounces -> PBVRT: W = 0, break; NEE: return
            W *= albedo; no W > 1e-4 -> PBVRT: break; NEE: return
            out += W transmittance_rt(x, L l, slab exit) hg_phase_eval(w . l, g)
            w <- hg_phase_sample(w, g); wo <- L w; d <- slab exit from x
        PBVRT: bounces > 0 -> alpha 0, out = out light_intensity + W env(w)

    `majorant(x, w)` returns the field's raw (value, distance);
    transmittance_rt is ratiotracking_transmittance_trait.h's loop (as
    transmittance_rt above). Returns [n, 4] (PBVRT) or [n, 3] (NEE, ENV).
    variant="env" is PBVR_ENV (pbvr_env.h): each NEE direction and its
    radiance / pdf come from xr_env_sample over (env_densities, env_levels)
    and `environment`, the term (tr W) * radiance / pdf."""
    env_nee = variant == "env"
    nee = variant in ("nee", "env")
    o, w_obj = object_space(origins, dirs, transform)
    w_world = np.asarray(dirs, dtype=np.float32).copy()
    L = _inverse3(transform)
    n = o.shape[0]
    n_out = 3 if nee else 4
    out = np.zeros((n, n_out), dtype=np.float32)
    if not nee:
        out[:, 3] = 1.0
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.float32(1.0) / w_obj
        xc = -o * inv
        sa = np.abs(inv)
        lo = xc - sa
        hi = xc + sa
    tmin = _glsl_max(_glsl_max(lo[:, 0], lo[:, 1]), lo[:, 2])
    tmax = _glsl_min(_glsl_min(hi[:, 0], hi[:, 1]), hi[:, 2])
    miss = (tmax <= 0) | (tmin >= tmax)
    hit = np.nonzero(~miss)[0]
    evals = 0
    if hit.size == 0:
        return (out, 0) if return_evaluations else out
    idx = np.arange(n) if index is None else np.asarray(index)
    state = random_spawn(seeds, idx[hit])
    for _ in range(draws_before):
        random_step(state)
    m = hit.size
    t0 = (_glsl_max(np.float32(0.0), tmin[hit]) + np.float32(1e-5)).astype(np.float32)
    x = (o[hit] + w_obj[hit] * t0[:, None]).astype(np.float32)
    d = (tmax[hit] - t0).astype(np.float32)
    wo = w_obj[hit].copy()
    w = w_world[hit].copy()
    W = np.ones((m, 3), dtype=np.float32)
    acc = np.zeros((m, 3), dtype=np.float32)
    alb = np.asarray(albedo, dtype=np.float32).reshape(1, 3)
    light = normalize3(light_direction) if not env_nee else np.array([0.0, 1.0, 0.0], np.float32)
    lo_dir = _apply3(L, light[None].astype(np.float32))[0]
    l_rows = np.broadcast_to(light, (m, 3)).astype(np.float32).copy()     # NEE direction per ray
    lo_rows = np.broadcast_to(lo_dir, (m, 3)).astype(np.float32).copy()
    ew = np.ones((m, 3), dtype=np.float32)
    bounces = np.zeros(m, dtype=np.int64)
    safety = np.zeros(m, dtype=np.int64)
    mode = np.zeros(m, dtype=np.int64)          # 0 main, 1 shadow
    xs = np.zeros((m, 3), dtype=np.float32)
    ds = np.zeros(m, dtype=np.float32)
    T = np.ones(m, dtype=np.float32)
    phase = np.zeros(m, dtype=np.float32)
    s_safety = np.zeros(m, dtype=np.int64)
    maj = np.ones(m, dtype=np.float32)
    running = np.ones(m, dtype=bool)
    ended = np.zeros(m, dtype=bool)             # main loop over: resolve the outputs
    f32 = np.float32
    dsc = f32(density_scale)

    def shadow_end(rows, t):
        tr = (t.astype(np.float32) * phase[rows]).astype(np.float32)
        term = ((tr[:, None] * W[rows]).astype(np.float32) * ew[rows]).astype(np.float32)
        acc[rows] = (acc[rows] + term).astype(np.float32)
        sub = state[rows]
        w[rows] = hg_phase_sample(w[rows], g, sub)
        state[rows] = sub
        wo[rows] = _apply3(L, w[rows])
        d[rows] = slab_exit(x[rows], wo[rows])
        mode[rows] = 0

    while running.any():
        pend = np.zeros(m, dtype=bool)
        # -- main-path steps
        mm = np.nonzero(running & (mode == 0))[0]
        if mm.size:
            cap = safety[mm] >= 16384
            ended[mm[cap]] = True
            running[mm[cap]] = False
            mm = mm[~cap]
            safety[mm] += 1
            mv, dist = majorant(x[mm], wo[mm])
            mj = (mv.astype(np.float32) + f32(1e-5)).astype(np.float32)
            dist = np.where(dist <= f32(1e-5), f32(1e-5), dist).astype(np.float32)
            sub = state[mm]
            u = random_draw(sub)
            state[mm] = sub
            with np.errstate(divide="ignore", over="ignore"):
                q = ((-_log_f32(f32(1.0) - u)) / (dsc * mj)).astype(np.float32)
            dt = _glsl_min(_glsl_min(d[mm], dist), q)
            x[mm] = (x[mm] + dt[:, None] * wo[mm]).astype(np.float32)
            d[mm] = (d[mm] - dt).astype(np.float32)
            moved = dt >= dist
            brk = ~moved & (d[mm] <= f32(1e-7))
            ended[mm[brk]] = True
            running[mm[brk]] = False
            coll = ~moved & ~brk
            maj[mm[coll]] = mj[coll]
            pend[mm[coll]] = True
        # -- shadow-ray steps
        ss = np.nonzero(running & (mode == 1))[0]
        if ss.size:
            done = ~(ds[ss] > 0) | (s_safety[ss] >= 1024)
            if done.any():
                shadow_end(ss[done], T[ss[done]])
            ss = ss[~done]
        if ss.size:
            s_safety[ss] += 1
            mv, dist = majorant(xs[ss], lo_rows[ss])
            mj = _glsl_max(mv.astype(np.float32), f32(1e-12))
            dist = _glsl_max(dist.astype(np.float32), f32(1e-6))
            sub = state[ss]
            u = random_draw(sub)
            state[ss] = sub
            with np.errstate(divide="ignore", over="ignore"):
                q = ((-_log_f32(f32(1.0) - u)) / (mj * dsc)).astype(np.float32)
            dt = _glsl_min(dist, q)
            ds[ss] = (ds[ss] - dt).astype(np.float32)
            xs[ss] = (xs[ss] + dt[:, None] * lo_rows[ss]).astype(np.float32)
            moved = dt >= dist
            fin = ~moved & (ds[ss] <= 0)
            if fin.any():
                shadow_end(ss[fin], T[ss[fin]])
            coll = ~moved & ~fin
            maj[ss[coll]] = mj[coll]
            pend[ss[coll]] = True
        # -- collisions: the extinction at the main or shadow point
        pi_ = np.nonzero(pend)[0]
        if pi_.size == 0:
            continue
        pts = np.where((mode[pi_] == 0)[:, None], x[pi_], xs[pi_]).astype(np.float32)
        sigma = np.asarray(extinction(pts), dtype=np.float32)
        evals += pi_.size
        ratio = (sigma / maj[pi_]).astype(np.float32)
        sh = mode[pi_] == 1
        if sh.any():
            rows = pi_[sh]
            T[rows] = (T[rows] * (f32(1.0) - ratio[sh])).astype(np.float32)
            low = rows[T[rows] < f32(0.05)]
            if low.size:
                sub = state[low]
                u2 = random_draw(sub)
                state[low] = sub
                kill = u2 >= T[low]
                if kill.any():
                    shadow_end(low[kill], np.zeros(int(kill.sum()), dtype=np.float32))
                T[low[~kill]] = 1.0
        mn = ~sh
        if mn.any():
            rows = pi_[mn]
            sub = state[rows]
            u2 = random_draw(sub)
            state[rows] = sub
            real = rows[~(u2 >= ratio[mn])]
            if real.size:
                bounces[real] += 1
                over = real[bounces[real] > max_bounces]
                if over.size:
                    if not nee:
                        W[over] = 0.0
                    ended[over] = True
                    running[over] = False
                go = real[bounces[real] <= max_bounces]
                W[go] = (W[go] * alb).astype(np.float32)
                low_w = ~np.any(W[go] > f32(1e-4), axis=1)
                ended[go[low_w]] = True
                running[go[low_w]] = False
                go = go[~low_w]
                if go.size:
                    if env_nee:
                        sub = state[go]
                        l_rows[go], ew[go] = xr_env_sample(env_densities, env_levels, environment, sub)
                        state[go] = sub
                        lo_rows[go] = _apply3(L, l_rows[go])
                    lg = l_rows[go]
                    cos_t = ((w[go, 0] * lg[:, 0] + w[go, 1] * lg[:, 1]).astype(np.float32) + w[go, 2] * lg[:, 2])
                    phase[go] = hg_phase_eval(cos_t.astype(np.float32), g)
                    xs[go] = x[go]
                    ds[go] = slab_exit(x[go], lo_rows[go])
                    T[go] = 1.0
                    s_safety[go] = 0
                    mode[go] = 1
    if nee:
        out[hit] = acc
    else:
        scat = bounces > 0
        res = np.zeros((m, 4), dtype=np.float32)
        res[:, 3] = 1.0
        if scat.any():
            e = np.nonzero(scat)[0]
            env = environment(w[e]).astype(np.float32)
            li = np.asarray(light_intensity, dtype=np.float32).reshape(1, 3)
            res[e, :3] = ((acc[e] * li).astype(np.float32) + (W[e] * env).astype(np.float32)).astype(np.float32)
            res[e, 3] = 0.0
        out[hit] = res
    return (out, evals) if return_evaluations else out
