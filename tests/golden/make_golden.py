"""Regenerates the golden fixtures in this directory from the reference itself.

Run where the reference checkout is present (its path: RDV_REFERENCE_ROOT, else
the default in oracle/_clib.py):

    python tests/golden/make_golden.py            # every fixture
    python tests/golden/make_golden.py coopmat    # coopmat.npz only
    python tests/golden/make_golden.py pbvr       # pbvr.npz only
    python tests/golden/make_golden.py samplers   # grid_sampler.npz only

Three sources, all the reference's own code:

* ``oracle/_ref/libref_shaders.so`` -- the reference's scalar GLSL functions
  (maps/linear.h, relu.h, composite.h, tensors/linear_tensor_op.h,
  relu_tensor_op.h, conv2d_tensor_op.h, the Winograd transforms,
  volumes/raymarching_transmittance_trait.h, libraries/random_library.h and
  volumes/ratiotracking_transmittance_trait.h) compiled as C++ from the
  reference checkout by ``make -C oracle ref``;
* ``oracle/_ref/libref_coopmat.so`` -- the reference's cooperative-matrix
  (float16 tensor-core) bodies: maps/linear_fast.h in Map chains of the
  config-5 and config-2 architectures, tensors/linear_tensor_op_{small,
  simple,fast,mine}.h and tensors/conv2d_tensor_op_winograd3x3.h, executed
  on the CPU by 32-thread workgroups (oracle/ref_shim/coopmat_prelude.hpp
  gives coopMatMulAdd its ascending-k fp32 summation);
* ``oracle/_ref/libref_pbvr.so`` -- the reference's PBVR body
  (volumes/pbvr.h) and its Henyey-Greenstein sampler
  (libraries/random_library.h) compiled as C++ (oracle/ref_shim/ref_pbvr.cpp);
* ``oracle/_ref/libref_samplers.so`` -- the reference's GridSampler
  (samplers/grid_sampler.h) compiled as C++ (oracle/ref_shim/ref_samplers.cpp);
* ``rdv/domain/nn.py``'s torch helpers ``_winograd_transform_weight``,
  ``_tile_weight_fp16`` and ``_cast_fp16`` and its ``_WINOGRAD_G`` table,
  executed from the reference source. The package itself cannot be
  imported (it needs the external ``vk`` module at import time), so these
  definitions are lifted out of the file with ``ast`` and executed on
  their own.

The fixtures are small ``.npz`` files; the CPU tests compare the oracle's
restatements against them, so they keep pinning the oracle where the
reference checkout is absent (e.g. the GPU box).
"""
from __future__ import annotations

import ast
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle._clib import (REFERENCE_ROOT, ptr, ptr_array, ref_coopmat_lib, ref_lib, ref_pbvr_lib,  # noqa: E402
                          ref_samplers_lib)


def xavier_uniform(rng, out_f, in_f):
    bound = np.sqrt(6.0 / (in_f + out_f))
    return rng.uniform(-bound, bound, size=(out_f, in_f)).astype(np.float32)


def reference_python_helpers():
    """Executes _WINOGRAD_G and _winograd_transform_weight from the
    reference's nn.py in an isolated namespace."""
    path = os.path.join(REFERENCE_ROOT, "src", "rdv", "domain", "nn.py")
    tree = ast.parse(open(path).read(), filename=path)
    wanted = {"_WINOGRAD_G", "_winograd_transform_weight", "_tile_weight_fp16", "_cast_fp16"}
    body = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in wanted:
            body.append(node)
        elif isinstance(node, ast.Assign) and any(getattr(t, "id", None) in wanted for t in node.targets):
            body.append(node)
    mod = ast.Module(body=body, type_ignores=[])
    ns: dict = {}
    exec(compile(mod, path, "exec"), ns)
    return ns


class _TorchHolder:
    """Stands in for RDVObject: the helper only calls .as_tensor('torch')."""

    def __init__(self, t):
        self.t = t

    def as_tensor(self, backend):
        assert backend == "torch"
        return self.t


def main():
    lib = ref_lib()
    rng = np.random.default_rng(20240601)
    out = {}

    # --- Map chain, BASELINE config-1 architecture (3->64->64->64->4) -------
    dims = [3, 64, 64, 64, 4]
    W = [xavier_uniform(rng, dims[i + 1], dims[i]) for i in range(4)]
    b = [rng.uniform(-0.1, 0.1, size=dims[i + 1]).astype(np.float32) for i in range(4)]
    x = rng.uniform(-1, 1, size=(96, 3)).astype(np.float32)
    y = np.zeros((96, 4), dtype=np.float32)
    lib.ref_mlp_c1(ptr(x), x.shape[0], ptr_array(W), ptr_array(b), ptr(y))
    np.savez_compressed(os.path.join(HERE, "mlp_c1.npz"), x=x, y=y,
                        **{f"W{i}": W[i] for i in range(4)}, **{f"b{i}": b[i] for i in range(4)})

    # --- odd widths 5 -> 16 -> ReLU -> 7 -------------------------------------
    W = [xavier_uniform(rng, 16, 5), xavier_uniform(rng, 7, 16)]
    b = [rng.uniform(-0.5, 0.5, size=16).astype(np.float32), rng.uniform(-0.5, 0.5, size=7).astype(np.float32)]
    x = rng.standard_normal((37, 5)).astype(np.float32)
    y = np.zeros((37, 7), dtype=np.float32)
    lib.ref_mlp_small(ptr(x), x.shape[0], ptr_array(W), ptr_array(b), ptr(y))
    np.savez_compressed(os.path.join(HERE, "mlp_small.npz"), x=x, y=y, W0=W[0], W1=W[1], b0=b[0], b1=b[1])

    # --- TensorOperation fp32 ------------------------------------------------
    x = rng.standard_normal((20, 16)).astype(np.float32)
    Wt = xavier_uniform(rng, 24, 16)
    bt = rng.uniform(-0.5, 0.5, size=24).astype(np.float32)
    y = np.zeros((20, 24), dtype=np.float32)
    lib.ref_linear_tensor_op_16_24(ptr(x), 20, ptr(Wt), ptr(bt), ptr(y))
    xr = rng.standard_normal((8, 16)).astype(np.float32)
    yr = np.zeros_like(xr)
    lib.ref_relu_tensor_op(ptr(xr), 8, 16, ptr(yr))
    xc = rng.standard_normal((16 * 16, 16)).astype(np.float32)
    wc = (rng.standard_normal((3, 3, 16, 32)) * np.sqrt(2.0 / (9 * 16))).astype(np.float32)
    bc = rng.uniform(-0.1, 0.1, size=32).astype(np.float32)
    yc = np.zeros((16 * 16, 32), dtype=np.float32)
    lib.ref_conv2d_tensor_op_3x3_16_32_16x16(ptr(xc), ptr(wc), ptr(bc), ptr(yc))
    np.savez_compressed(os.path.join(HERE, "tensor_ops.npz"), lin_x=x, lin_W=Wt, lin_b=bt, lin_y=y,
                        relu_x=xr, relu_y=yr, conv_x=xc, conv_w=wc, conv_b=bc, conv_y=yc)

    # --- Winograd scalar transforms and the filter transform ----------------
    d = rng.standard_normal((64, 16)).astype(np.float32)
    V = np.zeros_like(d)
    for i in range(64):
        lib.ref_winograd_fwd(ptr(d[i]), ptr(V[i]))
    M = rng.standard_normal((64, 16)).astype(np.float32)
    Y = np.zeros((64, 4), dtype=np.float32)
    for i in range(64):
        lib.ref_winograd_inv(ptr(M[i]), ptr(Y[i]))
    import torch
    ns = reference_python_helpers()
    wf = (rng.standard_normal((3, 3, 16, 32)) * 0.2).astype(np.float32)
    U = ns["_winograd_transform_weight"](_TorchHolder(torch.from_numpy(wf)), 16, 32).numpy()
    np.savez_compressed(os.path.join(HERE, "winograd.npz"), d=d, V=V, M=M, Y=Y, w=wf, U=U,
                        G=np.array(ns["_WINOGRAD_G"], dtype=np.float64))

    # --- fixed-step transmittance ---------------------------------------------
    nr = 48
    xs = rng.uniform(-1, 1, size=(nr, 3)).astype(np.float32)
    ws = rng.standard_normal((nr, 3)).astype(np.float32)
    ws /= np.linalg.norm(ws, axis=1, keepdims=True)
    ds = rng.uniform(0.0, 2.5, size=nr).astype(np.float32)
    ds[:4] = [0.0, -0.1, 1e-3, 3.0]
    c0 = rng.uniform(0.0, 3.0, size=nr).astype(np.float32)
    c1 = rng.uniform(0.0, 8.0, size=nr).astype(np.float32)
    c0[4:8] = 40.0  # tau crosses 16 -> early return 0
    T = np.zeros(nr, dtype=np.float32)
    for i in range(nr):
        T[i] = lib.ref_transmittance_rm(ctypes.c_float(c0[i]), ctypes.c_float(c1[i]), ptr(xs[i]), ptr(ws[i]),
                                        ctypes.c_float(ds[i]), ctypes.c_float(0.05), ctypes.c_float(1.0))
    np.savez_compressed(os.path.join(HERE, "transmittance.npz"), x=xs, w=ws, d=ds, c0=c0, c1=c1, T=T,
                        step=np.float32(0.05), scale=np.float32(1.0))
    # --- resampling / concatenation tensor ops -------------------------------
    xs = rng.standard_normal((8 * 12, 16)).astype(np.float32)
    down = np.zeros((4 * 6, 16), dtype=np.float32)
    lib.ref_downsample2x(ptr(xs), 8, 12, 16, ptr(down))
    xu = rng.standard_normal((4 * 6, 8)).astype(np.float32)
    up = np.zeros((8 * 12, 8), dtype=np.float32)
    lib.ref_upsample2x(ptr(xu), 4, 6, 8, ptr(up))
    x1 = rng.standard_normal((20, 16)).astype(np.float32)
    x2 = rng.standard_normal((20, 8)).astype(np.float32)
    cat = np.zeros((20, 24), dtype=np.float32)
    lib.ref_concat(ptr(x1), 16, ptr(x2), 8, 20, ptr(cat))
    np.savez_compressed(os.path.join(HERE, "resample.npz"), down_x=xs, down_y=down, up_x=xu, up_y=up,
                        cat_x1=x1, cat_x2=x2, cat_y=cat)
    # --- ratio tracking: the generator and transmittance_rt -------------------
    # random_library.h's per-invocation state (seeds spawned by the index)
    # and its first 64 draws; then transmittance_rt over ray segments with
    # the analytic extinction c0 + c1 |x|^2 and a 4x5x6 voxel majorant, for
    # three media (dense: mostly Russian roulette; medium; thin).
    seeds = np.array([777, 31337, 4242, 99991], dtype=np.uint32)
    rng_index = np.array([0, 1, 2, 31, 1000, 65535, 123456789, 2 ** 31 - 1], dtype=np.int64)
    rng_draws = np.zeros((rng_index.size, 64), dtype=np.float32)
    for i, idx in enumerate(rng_index):
        lib.ref_random_sequence(ptr(seeds), int(idx), 64, ptr(rng_draws[i]))
    nr = 96
    media = np.array([[1.5, 2.0, 1.0, 1.3], [0.2, 0.5, 1.0, 1.0], [0.05, 0.3, 3.0, 0.7]], dtype=np.float32)
    rt_x = rng.uniform(-0.999, 0.999, size=(len(media), nr, 3)).astype(np.float32)
    rt_w = rng.standard_normal((len(media), nr, 3)).astype(np.float32)
    rt_w /= np.linalg.norm(rt_w, axis=2, keepdims=True)
    rt_d = rng.uniform(0.0, 2.5, size=(len(media), nr)).astype(np.float32)
    rt_d[:, :3] = [0.0, -0.1, 1e-4]
    rt_index = rng.integers(0, 1 << 20, size=(len(media), nr)).astype(np.int64)
    grids = np.zeros((len(media), 4, 5, 6), dtype=np.float32)
    rt_T = np.zeros((len(media), nr), dtype=np.float32)
    for m, (c0m, c1m, gscale, dsm) in enumerate(media):
        grids[m] = (rng.uniform(0.5, 1.5, size=(4, 5, 6)) * (c0m + 3 * c1m) * gscale).astype(np.float32)
        for i in range(nr):
            rt_T[m, i] = lib.ref_transmittance_rt(
                ctypes.c_float(c0m), ctypes.c_float(c1m), ptr(grids[m]), 4, 5, 6, ptr(seeds), int(rt_index[m, i]),
                ptr(np.ascontiguousarray(rt_x[m, i])), ptr(np.ascontiguousarray(rt_w[m, i])),
                ctypes.c_float(rt_d[m, i]), ctypes.c_float(dsm))
    np.savez_compressed(os.path.join(HERE, "ratiotracking.npz"), seeds=seeds, rng_index=rng_index,
                        rng_draws=rng_draws, media=media, x=rt_x, w=rt_w, d=rt_d, index=rt_index, grids=grids,
                        T=rt_T)
    coopmat_goldens()
    pbvr_goldens()
    sampler_goldens()
    print("golden fixtures written to", HERE)


def _f16(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float16)).view(np.uint16)


def coopmat_goldens():
    """coopmat.npz: inputs, weights and outputs of the reference's float16
    (cooperative-matrix) code paths. Float16 weight images are made by the
    reference's own torch helpers."""
    import torch

    lib = ref_coopmat_lib()
    ns = reference_python_helpers()
    rng = np.random.default_rng(20261202)
    out = {}

    def kaiming(o, i):
        return (rng.standard_normal((o, i)) * np.sqrt(2.0 / i)).astype(np.float32)

    # Map chains: 3 full 32-row workgroups + a partial one (scalar fp32 path)
    for name, dims, rows in (("c5", [3, 64, 64, 64, 64, 4], 112), ("c2", [32] + [128] * 8 + [16], 80)):
        Ws = [kaiming(dims[i + 1], dims[i]) for i in range(len(dims) - 1)]
        if name == "c2":
            # multiples of 2^-7 stored as int8 codes, to keep the fixture
            # small (exact in float16, so staged and fallback rows see the
            # same weights)
            Ws = [np.clip(np.round(w * 128.0), -127, 127).astype(np.float32) / 128.0 for w in Ws]
        bs = [(rng.standard_normal(dims[i + 1]) * 0.1).astype(np.float32) for i in range(len(dims) - 1)]
        x = (rng.uniform(-1, 1, (rows, dims[0])) if name == "c5" else rng.standard_normal((rows, dims[0])))
        x = x.astype(np.float32)
        y = np.zeros((rows, dims[-1]), np.float32)
        getattr(lib, f"ref_cm_mlp_{name}")(ptr(x), rows, ptr_array(Ws), ptr_array(bs), ptr(y))
        out[f"{name}_x"], out[f"{name}_y"] = x, y
        for i, (w, b) in enumerate(zip(Ws, bs)):
            out[f"{name}_W{i}"] = (w * 128.0).astype(np.int8) if name == "c2" else w
            out[f"{name}_b{i}"] = b

    # TensorOps
    for name, inf, outf, batch, image in (("small_32_48", 32, 48, 64, "f32"), ("small_64_32", 64, 32, 64, "f32"),
                                          ("simple_32_64", 32, 64, 64, "cast"), ("fast_32_64", 32, 64, 64, "tiled"),
                                          ("mine_32_48", 32, 48, 64, "f32")):
        x = rng.standard_normal((batch, inf)).astype(np.float32)
        W = kaiming(outf, inf)
        b = (rng.standard_normal(outf) * 0.1).astype(np.float32)
        if image == "cast":
            img = _f16(ns["_cast_fp16"](_TorchHolder(torch.from_numpy(W))).numpy())
        elif image == "tiled":
            img = _f16(ns["_tile_weight_fp16"](_TorchHolder(torch.from_numpy(W)), outf, inf).numpy())
        else:
            img = W
        y = np.zeros((batch, outf), np.float32)
        getattr(lib, f"ref_cm_{name}")(ptr(x), batch, ptr(img), ptr(b), ptr(y))
        out.update({f"{name}_x": x, f"{name}_W": W, f"{name}_b": b, f"{name}_y": y})

    # Conv2DTensorOpWinograd3x3, one 16x16 image
    for c in (16, 48):
        x = rng.standard_normal((16, 16, c)).astype(np.float32)
        # float16 values (stored as float16)
        w = (rng.standard_normal((3, 3, c, c)) * np.sqrt(2.0 / (9 * c))).astype(np.float16).astype(np.float32)
        b = (rng.standard_normal(c) * 0.1).astype(np.float32)
        U = ns["_winograd_transform_weight"](_TorchHolder(torch.from_numpy(w)), c, c).numpy()
        U16 = _f16(U)
        y = np.zeros((256, c), np.float32)
        getattr(lib, f"ref_cm_winograd_{c}")(ptr(np.ascontiguousarray(x.reshape(256, c))), ptr(U16), ptr(b), ptr(y))
        out.update({f"wino{c}_x": x, f"wino{c}_w": w.astype(np.float16), f"wino{c}_b": b,
                    f"wino{c}_y": y.reshape(16, 16, c)})
    np.savez_compressed(os.path.join(HERE, "coopmat.npz"), **out)


def pbvr_goldens():
    """pbvr.npz: PBVR.forward of the reference (volumes/pbvr.h), and
    PBVRT / PBVR_NEE (volumes/pbvrt.h, pbvr_nee.h) as t_*, over world
    rays [n, 6] with the analytic extinction c0 + c1 |x|^2, a constant
    environment, a voxel and a sphere majorant field, several albedos,
    anisotropies and bounce budgets, an identity and a scaled + shifted
    transform (inverse exact in any formula); and hg_phase_sample
    directions for a few g (the uniform branch |g| < 0.001 included)."""
    lib = ref_pbvr_lib()
    rng = np.random.default_rng(424242)
    n = 384
    o = rng.uniform(-3, 3, (n, 3)).astype(np.float32)
    t = rng.uniform(-0.8, 0.8, (n, 3)).astype(np.float32)
    w = t - o
    w /= np.linalg.norm(w, axis=1, keepdims=True)
    w = w.astype(np.float32)
    w[: n // 8] *= -1.0                       # pointing away: misses
    o[n // 8: n // 4] *= np.float32(0.2)       # starting inside the box
    rays = np.ascontiguousarray(np.concatenate([o, w], 1).astype(np.float32))
    seeds = np.array([123457, 98765432, 5550123, 777777], np.uint32)
    c0, c1 = np.float32(0.5), np.float32(2.0)
    D, H, W = 3, 4, 5
    vox = (rng.uniform(1.0, 1.3, (D, H, W)) * (c0 + 3 * c1)).astype(np.float32)
    sph = np.stack([vox, rng.uniform(0.5, 2.5, (D, H, W)).astype(np.float32)], -1).astype(np.float32)
    env = np.array([0.3, 0.6, 0.9], np.float32)
    identity = np.array([1, 0, 0, 0, 1, 0, 0, 0, 1, 0, 0, 0], np.float32)
    scaled = np.array([2, 0, 0, 0, 0.5, 0, 0, 0, 4, 0.25, -0.5, 1.0], np.float32)
    # (field kind, g, albedo, max bounces, transform)
    cases = [(0, 0.0, (0.9, 0.8, 0.7), 32, 0), (0, 0.6, (0.95, 0.9, 0.99), 8, 0), (0, -0.4, (1, 1, 1), 3, 1),
             (1, 0.0, (0.9, 0.8, 0.7), 32, 0), (1, 0.6, (0.95, 0.9, 0.99), 8, 1), (1, 0.0005, (0.5, 0.5, 0.5), 0, 0)]
    kinds = np.array([c[0] for c in cases], np.int32)
    gs = np.array([c[1] for c in cases], np.float32)
    albedos = np.array([c[2] for c in cases], np.float32)
    bounces = np.array([c[3] for c in cases], np.int32)
    transforms = np.stack([identity, scaled])[[c[4] for c in cases]].astype(np.float32)
    out = np.zeros((len(cases), n, 3), np.float32)
    for k, (kind, g, alb, mb, _) in enumerate(cases):
        grid = vox if kind == 0 else sph
        lib.ref_pbvr(ctypes.c_float(c0), ctypes.c_float(c1), int(kind), ptr(grid), D, H, W, ptr(env),
                     ptr(np.ascontiguousarray(transforms[k])), ptr(np.ascontiguousarray(albedos[k])),
                     ctypes.c_float(g), int(mb), ptr(seeds), ptr(rays), n, ptr(out[k]))
    hg_g = np.array([0.0, 0.0005, 0.3, -0.7, 0.95], np.float32)
    hg_w = rng.standard_normal((24, 3)).astype(np.float32)
    hg_w /= np.linalg.norm(hg_w, axis=1, keepdims=True)
    hg_w[0] = [0.0, 0.0, 1.0]
    hg_w[1] = [0.0, 0.0, -1.0]
    hg_w = hg_w.astype(np.float32)
    hg_index = rng.integers(0, 1 << 20, size=24).astype(np.int64)
    hg_out = np.zeros((hg_g.size, 24, 3), np.float32)
    for a, g in enumerate(hg_g):
        for i in range(24):
            lib.ref_hg_phase_sample(ptr(seeds), int(hg_index[i]), 3, ptr(np.ascontiguousarray(hg_w[i])),
                                    ctypes.c_float(g), ptr(hg_out[a, i]))
    # PBVRT (variant 0, [n, 4]) and PBVR_NEE (variant 1, [n, 3]) on the same
    # rays, fields and media: (variant, field kind, g, albedo, max bounces,
    # density scale, transform)
    light_dir = np.array([0.3, 1.0, -0.2], np.float32)
    light_int = np.array([2.0, 1.5, 1.0], np.float32)
    t_cases = [(0, 0, 0.0, (0.9, 0.8, 0.7), 32, 1.0, 0), (0, 1, 0.6, (0.95, 0.9, 0.99), 3, 0.5, 1),
               (0, 0, -0.4, (1, 1, 1), 0, 2.0, 0), (1, 1, 0.0, (0.9, 0.8, 0.7), 32, 1.0, 0),
               (1, 0, 0.3, (0.8, 0.8, 0.8), 6, 1.5, 1)]
    t_out = np.zeros((len(t_cases), n, 4), np.float32)
    for k, (var, kind, g, alb, mb, dsc, ti) in enumerate(t_cases):
        grid = vox if kind == 0 else sph
        dst = np.zeros((n, 4 if var == 0 else 3), np.float32)
        lib.ref_pbvrt(int(var), ctypes.c_float(c0), ctypes.c_float(c1), int(kind), ptr(grid), D, H, W, ptr(env),
                      ptr(np.ascontiguousarray([identity, scaled][ti])), ptr(np.array(alb, np.float32)),
                      ptr(light_dir), ptr(light_int), ctypes.c_float(g), ctypes.c_float(dsc), int(mb), ptr(seeds),
                      ptr(rays), n, ptr(dst))
        t_out[k, :, :dst.shape[1]] = dst
    # PBVR_ENV: an XREnvironmentSampler quadtree (4 levels, from a skewed
    # density image) over the constant environment; (field kind, g, max
    # bounces, density scale)
    e_levels = 4
    e_image = (rng.uniform(0, 1, (1 << e_levels, 1 << e_levels)) ** 4).astype(np.float32)
    from oracle.raymarch import xr_quadtree
    e_tree = xr_quadtree(e_image, e_levels).astype(np.float32)
    e_cases = [(0, 0.0, 32, 1.0), (1, 0.5, 4, 0.7)]
    e_out = np.zeros((len(e_cases), n, 3), np.float32)
    for k, (kind, g, mb, dsc) in enumerate(e_cases):
        grid = vox if kind == 0 else sph
        lib.ref_pbvr_env(ctypes.c_float(c0), ctypes.c_float(c1), int(kind), ptr(grid), D, H, W, ptr(env),
                         ptr(identity), ptr(np.array((0.9, 0.8, 0.7), np.float32)), ptr(e_tree), e_levels,
                         ctypes.c_float(g), ctypes.c_float(dsc), int(mb), ptr(seeds), ptr(rays), n, ptr(e_out[k]))
    t_params = np.array([[c[0], c[1], c[2], c[4], c[5], c[6]] for c in t_cases], np.float32)
    t_albedo = np.array([c[3] for c in t_cases], np.float32)
    np.savez_compressed(os.path.join(HERE, "pbvr.npz"), rays=rays, seeds=seeds, c0=c0, c1=c1, vox=vox, sph=sph,
                        env=env, kinds=kinds, g=gs, albedo=albedos, max_bounces=bounces, transforms=transforms,
                        out=out, hg_g=hg_g, hg_w=hg_w, hg_index=hg_index, hg_draws_before=np.int32(3),
                        hg_out=hg_out, t_params=t_params, t_albedo=t_albedo, t_transforms=np.stack([identity, scaled]),
                        t_light_dir=light_dir, t_light_int=light_int, t_out=t_out, e_levels=np.int32(e_levels),
                        e_image=e_image, e_tree=e_tree, e_params=np.array(e_cases, np.float32), e_out=e_out)


GRID_CASES = ((1, 3, (7,)), (2, 3, (5, 9)), (3, 3, (4, 5, 6)), (4, 3, (3, 4, 2, 5)), (3, 5, (2, 3, 1)))


def sampler_goldens():
    """grid_sampler.npz: GridSampler.forward of the reference
    (samplers/grid_sampler.h) over dense grids, for every (clamp, aligned,
    linear) and the (IN, OUT) pairs of GRID_CASES; points in [-1.3, 1.3]^IN
    (outside the grid too) with the exact -1, 0, 1 and cell-centre
    coordinates first."""
    lib = ref_samplers_lib()
    rng = np.random.default_rng(2027)
    out = {}
    n = 256
    for c, (IN, OUT, shape) in enumerate(GRID_CASES):
        t = rng.standard_normal(tuple(shape) + (OUT,)).astype(np.float32)
        x = rng.uniform(-1.3, 1.3, (n, IN)).astype(np.float32)
        x[:8] = np.float32([-1, 1, 0, -1.0, 1.0, 0.5, -0.5, 0.25])[:, None]
        ys = np.zeros((8, n, OUT), np.float32)
        for f in range(8):
            clamp, aligned, linear = f & 1, (f >> 1) & 1, (f >> 2) & 1
            rc = lib.ref_grid_sampler(IN, OUT, ptr(np.array(shape, np.int32)), ptr(t), clamp, aligned, linear,
                                      ptr(x), n, ptr(ys[f]))
            assert rc == 0
        out.update({f"t{c}": t, f"x{c}": x, f"y{c}": ys})
    np.savez_compressed(os.path.join(HERE, "grid_sampler.npz"), **out)


if __name__ == "__main__":
    if sys.argv[1:] == ["coopmat"]:
        coopmat_goldens()
    elif sys.argv[1:] == ["pbvr"]:
        pbvr_goldens()
    elif sys.argv[1:] == ["samplers"]:
        sampler_goldens()
    else:
        main()
