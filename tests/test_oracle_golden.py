"""Pins the CPU oracle against golden vectors produced by the reference's own
code (tests/golden/make_golden.py). Runs without a GPU."""
import numpy as np
import pytest

from oracle import mlp as omlp
from oracle import raymarch as orm
from oracle import tensors as oten
from oracle import winograd as owg
from oracle._clib import ref_lib, ref_lib_available


def _layers_from(g, n, relu_last=False, math="f32"):
    return [{"W": g[f"W{i}"], "b": g[f"b{i}"], "math": math, "relu": (i < n - 1) or relu_last} for i in range(n)]


def test_c_oracle_fp32_chain_is_bit_exact_vs_reference_composite(golden):
    g = golden("mlp_c1.npz")
    y = omlp.mlp_forward(g["x"], _layers_from(g, 4))
    np.testing.assert_array_equal(y, g["y"])


def test_c_oracle_odd_widths_bit_exact(golden):
    g = golden("mlp_small.npz")
    y = omlp.mlp_forward(g["x"], _layers_from(g, 2))
    np.testing.assert_array_equal(y, g["y"])


def test_fp32_oracle_f64_agrees_within_fp32_tolerance(golden):
    g = golden("mlp_c1.npz")
    y = omlp.mlp_forward_f64(g["x"], _layers_from(g, 4))
    assert omlp.within_tolerance(g["y"], y, 1e-5)


def test_linear_tensor_op_matches_reference(golden):
    g = golden("tensor_ops.npz")
    layers = [{"W": g["lin_W"], "b": g["lin_b"], "math": "f32", "relu": False}]
    y = omlp.mlp_forward(g["lin_x"], layers)
    # LinearTensorOp seeds acc with bias and accumulates k ascending in 8-wide
    # chunks -- the same sequence as the Map path, so bit-exact.
    np.testing.assert_array_equal(y, g["lin_y"])
    np.testing.assert_array_equal(np.maximum(g["relu_x"], 0), g["relu_y"])


def test_direct_conv_oracle_matches_reference_conv2d_tensor_op(golden):
    g = golden("tensor_ops.npz")
    x = g["conv_x"].reshape(1, 16, 16, 16)
    y = owg.conv3x3_direct(x, g["conv_w"], g["conv_b"]).reshape(256, 32)
    nw, el = omlp.rel_errors(g["conv_y"], y)
    assert nw < 1e-6 and el < 1e-5, (nw, el)


def test_winograd_scalar_transforms_bit_exact(golden):
    g = golden("winograd.npz")
    np.testing.assert_array_equal(owg.winograd_fwd_f23(g["d"]), g["V"])
    np.testing.assert_array_equal(owg.winograd_inv_f23(g["M"]), g["Y"])
    # the matrix form used by the batched oracle is the same linear map
    d = g["d"].astype(np.float64).reshape(-1, 4, 4)
    V = np.einsum("ij,njk,lk->nil", owg.BT_F23, d, owg.BT_F23).reshape(-1, 16)
    np.testing.assert_allclose(V, g["V"], rtol=0, atol=1e-5)
    M = g["M"].astype(np.float64).reshape(-1, 4, 4)
    Y = np.einsum("pi,nij,qj->npq", owg.AT_F23, M, owg.AT_F23).reshape(-1, 4)
    np.testing.assert_allclose(Y, g["Y"], rtol=0, atol=1e-5)


def test_winograd_filter_transform_matches_reference_torch_helper(golden):
    g = golden("winograd.npz")
    np.testing.assert_array_equal(owg.G_F23, g["G"])
    U = owg.filter_transform(g["w"], "F2x2")
    np.testing.assert_array_equal(U.reshape(-1).astype(np.float16), g["U"])


@pytest.mark.parametrize("variant", ["F2x2", "F4x4"])
def test_winograd_identity_in_float64(variant):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 8, 12, 16)).astype(np.float32)
    w = (rng.standard_normal((3, 3, 16, 8)) * 0.1).astype(np.float32)
    b = rng.standard_normal(8).astype(np.float32)
    d = owg.conv3x3_direct(x, w, b)
    y = owg.conv3x3_winograd(x, w, b, variant, staged=False)
    np.testing.assert_allclose(y, d, rtol=0, atol=1e-12)


def test_toom_cook_reproduces_reference_f23_matrices():
    AT, G, BT = owg.toom_cook_matrices([0.0, 1.0, -1.0], 2)
    # same transforms up to the sign convention of the first point's row
    np.testing.assert_allclose(np.abs(AT), np.abs(owg.AT_F23))
    np.testing.assert_allclose(np.abs(G), np.abs(owg.G_F23))
    np.testing.assert_allclose(np.abs(BT), np.abs(owg.BT_F23))


def test_transmittance_restatement_matches_reference(golden):
    g = golden("transmittance.npz")
    T = np.empty_like(g["T"])
    for i in range(T.shape[0]):
        c0, c1 = g["c0"][i], g["c1"][i]

        def ext(p, c0=c0, c1=c1):
            return np.float32(c0) + np.float32(c1) * np.sum(p * p, axis=-1, dtype=np.float32)

        T[i] = orm.transmittance_rm(g["x"][i:i + 1], g["w"][i:i + 1], g["d"][i:i + 1], g["step"], g["scale"], ext)[0]
    np.testing.assert_allclose(T, g["T"], rtol=2e-6, atol=1e-7)
    assert np.all(T[4:8] == 0.0)


def test_generator_restatement_is_bit_exact(golden):
    """random_spawn + random() of the oracle against the reference's own
    random_library.h (64 draws for 8 invocation indices)."""
    g = golden("ratiotracking.npz")
    st = orm.random_spawn(g["seeds"], g["rng_index"])
    draws = np.stack([orm.random_draw(st) for _ in range(64)], axis=1)
    np.testing.assert_array_equal(draws, g["rng_draws"])
    assert np.all((draws >= 0) & (draws < 1))


def test_ratiotracking_restatement_matches_reference(golden):
    """transmittance_rt over the fixture's ray segments: the same random
    draws, collisions, Russian-roulette outcomes and values, bit for bit, as
    the reference's own loop (compiled with its floating literals as float,
    as GLSL reads them)."""
    g = golden("ratiotracking.npz")
    for m, (c0, c1, _, ds) in enumerate(g["media"]):
        def ext(p, c0=c0, c1=c1):
            return (np.float32(c0) + np.float32(c1) * ((p[:, 0] * p[:, 0] + p[:, 1] * p[:, 1]) + p[:, 2] * p[:, 2])
                    ).astype(np.float32)

        grid = g["grids"][m]
        state = orm.random_spawn(g["seeds"], g["index"][m])
        T = orm.transmittance_rt(g["x"][m], g["w"][m], g["d"][m], ds, ext,
                                 lambda x, w: orm.voxel_majorant(grid, x, w), state)
        ref = g["T"][m]
        np.testing.assert_array_equal(T, ref)
        np.testing.assert_array_equal(T == 0, ref == 0)
        np.testing.assert_array_equal(T == 1, ref == 1)
    assert (g["T"] == 0).any() and ((g["T"] > 0) & (g["T"] < 1)).any()


@pytest.mark.skipif(not ref_lib_available(), reason="reference shader library not built")
def test_live_reference_library_agrees_with_fixture(golden):
    """Where oracle/_ref is present, re-run one fixture through it."""
    g = golden("mlp_small.npz")
    from oracle._clib import ptr, ptr_array

    y = np.zeros_like(g["y"])
    ref_lib().ref_mlp_small(ptr(g["x"]), g["x"].shape[0], ptr_array([g["W0"], g["W1"]]),
                            ptr_array([g["b0"], g["b1"]]), ptr(y))
    np.testing.assert_array_equal(y, g["y"])


def test_fp16_staging_semantics():
    """LinearFast: products of float16-staged operands summed in fp32 from 0,
    bias added after; the trailing partial 32-row workgroup runs fp32."""
    rng = np.random.default_rng(3)
    layers = [{"W": rng.standard_normal((16, 8)).astype(np.float32), "b": rng.standard_normal(16).astype(np.float32),
               "math": "f16", "relu": True},
              {"W": rng.standard_normal((4, 16)).astype(np.float32), "b": rng.standard_normal(4).astype(np.float32),
               "math": "f16", "relu": False}]
    x = rng.standard_normal((70, 8)).astype(np.float32)
    y = omlp.mlp_forward(x, layers, tail_exact=True)
    ref16 = omlp.mlp_forward_f64(x, layers)
    f32_layers = [dict(l, math="f32") for l in layers]
    ref32 = omlp.mlp_forward_f64(x, f32_layers)
    assert omlp.within_tolerance(y[:64], ref16[:64], 1e-5)
    assert omlp.within_tolerance(y[64:], ref32[64:], 1e-5)
    # the f16 rows really differ from exact fp32
    assert not np.allclose(y[:64], ref32[:64], rtol=1e-6, atol=0)


def test_camera_rays_geometry():
    pose = orm.orbit_pose(0)
    o, w = orm.camera_rays(pose, 8, 6)
    assert o.shape == (48, 3) and w.shape == (48, 3)
    np.testing.assert_allclose(np.linalg.norm(w, axis=1), 1.0, atol=1e-6)
    # centre of the image looks at the target (the origin)
    centre = (w[2 * 8 + 3] + w[2 * 8 + 4] + w[3 * 8 + 3] + w[3 * 8 + 4]) / 4
    to_target = -pose[:3] / np.linalg.norm(pose[:3])
    assert np.dot(centre / np.linalg.norm(centre), to_target) > 0.99


def test_resample_and_concat_restatements_bit_exact_vs_reference(golden):
    g = golden("resample.npz")
    np.testing.assert_array_equal(oten.downsample2x(g["down_x"], 8, 12), g["down_y"])
    np.testing.assert_array_equal(oten.upsample2x(g["up_x"], 4, 6), g["up_y"])
    np.testing.assert_array_equal(oten.concat(g["cat_x1"], g["cat_x2"]), g["cat_y"])


@pytest.mark.parametrize("in_dim", [2, 3])
@pytest.mark.parametrize("clamp,aligned,linear", [(True, False, True), (False, False, True), (True, True, True),
                                                  (False, True, True), (True, False, False), (False, True, False)])
def test_tensor_sampler_restatement_matches_torch_grid_sample(in_dim, clamp, aligned, linear):
    """The reference documents TensorSampler as torch's grid_sample
    (align_corners = aligned, padding border / zeros = clamp); the
    restatement is checked against it on points spilling past the borders."""
    import torch
    import torch.nn.functional as F

    rng = np.random.default_rng(in_dim * 10 + clamp + 2 * aligned + 4 * linear)
    shape = (5, 7, 4) if in_dim == 2 else (4, 6, 5, 3)
    t = rng.standard_normal(shape).astype(np.float32)
    x = rng.uniform(-1.3, 1.3, size=(500, in_dim)).astype(np.float32)
    got = oten.tensor_sampler(t, x, clamp, aligned, linear)
    tt = torch.from_numpy(t).permute(in_dim, *range(in_dim)).unsqueeze(0)
    grid = torch.from_numpy(x).reshape((1, 500) + (1,) * (in_dim - 1) + (in_dim,))
    ref = F.grid_sample(tt, grid, mode="bilinear" if linear else "nearest",
                        padding_mode="border" if clamp else "zeros", align_corners=aligned)
    ref = ref.reshape(t.shape[-1], 500).T.numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


# ---------------------------------------------------------------------------
# The float16 (cooperative-matrix) paths: tests/golden/coopmat.npz holds the
# outputs of the reference's own coopmat bodies executed on the CPU
# (oracle/ref_shim/ref_coopmat.cpp; coopMatMulAdd sums in ascending k in
# fp32). The restatements must reproduce them bit for bit.
def _cm_chain(g, name):
    n = len([k for k in g if k.startswith(f"{name}_W")])
    Ws = [g[f"{name}_W{i}"] for i in range(n)]
    Ws = [w.astype(np.float32) / 128.0 if w.dtype == np.int8 else w for w in Ws]
    return [{"W": Ws[i], "b": g[f"{name}_b{i}"], "math": "f16", "relu": i < n - 1} for i in range(n)]


@pytest.mark.parametrize("name", ["c5", "c2"])
def test_linear_fast_chain_bit_exact_vs_reference_coopmat(golden, name):
    """LinearFast >> relu >> ... (maps/linear_fast.h:39-98 through
    cooperative_library.h's gate): float16 staging, fp32 sums from 0, bias
    after; the trailing partial workgroup in exact fp32."""
    g = golden("coopmat.npz")
    layers = _cm_chain(g, name)
    x = g[f"{name}_x"]
    assert x.shape[0] % 32 != 0  # the fixture includes a partial workgroup
    y = omlp.mlp_forward(x, layers, tail_exact=True)
    np.testing.assert_array_equal(y, g[f"{name}_y"])
    # without the tail rule the partial workgroup's rows differ (they are the
    # reference's scalar fp32 rows), the full workgroups' do not
    full = (x.shape[0] // 32) * 32
    y2 = omlp.mlp_forward(x, layers, tail_exact=False)
    np.testing.assert_array_equal(y2[:full], g[f"{name}_y"][:full])
    assert not np.array_equal(y2[full:], g[f"{name}_y"][full:])


@pytest.mark.parametrize("name,bias_first", [("small_32_48", True), ("small_64_32", True), ("simple_32_64", True),
                                             ("fast_32_64", False), ("mine_32_48", False)])
def test_linear_tensor_ops_bit_exact_vs_reference_coopmat(golden, name, bias_first):
    """LinearTensorOpSmall/Simple seed their accumulators with the bias
    (linear_tensor_op_small.h:99, linear_tensor_op_simple.h); Fast/Mine add
    it after (linear_tensor_op_fast.h, linear_tensor_op_mine.h)."""
    g = golden("coopmat.npz")
    layer = {"W": g[f"{name}_W"], "b": g[f"{name}_b"], "math": "f16", "relu": False, "bias_first": bias_first}
    y = omlp.mlp_forward(g[f"{name}_x"], [layer])
    np.testing.assert_array_equal(y, g[f"{name}_y"])
    # the other order is a different (fp32-rounding-level) result
    other = dict(layer, bias_first=not bias_first)
    y2 = omlp.mlp_forward(g[f"{name}_x"], [other])
    assert not np.array_equal(y2, g[f"{name}_y"])
    assert omlp.within_tolerance(y2, g[f"{name}_y"], 1e-6)


@pytest.mark.parametrize("c", [16, 48])
def test_winograd_op_bit_exact_vs_reference_coopmat(golden, c):
    """Conv2DTensorOpWinograd3x3.forward (conv2d_tensor_op_winograd3x3.h:
    95-177) with the float16 filter image of the reference's own
    _winograd_transform_weight: the ordered fp32 restatement reproduces it
    bit for bit, the float64-GEMM restatement within 1e-6."""
    g = golden("coopmat.npz")
    x, w, b = g[f"wino{c}_x"][None], g[f"wino{c}_w"].astype(np.float32), g[f"wino{c}_b"]
    U = owg.filter_transform(w, "F2x2")
    y = owg.conv3x3_winograd_f23_ordered(x, U, b)[0]
    np.testing.assert_array_equal(y, g[f"wino{c}_y"])
    y64 = owg.conv3x3_winograd(x, w, b, "F2x2", staged=True)[0]
    assert omlp.within_tolerance(y64, g[f"wino{c}_y"], 1e-6)
    # and the float16 Winograd is within the BASELINE fp16 tolerance of the direct convolution
    assert omlp.within_tolerance(g[f"wino{c}_y"], owg.conv3x3_direct(x, w, b)[0], 1e-2)


def test_live_reference_coopmat_library_agrees_with_fixture(golden):
    """Where the reference checkout is present, its coopmat bodies rerun on
    the fixture's inputs give the stored outputs."""
    if not ref_lib_available():
        pytest.skip("reference checkout not present")
    from oracle._clib import ptr, ptr_array, ref_coopmat_lib

    g = golden("coopmat.npz")
    lib = ref_coopmat_lib()
    for name in ("c5", "c2"):
        layers = _cm_chain(g, name)
        x = g[f"{name}_x"]
        y = np.zeros_like(g[f"{name}_y"])
        Ws = [np.ascontiguousarray(l["W"], dtype=np.float32) for l in layers]
        bs = [np.ascontiguousarray(l["b"]) for l in layers]
        getattr(lib, f"ref_cm_mlp_{name}")(ptr(x), x.shape[0], ptr_array(Ws), ptr_array(bs), ptr(y))
        np.testing.assert_array_equal(y, g[f"{name}_y"])
    x, b = g["small_64_32_x"], g["small_64_32_b"]
    W = np.ascontiguousarray(g["small_64_32_W"])
    y = np.zeros_like(g["small_64_32_y"])
    lib.ref_cm_small_64_32(ptr(x), x.shape[0], ptr(W), ptr(b), ptr(y))
    np.testing.assert_array_equal(y, g["small_64_32_y"])


def _pbvr_case(g, k):
    c0, c1 = np.float32(g["c0"]), np.float32(g["c1"])

    def ext(p):
        return (c0 + c1 * ((p[:, 0] * p[:, 0] + p[:, 1] * p[:, 1]) + p[:, 2] * p[:, 2])).astype(np.float32)

    if int(g["kinds"][k]) == 0:
        field = lambda x, w: orm.voxel_majorant(g["vox"], x, w)  # noqa: E731
    else:
        field = lambda x, w: orm.sphere_majorant(g["sph"], x, w)  # noqa: E731
    rays = g["rays"]
    return orm.pbvr(rays[:, :3], rays[:, 3:], ext, orm.constant_environment(g["env"]), field, g["seeds"],
                    transform=g["transforms"][k], albedo=g["albedo"][k], g=float(g["g"][k]),
                    max_bounces=int(g["max_bounces"][k]))


@pytest.mark.parametrize("k", range(6))
def test_pbvr_restatement_bit_exact_vs_reference(golden, k):
    """PBVR.forward (volumes/pbvr.h) of the oracle against the reference's
    own body compiled as C++ (voxel and sphere majorant fields, isotropic
    and forward/backward scattering, bounce budgets 0..32, an identity and
    a scaled + shifted transform): the same draws, collisions, directions
    and radiance on every ray."""
    g = golden("pbvr.npz")
    got = _pbvr_case(g, k)
    np.testing.assert_array_equal(got, g["out"][k])
    o, w = orm.object_space(g["rays"][:, :3], g["rays"][:, 3:], g["transforms"][k])
    tmin, tmax = orm.ray_box(o, w)
    miss = (tmax <= 0) | (tmin > tmax)
    assert miss.any()
    np.testing.assert_array_equal(g["out"][k][miss], np.broadcast_to(g["env"], (int(miss.sum()), 3)))


def test_pbvr_fixture_covers_the_path_outcomes(golden):
    """The fixture's paths reach every outcome: misses (environment), escapes
    after scattering (attenuated environment) and terminations (0)."""
    g = golden("pbvr.npz")
    out, env = g["out"], g["env"]
    assert (out == 0).all(axis=2).any()
    assert (out == env).all(axis=2).any()
    partial = (out > 0).all(axis=2) & (out < env).all(axis=2)
    assert partial.any()
    assert (out[5] <= env).all()   # max_bounces 0: no scattering survives


def test_hg_phase_sample_bit_exact_vs_reference(golden):
    """hg_phase_sample (random_library.h:224-239) of the oracle against the
    reference's own function, after 3 draws of each invocation's generator."""
    g = golden("pbvr.npz")
    for a, gg in enumerate(g["hg_g"]):
        st = orm.random_spawn(g["seeds"], g["hg_index"])
        for _ in range(int(g["hg_draws_before"])):
            orm.random_step(st)
        got = orm.hg_phase_sample(g["hg_w"], float(gg), st)
        np.testing.assert_array_equal(got, g["hg_out"][a])
        np.testing.assert_allclose(np.linalg.norm(got.astype(np.float64), axis=1), 1.0, atol=1e-5)


def test_live_reference_pbvr_library_agrees_with_fixture(golden):
    """Where the reference checkout is present, its PBVR body rerun on the
    fixture's first case gives the stored radiance."""
    if not ref_lib_available():
        pytest.skip("reference checkout not present")
    from oracle._clib import ptr, ref_pbvr_lib
    import ctypes

    g = golden("pbvr.npz")
    out = np.zeros_like(g["out"][0])
    ref_pbvr_lib().ref_pbvr(ctypes.c_float(g["c0"]), ctypes.c_float(g["c1"]), 0, ptr(g["vox"]), 3, 4, 5,
                            ptr(g["env"]), ptr(np.ascontiguousarray(g["transforms"][0])),
                            ptr(np.ascontiguousarray(g["albedo"][0])), ctypes.c_float(g["g"][0]),
                            int(g["max_bounces"][0]), ptr(g["seeds"]), ptr(g["rays"]), g["rays"].shape[0], ptr(out))
    np.testing.assert_array_equal(out, g["out"][0])


_GRID_PAIRS = ((1, 3), (2, 3), (3, 3), (4, 3), (3, 5))


@pytest.mark.parametrize("c", range(len(_GRID_PAIRS)))
def test_grid_sampler_restatement_bit_exact_vs_reference(golden, c):
    """GridSampler.forward (samplers/grid_sampler.h) of the oracle against
    the reference's own body, every (clamp, aligned, linear), IN 1..4."""
    g = golden("grid_sampler.npz")
    t, x, ys = g[f"t{c}"], g[f"x{c}"], g[f"y{c}"]
    assert (t.ndim - 1, t.shape[-1]) == _GRID_PAIRS[c]
    for f in range(8):
        got = oten.grid_sampler(t, x, clamp=bool(f & 1), aligned=bool(f & 2), linear=bool(f & 4))
        np.testing.assert_array_equal(got, ys[f], err_msg=f"flags {f}")


def test_grid_and_tensor_samplers_round_differently(golden):
    """The two samplers agree to rounding on the same tensor but are not the
    same arithmetic (positions t D - 0.5 against (x (D - a) + D) 0.5 - 0.5,
    bit-mask corner weights against paired lerps), as in the reference."""
    g = golden("grid_sampler.npz")
    t, x = g["t2"], g["x2"]
    a = oten.grid_sampler(t, x)
    b = oten.tensor_sampler(t, x)
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-5)
    assert not np.array_equal(a, b)


def test_live_reference_samplers_library_agrees_with_fixture(golden):
    if not ref_lib_available():
        pytest.skip("reference checkout not present")
    from oracle._clib import ptr, ref_samplers_lib

    g = golden("grid_sampler.npz")
    t, x = g["t2"], g["x2"]
    y = np.zeros_like(g["y2"][7])
    assert ref_samplers_lib().ref_grid_sampler(3, 3, ptr(np.array(t.shape[:3], np.int32)), ptr(t), 1, 1, 1, ptr(x),
                                               x.shape[0], ptr(y)) == 0
    np.testing.assert_array_equal(y, g["y2"][7])


@pytest.mark.parametrize("k", range(5))
def test_pbvrt_and_nee_restatement_bit_exact_vs_reference(golden, k):
    """PBVRT.forward (volumes/pbvrt.h, RGB + alpha) and PBVR_NEE.forward
    (volumes/pbvr_nee.h) of the oracle against the reference's own bodies:
    next-event estimation with its ratio-tracking shadow rays, voxel and
    sphere fields, density scales, bounce budgets 0..32, an identity and a
    scaled + shifted transform -- every value bit for bit."""
    g = golden("pbvr.npz")
    var, kind, gg, mb, dsc, ti = g["t_params"][k]
    c0, c1 = np.float32(g["c0"]), np.float32(g["c1"])

    def ext(p):
        return (c0 + c1 * ((p[:, 0] * p[:, 0] + p[:, 1] * p[:, 1]) + p[:, 2] * p[:, 2])).astype(np.float32)

    if int(kind) == 0:
        field = lambda x, w: orm.voxel_majorant(g["vox"], x, w)  # noqa: E731
    else:
        field = lambda x, w: orm.sphere_majorant(g["sph"], x, w)  # noqa: E731
    rays = g["rays"]
    got = orm.pbvrt(rays[:, :3], rays[:, 3:], ext, field, g["seeds"], g["t_albedo"][k], g["t_light_dir"],
                    g["t_light_int"], orm.constant_environment(g["env"]), transform=g["t_transforms"][int(ti)],
                    density_scale=float(dsc), g=float(gg), max_bounces=int(mb),
                    variant="pbvrt" if int(var) == 0 else "nee")
    ref = g["t_out"][k][:, :got.shape[1]]
    np.testing.assert_array_equal(got, ref)
    if int(var) == 0:
        assert set(np.unique(ref[:, 3])) <= {0.0, 1.0}


@pytest.mark.parametrize("k", range(2))
def test_pbvr_env_restatement_bit_exact_vs_reference(golden, k):
    """PBVR_ENV.forward (volumes/pbvr_env.h) with the XREnvironmentSampler
    (rendering/xr_environment_sampler.h) of the oracle against the
    reference's own bodies, on the fixture's quadtree: bit for bit."""
    g = golden("pbvr.npz")
    kind, gg, mb, dsc = g["e_params"][k]
    c0, c1 = np.float32(g["c0"]), np.float32(g["c1"])

    def ext(p):
        return (c0 + c1 * ((p[:, 0] * p[:, 0] + p[:, 1] * p[:, 1]) + p[:, 2] * p[:, 2])).astype(np.float32)

    field = (lambda x, w: orm.voxel_majorant(g["vox"], x, w)) if int(kind) == 0 else \
        (lambda x, w: orm.sphere_majorant(g["sph"], x, w))
    rays = g["rays"]
    got = orm.pbvrt(rays[:, :3], rays[:, 3:], ext, field, g["seeds"], (0.9, 0.8, 0.7), None,
                    environment=orm.constant_environment(g["env"]), density_scale=float(dsc), g=float(gg),
                    max_bounces=int(mb), variant="env", env_densities=g["e_tree"], env_levels=int(g["e_levels"]))
    np.testing.assert_array_equal(got, g["e_out"][k])
    assert (got.sum(1) > 0).mean() > 0.5


def test_xr_quadtree_layout():
    """The quadtree of rendering.py:175-278: 4 (4^L - 1) / 3 values,
    cumulative per node (non-decreasing, the last exactly 1), and the
    product of the chosen children's probabilities along each leaf's path
    equal to that leaf's normalised, solid-angle-weighted mass."""
    rng = np.random.default_rng(3)
    levels = 3
    img = rng.uniform(0, 1, (8, 8)) ** 3
    tree = orm.xr_quadtree(img, levels)
    assert tree.size == 4 * (4 ** levels - 1) // 3
    cum = tree.reshape(-1, 4)
    assert np.all(np.diff(cum, axis=1) >= -1e-15) and np.all(cum[:, 3] == 1.0)
    res = 1 << levels
    w = np.sin(((np.arange(res) + 1) / res * 2 - 1) * np.pi / 2) - np.sin((np.arange(res) / res * 2 - 1) * np.pi / 2)
    mass = img * w[:, None]
    mass = mass / mass.sum()
    for row in range(res):
        for col in range(res):
            node, prob = 0, 1.0
            for d in range(levels - 1, -1, -1):
                c = 2 * ((row >> d) & 1) + ((col >> d) & 1)
                cdf = tree[node * 4:node * 4 + 4]
                prob *= cdf[c] - (cdf[c - 1] if c else 0.0)
                node = node * 4 + 1 + c
            assert abs(prob - mass[row, col]) <= 1e-12
