"""GPU parity of PBVR (rdv/domain/volumes.py:257-326) and the
SphereMajorantField (volumes.py:215-224) against the CPU oracle
(oracle/raymarch.py: pbvr, sphere_majorant), whose delta-tracking loop,
majorant fields and Henyey-Greenstein sampler are pinned bit-exact to the
reference's own pbvr.h / random_library.h by tests/golden/pbvr.npz.

Both sides draw the same random numbers (ray i uses the dispatch seeds
spawned by index i), so the paths agree ray by ray. They may part where a
last-bit difference flips a decision: the GPU's logf, sinf, cosf, asinf and
atan2f against the oracle's correctly rounded ones, and fused against
separately rounded fp32 products in exact (Linear) extinction chains. The
tests therefore ask for agreement on almost every ray and for equal means;
the estimator itself is checked against properties that hold exactly (a
white furnace: albedo 1 and a constant environment give the environment on
every escaped path) and statistically (with albedo 0 its mean is the transmittance
times the environment; the voxel and the sphere fields estimate the same
radiance).
"""
import numpy as np
import pytest
import torch

from oracle import raymarch as orm
from oracle import tensors as oten
from test_gpu_ratiotracking import SEEDS, _chain, _extinction, _layers, _majorant, _rays

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rdv():
    import rdv_project_b200 as rdv
    return rdv


def _sphere_grid(vox, seed=0):
    """A sphere majorant grid [D, H, W, 2] from a voxel one [D, H, W, 1]:
    radius 0.5 (the voxel itself) or 1.5 voxels (the voxel and its
    neighbours) per cell, the majorant the largest voxel majorant the box
    touches."""
    v = vox[..., 0]
    D, H, W = v.shape
    rng = np.random.default_rng(seed)
    radius = np.where(rng.random((D, H, W)) < 0.5, 0.5, 1.5).astype(np.float32)
    out = np.zeros((D, H, W, 2), np.float32)
    for k in range(D):
        for j in range(H):
            for i in range(W):
                r = 1 if radius[k, j, i] > 1 else 0
                out[k, j, i, 0] = v[max(k - r, 0):k + r + 1, max(j - r, 0):j + r + 1, max(i - r, 0):i + r + 1].max()
                out[k, j, i, 1] = radius[k, j, i]
    return out


def _env_image(seed=3, h=8, w=16):
    rng = np.random.default_rng(seed)
    return rng.uniform(0.1, 1.0, (h, w, 3)).astype(np.float32)


def _agree(got, ref, frac=0.98):
    """Ray-by-ray agreement on at least `frac` of the rays, and means within
    5 standard errors of the per-ray spread (the rays that part are
    independent samples of the same estimator)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    d = np.abs(got - ref)
    tol = 2e-5 + 1e-4 * np.abs(ref)
    close = float(np.mean(np.all(d <= tol, axis=1)))
    assert close >= frac, (close, np.nonzero(~np.all(d <= tol, axis=1))[0][:8])
    sem = ref.std(axis=0) / np.sqrt(ref.shape[0])
    assert np.all(np.abs(got.mean(axis=0) - ref.mean(axis=0)) <= 5 * sem + 1e-6), (got.mean(0), ref.mean(0), sem)
    return close


def _miss_mask(rays, transform=None):
    o, w = orm.object_space(rays[:, :3], rays[:, 3:], transform)
    tmin, tmax = orm.ray_box(o, w)
    return (tmax <= 0) | (tmin > tmax)


@pytest.mark.parametrize("math_,dims,field,env,g,albedo,bounces", [
    ("f32", [3, 32, 1], "voxel", "const", 0.0, (0.9, 0.8, 0.7), 32),
    ("f16", [3, 64, 64, 1], "sphere", "image", 0.6, (0.95, 0.9, 0.99), 8),
    ("bf16", [3, 48, 1], "voxel", "image", -0.4, (1.0, 1.0, 1.0), 3),
    ("f16", [3, 32, 1], "sphere", "const", 0.0005, (0.5, 0.6, 0.7), 0),
])
def test_pbvr_matches_oracle(rdv, cuda_device, math_, dims, field, env, g, albedo, bounces):
    n = 6000
    layers = _layers(dims, math_, seed=len(dims) * 7 + bounces)
    vox = _majorant(layers, (4, 3, 5))
    rays = _rays(n, seed=n + bounces)
    if field == "voxel":
        grid, fld = vox, rdv.VoxelMajorantField(torch.from_numpy(vox).to(cuda_device))
        maj = lambda x, w: orm.voxel_majorant(vox[..., 0], x, w)  # noqa: E731
    else:
        sph = _sphere_grid(vox)
        grid, fld = sph, rdv.SphereMajorantField(torch.from_numpy(sph).to(cuda_device))
        maj = lambda x, w: orm.sphere_majorant(sph, x, w)  # noqa: E731
    if env == "const":
        rgb = np.array([0.3, 0.6, 0.9], np.float32)
        environment, ref_env = rdv.Constant(rgb), orm.constant_environment(rgb)
    else:
        img = _env_image()
        environment = rdv.XRProject() >> rdv.TensorSampler(torch.from_numpy(img).to(cuda_device))
        ref_env = orm.equirect_environment(img)
    node = rdv.PBVR(_chain(rdv, layers, cuda_device), environment, fld, albedo=albedo, g=g, max_bounces=bounces)
    got = node(torch.from_numpy(rays).to(cuda_device), seeds=SEEDS).as_tensor("torch")
    torch.cuda.synchronize()
    assert tuple(got.shape) == (n, 3)
    got = got.cpu().numpy()
    ref, evals = orm.pbvr(rays[:, :3], rays[:, 3:], _extinction(layers), ref_env, maj, SEEDS, albedo=albedo, g=g,
                          max_bounces=bounces, return_evaluations=True)
    _agree(got, ref)
    miss = _miss_mask(rays)
    assert miss.any()
    if env == "const":
        assert np.all(got[miss] == ref_env(rays[miss, 3:]))       # misses see the environment exactly
    else:
        np.testing.assert_allclose(got[miss], ref[miss], rtol=1e-4, atol=1e-5)
    zero = (ref == 0).all(axis=1)
    assert zero.any() and (~zero & ~miss).any()                    # terminated and escaped paths
    gpu_evals = node.last_evaluations()
    assert abs(gpu_evals - evals) <= max(20, 0.02 * evals), (gpu_evals, evals)
    assert rdv.device_status() == 0


def test_transform_and_seeds(rdv, cuda_device):
    """A scaled, rotated, shifted volume; the same seeds give the same
    radiance twice; fresh seeds another sample."""
    layers = _layers([3, 32, 1], "f32", seed=5)
    vox = _majorant(layers, (2, 2, 2))
    c, s = np.cos(0.4), np.sin(0.4)
    M = np.array([[1.5 * c, 0, -1.5 * s], [0, 0.8, 0], [1.5 * s, 0, 1.5 * c]], dtype=np.float32)  # columns
    transform = np.concatenate([M.reshape(-1), np.array([0.3, -0.2, 0.1], np.float32)])
    rays = _rays(4000, seed=11, spread=4.0)
    rgb = np.array([1.0, 0.5, 0.25], np.float32)
    node = rdv.PBVR(_chain(rdv, layers, cuda_device), rdv.Constant(rgb), torch.from_numpy(vox).to(cuda_device),
                    transform=transform, albedo=(0.8, 0.8, 0.8), g=0.3)
    r = torch.from_numpy(rays).to(cuda_device)
    a = node(r, seeds=SEEDS).as_tensor("torch").cpu().numpy()
    b = node(r, seeds=SEEDS).as_tensor("torch").cpu().numpy()
    assert np.array_equal(a, b)
    ref = orm.pbvr(rays[:, :3], rays[:, 3:], _extinction(layers), orm.constant_environment(rgb),
                   lambda x, w: orm.voxel_majorant(vox[..., 0], x, w), SEEDS, transform=transform,
                   albedo=(0.8, 0.8, 0.8), g=0.3)
    _agree(a, ref)
    c2 = node(r).as_tensor("torch").cpu().numpy()
    assert node.last_seeds != SEEDS and not np.array_equal(a, c2)


def test_white_furnace(rdv, cuda_device):
    """Albedo 1 and a constant environment: a path keeps throughput 1, so it
    returns the environment exactly when it escapes and 0 when it runs out
    of iterations (8192). The reference's own loop runs out on a few paths:
    a point on a voxel face with a grazing direction advances by the 1e-6
    floor of the step, below the float spacing of that coordinate, and
    stays on the face. At a full-size batch of 2^20 rays every output is exactly the
    environment or exactly 0, the environment on at least 99.5 % of rays,
    and on every 64th ray the GPU agrees with the oracle."""
    layers = _layers([3, 64, 64, 1], "f16", seed=9, out_bias=1.0)
    vox = _majorant(layers, (6, 5, 4))
    sph = _sphere_grid(vox, seed=4)
    rays = _rays(1 << 20, seed=77)
    sub = np.arange(0, rays.shape[0], 64)
    rgb = np.array([0.25, 0.5, 1.0], np.float32)
    fields = ((rdv.VoxelMajorantField(torch.from_numpy(vox).to(cuda_device)),
               lambda x, w: orm.voxel_majorant(vox[..., 0], x, w)),
              (rdv.SphereMajorantField(torch.from_numpy(sph).to(cuda_device)),
               lambda x, w: orm.sphere_majorant(sph, x, w)))
    for fld, maj in fields:
        node = rdv.PBVR(_chain(rdv, layers, cuda_device), rdv.Constant(rgb), fld, albedo=(1, 1, 1), g=0.7,
                        max_bounces=100000)
        out = node(torch.from_numpy(rays).to(cuda_device), seeds=SEEDS).as_tensor("torch").cpu().numpy()
        env = np.all(out == rgb, axis=1)
        zero = np.all(out == 0, axis=1)
        assert np.all(env | zero)
        assert env.mean() >= 0.995, env.mean()
        assert node.last_evaluations() > rays.shape[0]               # the medium was crossed, not skipped
        ref = orm.pbvr(rays[sub, :3], rays[sub, 3:], _extinction(layers), orm.constant_environment(rgb), maj, SEEDS,
                       albedo=(1, 1, 1), g=0.7, max_bounces=100000, index=sub)
        assert np.mean(np.all(out[sub] == ref, axis=1)) >= 0.998
    assert rdv.device_status() == 0


def test_absorbing_medium_is_unbiased_against_the_fixed_step_march(rdv, cuda_device):
    """Albedo 0: a path's first real collision ends it with 0, so the mean
    of many samples is transmittance * environment, which the fixed-step
    RaymarchingTransmittance approximates with a small step. The voxel and
    the sphere fields both converge to it."""
    layers = _layers([3, 32, 1], "f32", seed=21, out_bias=0.3)
    ext = _chain(rdv, layers, cuda_device)
    vox = _majorant(layers, (3, 3, 3), margin=2.0)
    sph = _sphere_grid(vox, seed=8)
    base = _rays(64, seed=3)[16:]
    reps = 4096
    rays = torch.from_numpy(np.repeat(base, reps, axis=0)).to(cuda_device)
    rm = rdv.RaymarchingTransmittance(ext, step_size=0.001)
    T = rm(torch.from_numpy(base).to(cuda_device)).as_tensor("torch").cpu().numpy()[:, 0]
    rgb = np.array([1.0, 0.5, 2.0], np.float32)
    for fld in (rdv.VoxelMajorantField(torch.from_numpy(vox).to(cuda_device)),
                rdv.SphereMajorantField(torch.from_numpy(sph).to(cuda_device))):
        node = rdv.PBVR(ext, rdv.Constant(rgb), fld, albedo=(0, 0, 0))
        est = node(rays, seeds=SEEDS).as_tensor("torch").cpu().numpy().reshape(-1, reps, 3)
        for k in range(3):
            mean = est[..., k].mean(axis=1)
            sem = est[..., k].std(axis=1) / np.sqrt(reps)
            z = (mean - T * rgb[k]) / np.maximum(sem, 1e-4)
            assert np.all(np.abs(z) < 5.0), z
            assert np.abs(z).mean() < 1.5


def test_voxel_and_sphere_fields_estimate_the_same_radiance(rdv, cuda_device):
    """A scattering medium rendered with both fields: different paths, the
    same expectation (per-ray means over many samples agree)."""
    layers = _layers([3, 32, 1], "f16", seed=41, out_bias=0.5)
    ext = _chain(rdv, layers, cuda_device)
    vox = _majorant(layers, (4, 4, 4), margin=1.5)
    sph = _sphere_grid(vox, seed=2)
    base = _rays(48, seed=5)[12:]
    reps = 4096
    rays = torch.from_numpy(np.repeat(base, reps, axis=0)).to(cuda_device)
    img = torch.from_numpy(_env_image(seed=6)).to(cuda_device)
    env = rdv.XRProject() >> rdv.TensorSampler(img)
    means, sems = [], []
    for fld in (rdv.VoxelMajorantField(torch.from_numpy(vox).to(cuda_device)),
                rdv.SphereMajorantField(torch.from_numpy(sph).to(cuda_device))):
        node = rdv.PBVR(ext, env, fld, albedo=(0.9, 0.7, 0.5), g=0.4, max_bounces=16)
        est = node(rays, seeds=SEEDS).as_tensor("torch").cpu().numpy().reshape(-1, reps, 3)
        means.append(est.mean(axis=1))
        sems.append(est.std(axis=1) / np.sqrt(reps))
    z = (means[0] - means[1]) / np.maximum(np.sqrt(sems[0] ** 2 + sems[1] ** 2), 1e-4)
    assert np.all(np.abs(z) < 5.0), z
    assert np.abs(z).mean() < 1.5


def test_xr_project_and_environment_map(rdv, cuda_device):
    """XRProject alone (rdvb_xr_project) and XRProject >> TensorSampler as a
    map against the oracle's dir2xr and 2-D sampler."""
    rng = np.random.default_rng(12)
    w = rng.standard_normal((5000, 3)).astype(np.float32)
    w /= np.linalg.norm(w, axis=1, keepdims=True)
    w[:4] = [[0, 1, 0], [0, -1, 0], [-0.0, 0.5, -0.5], [0, 0, -1]]
    w = w.astype(np.float32)
    uv = rdv.XRProject()(torch.from_numpy(w).to(cuda_device)).as_tensor("torch").cpu().numpy()
    np.testing.assert_allclose(uv, orm.dir2xr(w), rtol=0, atol=2e-7)
    img = _env_image(seed=1)
    env = rdv.XRProject() >> rdv.TensorSampler(torch.from_numpy(img).to(cuda_device))
    got = env(torch.from_numpy(w).to(cuda_device)).as_tensor("torch").cpu().numpy()
    np.testing.assert_allclose(got, orm.equirect_environment(img)(w), rtol=1e-4, atol=1e-5)
    c = rdv.Constant([0.1, 0.2, 0.3])(torch.from_numpy(w).to(cuda_device)).as_tensor("torch").cpu().numpy()
    assert c.shape == (5000, 3) and np.all(c == np.array([0.1, 0.2, 0.3], np.float32))


def test_empty_and_jittered_camera_composition(rdv, cuda_device):
    """No rays; Cameras(jitter=True) >> PBVR continues each pixel's
    generator after the camera's two draws, as ratio tracking does."""
    layers = _layers([3, 32, 1], "f32", seed=31)
    vox = _majorant(layers, (2, 2, 2))
    rgb = np.array([0.5, 0.5, 0.5], np.float32)
    node = rdv.PBVR(_chain(rdv, layers, cuda_device), rdv.Constant(rgb), torch.from_numpy(vox).to(cuda_device),
                    albedo=(0.7, 0.8, 0.9), g=0.2)
    out = node(torch.zeros(0, 6, device=cuda_device)).as_tensor("torch")
    assert tuple(out.shape) == (0, 3)
    pose = orm.orbit_pose(1)
    cams = rdv.Cameras(40, 30, torch.from_numpy(pose[None]), jitter=True)
    img = (cams >> node)(seeds=SEEDS).as_tensor("torch").cpu().numpy()
    assert img.shape == (1, 30, 40, 3)
    o, w = orm.camera_rays(pose, 40, 30, jitter_seeds=SEEDS)
    ref = orm.pbvr(o, w, _extinction(layers), orm.constant_environment(rgb),
                   lambda x, ww: orm.voxel_majorant(vox[..., 0], x, ww), SEEDS, albedo=(0.7, 0.8, 0.9), g=0.2,
                   draws_before=2)
    _agree(img.reshape(-1, 3), ref)
    assert rdv.device_status() == 0


# ------------------------------------------------------------ PBVRT, PBVR_NEE
LIGHT = (0.3, 1.0, -0.2)


@pytest.mark.parametrize("variant,math_,field,g,bounces,scale", [
    ("pbvrt", "f32", "voxel", 0.0, 32, 1.0),
    ("pbvrt", "f16", "sphere", 0.6, 4, 0.5),
    ("nee", "f16", "voxel", -0.3, 8, 1.5),
    ("nee", "bf16", "sphere", 0.0, 32, 1.0),
])
def test_pbvrt_and_nee_match_oracle(rdv, cuda_device, variant, math_, field, g, bounces, scale):
    n = 4000
    layers = _layers([3, 32, 1] if math_ != "f16" else [3, 64, 64, 1], math_, seed=bounces * 3 + len(variant))
    vox = _majorant(layers, (4, 3, 5))
    rays = _rays(n, seed=n + bounces)
    if field == "voxel":
        fld = rdv.VoxelMajorantField(torch.from_numpy(vox).to(cuda_device))
        maj = lambda x, w: orm.voxel_majorant(vox[..., 0], x, w)  # noqa: E731
    else:
        sph = _sphere_grid(vox)
        fld = rdv.SphereMajorantField(torch.from_numpy(sph).to(cuda_device))
        maj = lambda x, w: orm.sphere_majorant(sph, x, w)  # noqa: E731
    albedo = (0.9, 0.8, 0.7)
    rgb = np.array([0.3, 0.6, 0.9], np.float32)
    chain = _chain(rdv, layers, cuda_device)
    if variant == "pbvrt":
        node = rdv.PBVRT(chain, fld, rdv.Constant(rgb), rdv.Constant(albedo), light_direction=LIGHT,
                         light_intensity=(2.0, 1.5, 1.0), density_scale=scale, g=g, max_bounces=bounces)
    else:
        node = rdv.PBVR_NEE(chain, fld, rdv.Constant(albedo), light_direction=LIGHT, density_scale=scale, g=g,
                            max_bounces=bounces)
    got = node(torch.from_numpy(rays).to(cuda_device), seeds=SEEDS).as_tensor("torch")
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    ref, evals = orm.pbvrt(rays[:, :3], rays[:, 3:], _extinction(layers), maj, SEEDS, albedo, LIGHT, (2.0, 1.5, 1.0),
                           orm.constant_environment(rgb), density_scale=scale, g=g, max_bounces=bounces,
                           variant=variant, return_evaluations=True)
    assert got.shape == ref.shape == (n, 4 if variant == "pbvrt" else 3)
    # paths here are long (each real collision adds a ratio-tracking shadow
    # ray) and Henyey-Greenstein sampling with g != 0 magnifies last-bit
    # differences of the transcendentals: measured 2.2 % of rays parting
    # with 32 bounces (g = 0), 5.8-6.5 % with the denser 64-wide medium and
    # g = -0.3 (float16 and exact chains alike), the means within a tenth of
    # their standard error, every alpha equal
    _agree(got[:, :3], ref[:, :3], frac=0.9)
    miss = _miss_mask(rays)
    assert np.all(got[miss, :3] == 0)
    if variant == "pbvrt":
        assert np.mean(got[:, 3] == ref[:, 3]) >= 0.99
        assert np.all(got[miss, 3] == 1.0) and (got[:, 3] == 0).any()
    assert (ref[~miss, :3].sum(1) > 0).any()
    assert abs(node.last_evaluations() - evals) <= max(50, 0.03 * evals), (node.last_evaluations(), evals)
    assert rdv.device_status() == 0


def test_pbvrt_alpha_is_an_unbiased_transmittance(rdv, cuda_device):
    """PBVRT's alpha is 1 exactly when the path leaves the box without a real
    collision, so its mean is the transmittance along the ray: the
    fixed-step march's value for the same medium and density scale (both
    fields)."""
    layers = _layers([3, 32, 1], "f32", seed=21, out_bias=0.3)
    ext = _chain(rdv, layers, cuda_device)
    vox = _majorant(layers, (3, 3, 3), margin=2.0)
    sph = _sphere_grid(vox, seed=8)
    base = _rays(64, seed=3)[16:]
    reps = 4096
    rays = torch.from_numpy(np.repeat(base, reps, axis=0)).to(cuda_device)
    rm = rdv.RaymarchingTransmittance(ext, step_size=0.001, density_scale=1.3)
    T = rm(torch.from_numpy(base).to(cuda_device)).as_tensor("torch").cpu().numpy()[:, 0]
    for fld in (rdv.VoxelMajorantField(torch.from_numpy(vox).to(cuda_device)),
                rdv.SphereMajorantField(torch.from_numpy(sph).to(cuda_device))):
        node = rdv.PBVRT(ext, fld, rdv.Constant([0.5, 0.5, 0.5]), rdv.Constant([0.8, 0.8, 0.8]), density_scale=1.3,
                         g=0.2, max_bounces=4)
        alpha = node(rays, seeds=SEEDS).as_tensor("torch").cpu().numpy()[:, 3].reshape(-1, reps)
        mean = alpha.mean(axis=1)
        sem = alpha.std(axis=1) / np.sqrt(reps)
        z = (mean - T) / np.maximum(sem, 1e-4)
        assert np.all(np.abs(z) < 5.0), z
        assert np.abs(z).mean() < 1.5
    assert rdv.device_status() == 0


def test_nee_jittered_camera_composition(rdv, cuda_device):
    layers = _layers([3, 32, 1], "f32", seed=31)
    vox = _majorant(layers, (2, 2, 2))
    node = rdv.PBVR_NEE(_chain(rdv, layers, cuda_device), torch.from_numpy(vox).to(cuda_device),
                        (0.7, 0.8, 0.9), light_direction=LIGHT, g=0.2)
    pose = orm.orbit_pose(1)
    cams = rdv.Cameras(40, 30, torch.from_numpy(pose[None]), jitter=True)
    img = (cams >> node)(seeds=SEEDS).as_tensor("torch").cpu().numpy()
    assert img.shape == (1, 30, 40, 3)
    # the oracle follows the camera's own rays (the jittered camera itself is
    # checked against the oracle in test_gpu_ratiotracking.py), each ray's
    # generator two draws in
    r = cams(seeds=SEEDS).as_tensor("torch").cpu().numpy().reshape(-1, 6)
    ref = orm.pbvrt(r[:, :3], r[:, 3:], _extinction(layers), lambda x, ww: orm.voxel_majorant(vox[..., 0], x, ww),
                    SEEDS, (0.7, 0.8, 0.9), LIGHT, g=0.2, variant="nee", draws_before=2)
    _agree(img.reshape(-1, 3), ref, frac=0.9)
    empty = node(torch.zeros(0, 6, device=cuda_device)).as_tensor("torch")
    assert tuple(empty.shape) == (0, 3)
    assert rdv.device_status() == 0


# ---------------------------------------------------------------- PBVR_ENV
def _env_sampler(rdv, cuda_device, img, levels=5):
    env = rdv.XRProject() >> rdv.TensorSampler(torch.from_numpy(img).to(cuda_device))
    return rdv.XREnvironmentSampler(env, torch.from_numpy(img).to(cuda_device), levels=levels)


def test_xr_quadtree_build_matches_oracle(rdv, cuda_device):
    """XREnvironmentSampler's quadtree: the image resampled at the 2^L cell
    centres by the GridSampler kernel, then the solid-angle-weighted mass
    pyramid as cumulative child probabilities (oracle.raymarch.xr_quadtree,
    float64): equal within float32 rounding, the layout exact."""
    img = _env_image(seed=4, h=24, w=40)
    smp = _env_sampler(rdv, cuda_device, img, levels=5)
    tree = smp.densities.cpu().numpy()
    res = 32
    c = ((np.arange(res, dtype=np.float32) + np.float32(0.5)) / np.float32(res) * np.float32(2) - np.float32(1))
    yy, xx = np.meshgrid(c, c, indexing="ij")
    pts = np.stack([xx, yy], -1).reshape(-1, 2).astype(np.float32)
    dens = oten.grid_sampler(img, pts, clamp=True, aligned=False).reshape(res, res, 3).astype(np.float64).sum(-1)
    ref = orm.xr_quadtree(dens, 5)
    assert tree.shape == ref.shape
    np.testing.assert_allclose(tree, ref, rtol=2e-5, atol=2e-6)
    assert np.all(tree.reshape(-1, 4)[:, 3] == 1.0)


# each collision adds an environment sample (sin, cos, asin and the
# equirectangular lookup) and a shadow ray: measured with an exact chain,
# 0.3 % of rays part with one bounce, 14 % with 32 (the means within one
# standard error)
@pytest.mark.parametrize("field,g,bounces,frac", [("voxel", 0.0, 32, 0.8), ("sphere", 0.5, 4, 0.9),
                                                  ("voxel", 0.3, 1, 0.99)])
def test_pbvr_env_matches_oracle(rdv, cuda_device, field, g, bounces, frac):
    n = 4000
    layers = _layers([3, 32, 1], "f32", seed=61 + bounces)
    vox = _majorant(layers, (4, 3, 5))
    rays = _rays(n, seed=n + bounces)
    if field == "voxel":
        fld = rdv.VoxelMajorantField(torch.from_numpy(vox).to(cuda_device))
        maj = lambda x, w: orm.voxel_majorant(vox[..., 0], x, w)  # noqa: E731
    else:
        sph = _sphere_grid(vox)
        fld = rdv.SphereMajorantField(torch.from_numpy(sph).to(cuda_device))
        maj = lambda x, w: orm.sphere_majorant(sph, x, w)  # noqa: E731
    img = _env_image(seed=9, h=16, w=32)
    smp = _env_sampler(rdv, cuda_device, img, levels=4)
    node = rdv.PBVR_ENV(_chain(rdv, layers, cuda_device), fld, rdv.Constant((0.9, 0.8, 0.7)), smp, g=g,
                        max_bounces=bounces)
    got = node(torch.from_numpy(rays).to(cuda_device), seeds=SEEDS).as_tensor("torch").cpu().numpy()
    ref = orm.pbvrt(rays[:, :3], rays[:, 3:], _extinction(layers), maj, SEEDS, (0.9, 0.8, 0.7), None,
                    environment=orm.equirect_environment(img), g=g, max_bounces=bounces, variant="env",
                    env_densities=smp.densities.cpu().numpy(), env_levels=4)
    assert got.shape == ref.shape == (n, 3)
    _agree(got, ref, frac=frac)
    assert np.all(got[_miss_mask(rays)] == 0) and (ref.sum(1) > 0).any()
    assert rdv.device_status() == 0


def test_pbvr_env_completes_the_transmitted_environment(rdv, cuda_device):
    """For a constant environment L, PBVR (whose escaped paths see L) and
    PBVR_ENV (next-event estimation of the same scattered light, directions
    importance-sampled from a non-uniform quadtree) estimate the same
    radiance up to the light the ray transmits unscattered:
    E[PBVR] = T L + E[PBVR_ENV], T the ray's transmittance."""
    layers = _layers([3, 32, 1], "f32", seed=21, out_bias=0.6)
    ext = _chain(rdv, layers, cuda_device)
    vox = _majorant(layers, (3, 3, 3), margin=1.5)
    base = _rays(48, seed=3)[12:]
    reps = 8192
    rays = torch.from_numpy(np.repeat(base, reps, axis=0)).to(cuda_device)
    L = np.array([0.5, 1.0, 2.0], np.float32)
    img = np.ones((16, 32, 3), np.float32)
    img[2:6, 4:12] = 20.0                                  # a bright patch: a skewed sampling pdf
    smp = rdv.XREnvironmentSampler(rdv.Constant(L), torch.from_numpy(img).to(cuda_device), levels=4)
    fld = torch.from_numpy(vox).to(cuda_device)
    kw = dict(g=0.3, max_bounces=6)
    full = rdv.PBVR(ext, rdv.Constant(L), fld, albedo=(0.8, 0.8, 0.8), **kw)
    nee = rdv.PBVR_ENV(ext, fld, rdv.Constant((0.8, 0.8, 0.8)), smp, **kw)
    a = full(rays, seeds=SEEDS).as_tensor("torch").cpu().numpy().reshape(-1, reps, 3)
    b = nee(rays, seeds=(5, 6, 7, 8)).as_tensor("torch").cpu().numpy().reshape(-1, reps, 3)
    T = rdv.RaymarchingTransmittance(ext, step_size=0.001)(torch.from_numpy(base).to(cuda_device))
    T = T.as_tensor("torch").cpu().numpy()[:, 0]
    lhs = a.mean(axis=1)
    rhs = T[:, None] * L[None] + b.mean(axis=1)
    sem = np.sqrt(a.var(axis=1) / reps + b.var(axis=1) / reps)
    z = (lhs - rhs) / np.maximum(sem, 1e-4)
    assert np.all(np.abs(z) < 5.0), z
    assert np.abs(z).mean() < 1.5
    assert rdv.device_status() == 0
