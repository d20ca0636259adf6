"""GPU parity of RatiotrackingTransmittance (rdv/domain/volumes.py:144-170)
against the CPU oracle (oracle/raymarch.py: ratiotracking_transmittance,
whose generator and tracking loop are pinned to the reference's own
random_library.h and ratiotracking_transmittance_trait.h by
tests/golden/ratiotracking.npz).

Both sides draw the same random numbers (ray i uses the dispatch seeds
spawned by index i), so the estimates agree ray by ray. They may differ
where a last-bit difference flips a decision: the GPU's logf against the
oracle's correctly rounded log, and fused against separately rounded fp32
products in exact (Linear) extinction chains. The tests therefore ask for
agreement on almost every ray and for equal means; the estimator itself is
checked statistically against the fixed-step march of the same medium.
"""
import numpy as np
import pytest
import torch

from oracle import mlp as omlp
from oracle import raymarch as orm

pytestmark = pytest.mark.gpu

SEEDS = (123457, 98765432, 5550123, 777777)


@pytest.fixture(scope="module")
def rdv():
    import rdv_project_b200 as rdv
    return rdv


def _layers(dims, math_, seed, out_bias=0.6):
    rng = np.random.default_rng(seed)
    layers = []
    for i in range(len(dims) - 1):
        W = (rng.standard_normal((dims[i + 1], dims[i])) * np.sqrt(2.0 / dims[i])).astype(np.float32)
        b = (rng.standard_normal(dims[i + 1]) * 0.2).astype(np.float32)
        if i == len(dims) - 2:
            b = b + np.float32(out_bias)
        # a ReLU after every layer, the last included: extinction >= 0
        layers.append({"W": W, "b": b, "math": math_, "relu": True})
    return layers


def _chain(rdv, layers, dev):
    cls = {"f32": rdv.Linear, "f16": rdv.LinearFast, "bf16": rdv.LinearFastBF16}
    m = None
    for l in layers:
        lin = cls[l["math"]](torch.from_numpy(l["W"]).to(dev), torch.from_numpy(l["b"]).to(dev))
        m = lin if m is None else (m >> lin)
        m = m >> rdv.relu
    return m


def _rays(n, seed, spread=3.0):
    rng = np.random.default_rng(seed)
    o = rng.uniform(-spread, spread, size=(n, 3)).astype(np.float32)
    target = rng.uniform(-0.8, 0.8, size=(n, 3)).astype(np.float32)
    w = target - o
    w /= np.linalg.norm(w, axis=1, keepdims=True)
    w = w.astype(np.float32)
    w[: n // 8] *= -1.0                         # pointing away: misses
    o[n // 8: n // 4] *= np.float32(0.2)         # starting inside the box
    return np.concatenate([o, w], axis=1).astype(np.float32)


def _extinction(layers):
    def ext(p):
        return omlp.mlp_forward(np.ascontiguousarray(p, dtype=np.float32), layers)[:, 0]
    return ext


def _majorant(layers, shape, margin=1.3, sub=6):
    """A voxel majorant [D, H, W, 1] of the chain: the largest value on a
    sub x sub x sub lattice of every cell (its faces included), times margin."""
    D, H, W = shape
    zs = np.linspace(-1, 1, D * (sub - 1) + 1, dtype=np.float32)
    ys = np.linspace(-1, 1, H * (sub - 1) + 1, dtype=np.float32)
    xs = np.linspace(-1, 1, W * (sub - 1) + 1, dtype=np.float32)
    Z, Y, X = np.meshgrid(zs, ys, xs, indexing="ij")
    v = omlp.mlp_forward_f64(np.stack([X, Y, Z], -1).reshape(-1, 3).astype(np.float32), layers)[:, 0]
    v = v.reshape(Z.shape)
    g = np.zeros((D, H, W), dtype=np.float32)
    for k in range(D):
        for j in range(H):
            for i in range(W):
                cell = v[k * (sub - 1):(k + 1) * (sub - 1) + 1, j * (sub - 1):(j + 1) * (sub - 1) + 1,
                         i * (sub - 1):(i + 1) * (sub - 1) + 1]
                g[k, j, i] = max(float(cell.max()), 0.0) * margin + 0.05
    return g[..., None]


def _agree(got, ref, frac=0.995, tol=1e-5):
    d = np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64))
    close = float(np.mean(d <= tol))
    assert close >= frac, (close, np.nonzero(d > tol)[0][:8])
    assert abs(float(np.mean(got)) - float(np.mean(ref))) <= 2e-3
    return close


@pytest.mark.parametrize("math_,dims,n,scale", [
    ("f32", [3, 32, 1], 6000, 1.0),
    ("f16", [3, 64, 64, 1], 6000, 2.0),
    ("bf16", [3, 48, 1], 4000, 0.5),
])
def test_ratiotracking_matches_oracle(rdv, cuda_device, math_, dims, n, scale):
    layers = _layers(dims, math_, seed=len(dims) * 10 + n)
    grid = _majorant(layers, (4, 3, 5))
    rays = _rays(n, seed=n)
    node = rdv.RatiotrackingTransmittance(_chain(rdv, layers, cuda_device),
                                          torch.from_numpy(grid).to(cuda_device), density_scale=scale)
    got = node(torch.from_numpy(rays).to(cuda_device), seeds=SEEDS).as_tensor("torch")
    torch.cuda.synchronize()
    assert tuple(got.shape) == (n, 1)
    got = got.cpu().numpy()[:, 0]
    ref, evals = orm.ratiotracking_transmittance(rays[:, :3], rays[:, 3:], scale, _extinction(layers), grid,
                                                 SEEDS, return_evaluations=True)
    _agree(got, ref)
    assert np.all(got[: n // 8][ref[: n // 8] == 1.0] == 1.0)   # misses
    assert (ref == 0).any() and ((ref > 0) & (ref < 1)).any()   # roulette kills and partial transmittance
    gpu_evals = node.last_evaluations()
    assert abs(gpu_evals - evals) <= max(10, 0.01 * evals), (gpu_evals, evals)
    assert rdv.device_status() == 0


def test_transform_single_cell_majorant_and_tensor_grid(rdv, cuda_device):
    """A scaled, rotated, shifted box; a one-cell (global) majorant given as
    a TensorGrid; the same seeds give the same estimate twice."""
    layers = _layers([3, 32, 1], "f32", seed=5)
    grid = _majorant(layers, (1, 1, 1))
    c, s = np.cos(0.4), np.sin(0.4)
    M = np.array([[1.5 * c, 0, -1.5 * s], [0, 0.8, 0], [1.5 * s, 0, 1.5 * c]], dtype=np.float32)  # columns
    transform = np.concatenate([M.reshape(-1), np.array([0.3, -0.2, 0.1], np.float32)])
    rays = _rays(4000, seed=11, spread=4.0)
    tg = rdv.TensorGrid(torch.from_numpy(grid).to(cuda_device))
    node = rdv.RatiotrackingTransmittance(_chain(rdv, layers, cuda_device), tg, transform=transform,
                                          density_scale=1.5)
    r = torch.from_numpy(rays).to(cuda_device)
    a = node(r, seeds=SEEDS).as_tensor("torch").cpu().numpy()[:, 0]
    b = node(r, seeds=SEEDS).as_tensor("torch").cpu().numpy()[:, 0]
    assert np.array_equal(a, b)
    ref = orm.ratiotracking_transmittance(rays[:, :3], rays[:, 3:], 1.5, _extinction(layers), grid, SEEDS,
                                          transform=transform)
    _agree(a, ref)
    c2 = node(r).as_tensor("torch").cpu().numpy()[:, 0]   # fresh seeds: another estimate
    assert node.last_seeds != SEEDS and not np.array_equal(a, c2)


def test_estimator_is_unbiased_against_the_fixed_step_march(rdv, cuda_device):
    """Averaged over many independent estimates (the same ray repeated, each
    copy with its own generator), ratio tracking converges to the
    transmittance exp(-integral of density_scale * extinction), which the
    fixed-step RaymarchingTransmittance approximates with a small step."""
    layers = _layers([3, 32, 1], "f32", seed=21, out_bias=0.3)
    ext = _chain(rdv, layers, cuda_device)
    grid = _majorant(layers, (2, 2, 2), margin=2.0)
    base = _rays(64, seed=3)
    base = base[64 // 4:]                       # rays that reach the box from outside
    reps = 4096
    rays = np.repeat(base, reps, axis=0)
    rt = rdv.RatiotrackingTransmittance(ext, torch.from_numpy(grid).to(cuda_device), density_scale=0.8)
    est = rt(torch.from_numpy(rays).to(cuda_device), seeds=SEEDS).as_tensor("torch").cpu().numpy()[:, 0]
    mean = est.reshape(-1, reps).mean(axis=1)
    sem = est.reshape(-1, reps).std(axis=1) / np.sqrt(reps)
    rm = rdv.RaymarchingTransmittance(ext, step_size=0.001, density_scale=0.8)
    T = rm(torch.from_numpy(base).to(cuda_device)).as_tensor("torch").cpu().numpy()[:, 0]
    z = (mean - T) / np.maximum(sem, 1e-4)
    assert np.all(np.abs(z) < 5.0), z
    assert np.abs(z).mean() < 1.5


def test_empty_and_camera_composition(rdv, cuda_device):
    layers = _layers([3, 16, 1], "f16", seed=2)
    grid = torch.from_numpy(_majorant(layers, (2, 2, 2))).to(cuda_device)
    node = rdv.RatiotrackingTransmittance(_chain(rdv, layers, cuda_device), rdv.VoxelMajorantField(grid))
    out = node(torch.zeros(0, 6, device=cuda_device)).as_tensor("torch")
    assert tuple(out.shape) == (0, 1)
    pose = torch.tensor([[3.0, 0.5, 0.0, 0.0, 0.0, 0.0, 0.0, 1.0, 0.0]], device=cuda_device)
    cam = rdv.Cameras(48, 32, pose)
    t = (cam >> node)().as_tensor("torch")   # fresh seeds per call, as the reference
    assert tuple(t.shape) == (1, 32, 48, 1)
    v = t.cpu().numpy()
    assert np.all(np.isfinite(v)) and (v < 1).any() and (v == 1).any()
    assert rdv.device_status() == 0



def test_jittered_cameras_vs_oracle(rdv, cuda_device):
    """Cameras(jitter=True) (cameras.h:7): each pixel's ray passes through
    (column + r0, row + r1), the first two draws of the pixel's generator
    (seeds spawned by the flat pixel index over all cameras)."""
    poses = np.stack([orm.orbit_pose(0), orm.orbit_pose(3)]).astype(np.float32)
    cams = rdv.Cameras(24, 16, torch.from_numpy(poses), jitter=True)
    rays = cams(seeds=SEEDS).as_tensor("torch").cpu().numpy()
    assert rays.shape == (2, 16, 24, 6)
    centre = rdv.Cameras(24, 16, torch.from_numpy(poses))().as_tensor("torch").cpu().numpy()
    for c in range(2):
        o, w = orm.camera_rays(poses[c], 24, 16, jitter_seeds=SEEDS, camera_index=c)
        np.testing.assert_allclose(rays[c].reshape(-1, 6)[:, :3], o, rtol=0, atol=1e-6)
        np.testing.assert_allclose(rays[c].reshape(-1, 6)[:, 3:], w, rtol=0, atol=1e-5)
    assert np.abs(rays[..., 3:] - centre[..., 3:]).max() > 1e-3          # off-centre
    again = cams(seeds=SEEDS).as_tensor("torch").cpu().numpy()
    assert np.array_equal(rays, again)
    fresh = cams().as_tensor("torch").cpu().numpy()                       # new seeds per call
    assert cams.last_seeds != SEEDS and not np.array_equal(rays, fresh)


def test_jittered_cameras_composed_with_ratio_tracking(rdv, cuda_device):
    """Cameras(jitter=True) >> RatiotrackingTransmittance: as in the
    reference's single per-thread generator, ratio tracking continues each
    pixel's sequence after the camera's two draws (draws_before = 2)."""
    layers = _layers([3, 32, 1], "f32", seed=31)
    grid = _majorant(layers, (2, 2, 2))
    pose = orm.orbit_pose(1)
    cams = rdv.Cameras(40, 30, torch.from_numpy(pose[None]), jitter=True)
    node = rdv.RatiotrackingTransmittance(_chain(rdv, layers, cuda_device), torch.from_numpy(grid).to(cuda_device),
                                          density_scale=1.2)
    img = (cams >> node)(seeds=SEEDS).as_tensor("torch").cpu().numpy()
    assert img.shape == (1, 30, 40, 1)
    o, w = orm.camera_rays(pose, 40, 30, jitter_seeds=SEEDS)
    ref = orm.ratiotracking_transmittance(o, w, 1.2, _extinction(layers), grid, SEEDS, draws_before=2)
    got = img.reshape(-1)
    _agree(got, ref)
    # without the skip the estimates would be those of other random numbers
    other = orm.ratiotracking_transmittance(o, w, 1.2, _extinction(layers), grid, SEEDS, draws_before=0)
    assert np.mean(np.abs(got - other) > 1e-3) > 0.05
    assert rdv.device_status() == 0
