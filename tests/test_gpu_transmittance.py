"""GPU parity of RaymarchingTransmittance (rdv/domain/volumes.py:124-141)
against the CPU oracle (oracle/raymarch.py: raymarching_transmittance, whose
march loop is pinned to the reference's own transmittance_rm by
tests/golden/transmittance.npz).

The march (object-space transform, slab test, step count, positions, the
tau > 16 exit) is fp32 arithmetic done in the same order on both sides; the
extinction MLP differs only by fp32 rounding (exact Linear layers) or runs
with float16 operands (LinearFast). Tolerances are BASELINE's: 1e-5 for fp32
chains, 1e-2 for float16 chains, normwise and elementwise
(|d| / (|ref| + rms(ref))).
"""
import math

import numpy as np
import pytest
import torch

from oracle import mlp as omlp
from oracle import raymarch as orm

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5
TOL_F16 = 1e-2


@pytest.fixture(scope="module")
def rdv():
    import rdv_project_b200 as rdv
    return rdv


def _layers(dims, math_, seed, out_bias=0.5, final_relu=False):
    rng = np.random.default_rng(seed)
    layers = []
    for i in range(len(dims) - 1):
        W = (rng.standard_normal((dims[i + 1], dims[i])) * np.sqrt(2.0 / dims[i])).astype(np.float32)
        b = (rng.standard_normal(dims[i + 1]) * 0.2).astype(np.float32)
        if i == len(dims) - 2:
            b = b + np.float32(out_bias)  # mostly positive extinction
        layers.append({"W": W, "b": b, "math": math_, "relu": i < len(dims) - 2 or final_relu})
    return layers


def _chain(rdv, layers, dev):
    cls = {"f32": rdv.Linear, "f16": rdv.LinearFast, "bf16": rdv.LinearFastBF16}
    m = None
    for l in layers:
        lin = cls[l["math"]](torch.from_numpy(l["W"]).to(dev), torch.from_numpy(l["b"]).to(dev))
        m = lin if m is None else (m >> lin)
        if l["relu"]:
            m = m >> rdv.relu
    return m


def _rays(n, seed, spread=3.0):
    rng = np.random.default_rng(seed)
    o = rng.uniform(-spread, spread, size=(n, 3)).astype(np.float32)
    target = rng.uniform(-0.8, 0.8, size=(n, 3)).astype(np.float32)
    w = target - o
    w /= np.linalg.norm(w, axis=1, keepdims=True)
    w = w.astype(np.float32)
    # a quarter of the rays point away from the box, some start inside it
    w[: n // 4] *= -1.0
    o[n // 4: n // 4 + n // 8] *= np.float32(0.2)
    return np.concatenate([o, w], axis=1).astype(np.float32)


def _check(y, ref, tol):
    nw, el = omlp.rel_errors(np.asarray(y, dtype=np.float64), np.asarray(ref, dtype=np.float64))
    assert nw <= tol and el <= tol, (nw, el)
    return nw, el


def _run(rdv, layers, rays, dev, **kw):
    node = rdv.RaymarchingTransmittance(_chain(rdv, layers, dev), **kw)
    out = node(torch.from_numpy(rays).to(dev)).as_tensor("torch")
    torch.cuda.synchronize()
    assert tuple(out.shape) == (rays.shape[0], 1)
    return out[:, 0].cpu().numpy()


def _oracle(layers, rays, step_size=0.002, density_scale=1.0, transform=None):
    return orm.raymarching_transmittance(rays[:, :3], rays[:, 3:], step_size, density_scale,
                                         orm.mlp_extinction(layers), transform)


@pytest.mark.parametrize("dims,step,scale,final_relu", [((3, 32, 1), 0.02, 1.0, False),
                                                        ((3, 64, 64, 1), 0.01, 2.0, True),
                                                        ((3, 16, 16, 16, 1), 0.05, 4.0, False),
                                                        ((3, 128, 1), 0.01, 1.0, True)])
def test_fp32_chain_matches_oracle(rdv, cuda_device, dims, step, scale, final_relu):
    # final_relu: extinction = ReLU(MLP) >= 0, the usual density; without it
    # the field also takes negative values (tau may fall), as any Map may
    layers = _layers(dims, "f32", seed=len(dims), final_relu=final_relu)
    rays = _rays(1536, seed=1)
    node = rdv.RaymarchingTransmittance(_chain(rdv, layers, cuda_device), step_size=step, density_scale=scale)
    got = node(torch.from_numpy(rays).to(cuda_device)).as_tensor("torch")[:, 0].cpu().numpy()
    ref, evals = orm.raymarching_transmittance(rays[:, :3], rays[:, 3:], step, scale, orm.mlp_extinction(layers),
                                               return_evaluations=True)
    _check(got, ref, TOL_F32)
    # same number of march steps (positions, d and the exits follow the same fp32 operations)
    # (a ray whose tau ends within rounding of 16 may exit on one side only)
    flips = np.any((got == 0.0) != (ref == 0.0))
    assert node.last_evaluations() == evals or flips, (node.last_evaluations(), evals)
    # the march outcomes themselves agree: misses give exactly 1, early exits exactly 0
    assert np.array_equal(got == 1.0, ref == 1.0)
    assert np.sum((got == 0.0) != (ref == 0.0)) <= 2  # a tau within rounding of 16 may exit on one side only


@pytest.mark.parametrize("math_", ["f16", "bf16"])
def test_staged_chain_matches_oracle(rdv, cuda_device, math_):
    layers = _layers((3, 64, 64, 1), math_, seed=7, final_relu=True)
    rays = _rays(2048, seed=2)
    got = _run(rdv, layers, rays, cuda_device, step_size=0.01, density_scale=1.5)
    ref = _oracle(layers, rays, 0.01, 1.5)
    _check(got, ref, TOL_F16)


def test_tensor_core_march_step_count_and_batches(rdv, cuda_device):
    """float16 chains run the chunked tensor-core march: every step of a ray
    is evaluated (Σ of the reference loop's step counts, no early exit), and
    more rays than one batch (262,144) are processed in order."""
    layers = _layers((3, 16, 1), "f16", seed=11, final_relu=True)
    rays = _rays(300_000, seed=12)
    node = rdv.RaymarchingTransmittance(_chain(rdv, layers, cuda_device), step_size=0.05, density_scale=1.0)
    got = node(torch.from_numpy(rays).to(cuda_device)).as_tensor("torch")[:, 0].cpu().numpy()
    ref = _oracle(layers, rays, 0.05, 1.0)
    _check(got, ref, TOL_F16)
    _, steps = orm.raymarching_transmittance(rays[:, :3], rays[:, 3:], 0.05, 0.0, orm.mlp_extinction(layers),
                                             return_evaluations=True)
    assert node.last_evaluations() == steps


def test_mixed_precision_chain_runs_on_cuda_cores(rdv, cuda_device):
    """A chain mixing exact and float16 layers takes the CUDA-core march with
    float16 staging of the LinearFast layer's operands."""
    layers = _layers((3, 32, 1), "f32", seed=13, final_relu=True)
    layers[1]["math"] = "f16"
    rays = _rays(1024, seed=14)
    got = _run(rdv, layers, rays, cuda_device, step_size=0.02, density_scale=2.0)
    ref = _oracle(layers, rays, 0.02, 2.0)
    _check(got, ref, TOL_F16)


def test_transform_matches_oracle(rdv, cuda_device):
    layers = _layers((3, 32, 1), "f32", seed=3)
    rays = _rays(1024, seed=4, spread=5.0)
    c, s = math.cos(0.6), math.sin(0.6)
    R = np.array([[c, -s, 0.0], [s, c, 0.0], [0.0, 0.0, 1.0]]) * np.array([1.5, 0.8, 1.2])
    T = np.array([0.3, -0.2, 0.5])
    mat4x3 = np.concatenate([R.T.reshape(-1), T])  # columns of the 3x3 part, then the origin
    got = _run(rdv, layers, rays, cuda_device, step_size=0.02, density_scale=1.0, transform=mat4x3)
    ref = _oracle(layers, rays, 0.02, 1.0, mat4x3)
    _check(got, ref, TOL_F32)
    # the same node with the transform given as four vec3 columns
    got2 = _run(rdv, layers, rays, cuda_device, step_size=0.02, transform=mat4x3.reshape(4, 3))
    assert np.array_equal(got, got2)


def test_misses_exits_and_safety_cap(rdv, cuda_device):
    layers = _layers((3, 16, 1), "f32", seed=5, out_bias=3.0)
    rays = _rays(512, seed=6)
    # huge density: every hitting ray with a long enough segment exits with exactly 0
    got = _run(rdv, layers, rays, cuda_device, step_size=0.05, density_scale=200.0)
    ref = _oracle(layers, rays, 0.05, 200.0)
    _check(got, ref, TOL_F32)
    assert np.any(ref == 0.0) and np.array_equal(got == 0.0, ref == 0.0)
    assert np.array_equal(got == 1.0, ref == 1.0) and np.any(ref == 1.0)
    # tiny steps: long segments stop after 4096 steps (the reference's safety cap)
    step = 2e-4
    got = _run(rdv, layers, rays, cuda_device, step_size=step, density_scale=0.05)
    ref = _oracle(layers, rays, step, 0.05)
    _check(got, ref, TOL_F32)
    o, w = rays[:, :3], rays[:, 3:]
    tmin, tmax = orm.ray_box(o, w)
    assert np.any(tmax - np.maximum(tmin, 0) > 4096 * step)  # the cap is reached by some rays


def test_empty_and_generic_extinction(rdv, cuda_device):
    layers = _layers((3, 8, 1), "f32", seed=8)
    node = rdv.RaymarchingTransmittance(_chain(rdv, layers, cuda_device))
    out = node(torch.zeros(0, 6, device=cuda_device)).as_tensor("torch")
    assert tuple(out.shape) == (0, 1)
    with pytest.raises(AssertionError):
        rdv.RaymarchingTransmittance(rdv.Linear(torch.zeros(2, 3), torch.zeros(2)))  # not a Map[3, 1]
    # leading batch dimensions are kept
    rays = _rays(96, seed=9).reshape(4, 24, 6)
    out = node(torch.from_numpy(rays).to(cuda_device)).as_tensor("torch")
    assert tuple(out.shape) == (4, 24, 1)


def test_cameras_compose_with_transmittance(rdv, cuda_device):
    layers = _layers((3, 32, 32, 1), "f16", seed=10)
    pose = orm.orbit_pose(1)
    cams = rdv.Cameras(48, 32, torch.from_numpy(pose[None]))
    node = rdv.RaymarchingTransmittance(_chain(rdv, layers, cuda_device), step_size=0.01, density_scale=2.0)
    img = (cams >> node)().as_tensor("torch")
    torch.cuda.synchronize()
    assert tuple(img.shape) == (1, 32, 48, 1)
    o, w = orm.camera_rays(pose, 48, 32)
    ref = orm.raymarching_transmittance(o, w, 0.01, 2.0, orm.mlp_extinction(layers))
    _check(img.reshape(-1).cpu().numpy(), ref, TOL_F16)
    assert rdv.device_status() == 0
