"""GPU parity of the camera rays and the MLP volume ray-march (BASELINE
config 4) against the CPU oracle (oracle/raymarch.py).

Tolerances: camera rays are fp32 arithmetic (1e-5); the render runs the MLP
with float16 operands and fp32 accumulation, so BASELINE's 1e-2 applies,
normwise and elementwise (|d| / (|ref| + rms(ref))). Pixels whose ray misses
the box are 0 (up to rays grazing an edge, which the GPU's and the oracle's
fp32 directions may classify differently).
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


def _mlp_layers(seed=0, dims=(3, 64, 64, 4), math_="f16", bias_scale=0.2):
    rng = np.random.default_rng(seed)
    layers = []
    for i in range(len(dims) - 1):
        W = (rng.standard_normal((dims[i + 1], dims[i])) * np.sqrt(2.0 / dims[i])).astype(np.float32)
        b = (rng.standard_normal(dims[i + 1]) * bias_scale).astype(np.float32)
        layers.append({"W": W, "b": b, "math": math_, "relu": i < len(dims) - 2})
    return layers


def _build(rdv, layers, dev):
    m = None
    for l in layers:
        cls = rdv.LinearFast if l["math"] == "f16" else rdv.LinearFastBF16
        lin = cls(torch.from_numpy(l["W"]).to(dev), torch.from_numpy(l["b"]).to(dev))
        m = lin if m is None else (m >> lin)
        if l["relu"]:
            m = m >> rdv.relu
    return m


def _check(y, ref, tol):
    nw, el = omlp.rel_errors(np.asarray(y, dtype=np.float64), np.asarray(ref, dtype=np.float64))
    assert nw <= tol and el <= tol, (nw, el)
    return nw, el


def test_camera_rays_vs_oracle(rdv, cuda_device):
    poses = np.stack([orm.orbit_pose(0), orm.orbit_pose(3)]).astype(np.float32)
    cams = rdv.Cameras(24, 16, torch.from_numpy(poses))
    rays = cams().as_tensor("torch").cpu().numpy()
    assert rays.shape == (2, 16, 24, 6)
    for c in range(2):
        o, w = orm.camera_rays(poses[c], 24, 16)
        np.testing.assert_allclose(rays[c].reshape(-1, 6)[:, :3], o, rtol=0, atol=1e-6)
        np.testing.assert_allclose(rays[c].reshape(-1, 6)[:, 3:], w, rtol=0, atol=TOL_F32)


@pytest.mark.parametrize("frame", [0, 1, 5])
def test_render_vs_oracle(rdv, cuda_device, frame):
    layers = _mlp_layers(seed=frame)
    ren = rdv.VolumeRenderer(_build(rdv, layers, cuda_device))
    pose = orm.orbit_pose(frame)
    img = ren.render(torch.from_numpy(pose), 64, 48).cpu().numpy()
    ref = orm.render_emission_absorption(pose, 64, 48, 128, layers)
    o, w = orm.camera_rays(pose, 64, 48)
    tmin, tmax = orm.ray_box(o, w)
    miss = ((tmax <= 0) | (tmin > tmax)).reshape(48, 64)
    assert miss.any() and (~miss).any()
    # (a ray grazing the box edge may land on either side of the slab test)
    assert np.abs(img[miss]).max() <= 1e-3
    assert np.all(img[~miss][:, 3] >= 0.0) and (img[~miss][:, 3] > 0.0).mean() > 0.99
    _check(img, ref, TOL_F16)
    assert rdv.device_status() == 0


def test_render_bf16_and_bands(rdv, cuda_device):
    layers = _mlp_layers(seed=7, math_="bf16")
    ren = rdv.VolumeRenderer(_build(rdv, layers, cuda_device))
    pose = orm.orbit_pose(2)
    full = ren.render(torch.from_numpy(pose), 40, 30).cpu().numpy()
    _check(full, orm.render_emission_absorption(pose, 40, 30, 128, layers), TOL_F16)
    # a band of rows is exactly those rows of the full image (rays are independent)
    band = ren.render(torch.from_numpy(pose), 40, 30, row_begin=9, row_end=21).cpu().numpy()
    np.testing.assert_array_equal(band, full[9:21])


def test_render_config4_full_width_band(rdv, cuda_device):
    # BASELINE config 4 geometry: 1920x1080, fov pi/4, 128 samples, MLP
    # 3-64-64-4 float16, Kaiming-normal weights (seeded), zero biases; the
    # oracle checks a band of 6 full-width rows through the cube's middle
    g = torch.Generator().manual_seed(1000)
    dims = [3, 64, 64, 4]
    layers = []
    for i in range(3):
        W = (torch.randn((dims[i + 1], dims[i]), generator=g) * math.sqrt(2.0 / dims[i])).numpy()
        layers.append({"W": W.astype(np.float32), "b": np.zeros(dims[i + 1], np.float32), "math": "f16",
                       "relu": i < 2})
    ren = rdv.VolumeRenderer(_build(rdv, layers, cuda_device))
    pose = orm.orbit_pose(0)
    img = ren.render(torch.from_numpy(pose), 1920, 1080)
    assert img.shape == (1080, 1920, 4)
    band = img[537:543].cpu().numpy()
    ref = orm.render_emission_absorption(pose, 1920, 1080, 128, layers, row_begin=537, row_end=543)
    _check(band, ref, TOL_F16)
    assert rdv.device_status() == 0


def test_render_errors(rdv, cuda_device):
    import rdv_project_b200._native as N
    layers = _mlp_layers()
    m = _build(rdv, layers, cuda_device)
    with pytest.raises(AssertionError, match="n_samples must be 128"):
        rdv.VolumeRenderer(m, n_samples=64)
    bad = _build(rdv, _mlp_layers(dims=(3, 32, 5)), cuda_device)
    with pytest.raises(AssertionError, match=r"\(density, r, g, b\)"):
        rdv.VolumeRenderer(bad)
    lib = N.lib()
    dummy = torch.zeros(1 << 16, device=cuda_device)
    rc = lib.rdvb_raymarch_render(N.float_array(orm.orbit_pose(0)), 8, 8, 0.0, 0.0, 64, 3, N.int_array([3, 64, 64, 4]),
                                  N.int_array([1 | 4, 1 | 4, 1]), dummy.data_ptr(), 0, 8, dummy.data_ptr(),
                                  dummy.numel() * 4, dummy.data_ptr(), None)
    assert rc == -2 and "n_samples" in N.last_error()
    rc = lib.rdvb_raymarch_render(N.float_array(orm.orbit_pose(0)), 8, 8, 0.0, 0.0, 128, 3,
                                  N.int_array([3, 64, 64, 4]), N.int_array([1 | 4, 1 | 4, 1]), dummy.data_ptr(), 0, 9,
                                  dummy.data_ptr(), dummy.numel() * 4, dummy.data_ptr(), None)
    assert rc == -1 and "rows" in N.last_error()
