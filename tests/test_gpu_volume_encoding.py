"""Volume nodes whose extinction starts with a sampler of a dense 3-D grid
(GridSampler / TensorSampler >> Linear ..., or the sampler alone: a density
volume), the reference's usual form of a Map[3, 1] extinction besides a pure
MLP (rdv/domain/volumes.py:7-19 accepts any). The sampler runs inside the
march / tracking kernels as the chain's input encoding (rdvb_encoding);
parity against the oracle's sampler (pinned bit-exact to the reference's
grid_sampler.h) composed with its chain."""
import numpy as np
import pytest
import torch

from oracle import mlp as omlp
from oracle import raymarch as orm
from oracle import tensors as oten
from test_gpu_ratiotracking import SEEDS, _agree, _rays

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rdv():
    import rdv_project_b200 as rdv
    return rdv


def _density(seed, shape=(12, 10, 14), feats=1, scale=2.0):
    rng = np.random.default_rng(seed)
    return (np.abs(rng.standard_normal(shape + (feats,))) * scale).astype(np.float32)


def _layers(dims, math_, seed):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(len(dims) - 1):
        W = (rng.standard_normal((dims[i + 1], dims[i])) * np.sqrt(2.0 / dims[i])).astype(np.float32)
        b = (rng.standard_normal(dims[i + 1]) * 0.2 + (0.5 if i == len(dims) - 2 else 0.0)).astype(np.float32)
        out.append({"W": W, "b": b, "math": math_, "relu": True})
    return out


def _map(rdv, smp, layers, dev):
    m = smp
    cls = {"f32": rdv.Linear, "f16": rdv.LinearFast, "bf16": rdv.LinearFastBF16}
    for l in layers:
        m = m >> cls[l["math"]](torch.from_numpy(l["W"]).to(dev), torch.from_numpy(l["b"]).to(dev)) >> rdv.relu
    return m


def _ext(sample, layers):
    def ext(p):
        f = sample(np.ascontiguousarray(p, dtype=np.float32))
        if not layers:
            return f[:, 0].astype(np.float32)
        return omlp.mlp_forward(f, layers)[:, 0].astype(np.float32)
    return ext


@pytest.mark.parametrize("kind,clamp,aligned", [("grid", True, False), ("tensor", False, True)])
def test_density_volume_raymarch(rdv, cuda_device, kind, clamp, aligned):
    """A bare sampler as the extinction: the fixed-step march of a density
    grid."""
    dens = _density(3)
    rays = _rays(3000, seed=8)
    t = torch.from_numpy(dens).to(cuda_device)
    smp = rdv.GridSampler(t, clamp=clamp, aligned=aligned) if kind == "grid" else \
        rdv.TensorSampler(t, clamp=clamp, aligned=aligned)
    node = rdv.RaymarchingTransmittance(smp, step_size=0.01, density_scale=0.7)
    got = node(torch.from_numpy(rays).to(cuda_device)).as_tensor("torch").cpu().numpy()[:, 0]
    sample = (lambda p: oten.grid_sampler(dens, p, clamp, aligned)) if kind == "grid" else \
        (lambda p: oten.tensor_sampler(dens, p, clamp, aligned))
    ref = orm.raymarching_transmittance(rays[:, :3], rays[:, 3:], 0.01, 0.7, _ext(sample, []))
    np.testing.assert_allclose(got, ref, rtol=0, atol=1e-5)
    assert (ref < 0.5).any() and (ref == 1).any()
    assert rdv.device_status() == 0


@pytest.mark.parametrize("math_", ["f32", "f16"])
def test_feature_grid_mlp_raymarch(rdv, cuda_device, math_):
    """GridSampler (8 features) >> MLP: float16 chains with an encoding run on
    the CUDA cores (the tensor-core march takes positions only)."""
    feats = _density(5, (6, 7, 8), feats=8, scale=1.0)
    layers = _layers([8, 16, 1], math_, seed=11)
    rays = _rays(2000, seed=9)
    smp = rdv.GridSampler(torch.from_numpy(feats).to(cuda_device), aligned=True)
    node = rdv.RaymarchingTransmittance(_map(rdv, smp, layers, cuda_device), step_size=0.02, density_scale=1.2)
    got = node(torch.from_numpy(rays).to(cuda_device)).as_tensor("torch").cpu().numpy()[:, 0]
    ref = orm.raymarching_transmittance(rays[:, :3], rays[:, 3:], 0.02, 1.2,
                                        _ext(lambda p: oten.grid_sampler(feats, p, aligned=True), layers))
    np.testing.assert_allclose(got, ref, rtol=0, atol=1e-5 if math_ == "f32" else 2e-3)
    assert rdv.device_status() == 0


def test_density_volume_ratio_tracking_and_pbvr(rdv, cuda_device):
    """Ratio tracking and PBVR through a density grid (GridSampler alone),
    ray by ray against the oracle with the same seeds."""
    dens = _density(7, (8, 8, 8), scale=1.5)
    maj = np.full((2, 2, 2, 1), float(dens.max()) * 1.05 + 0.01, np.float32)
    rays = _rays(4000, seed=12)
    t = torch.from_numpy(dens).to(cuda_device)
    ext = _ext(lambda p: oten.grid_sampler(dens, p), [])
    rt = rdv.RatiotrackingTransmittance(rdv.GridSampler(t), torch.from_numpy(maj).to(cuda_device))
    got = rt(torch.from_numpy(rays).to(cuda_device), seeds=SEEDS).as_tensor("torch").cpu().numpy()[:, 0]
    ref = orm.ratiotracking_transmittance(rays[:, :3], rays[:, 3:], 1.0, ext, maj, SEEDS)
    _agree(got, ref)
    rgb = np.array([0.2, 0.4, 0.8], np.float32)
    pb = rdv.PBVR(rdv.GridSampler(t), rdv.Constant(rgb), torch.from_numpy(maj).to(cuda_device), albedo=(0.8, 0.8, 0.8),
                  g=0.3, max_bounces=8)
    got = pb(torch.from_numpy(rays).to(cuda_device), seeds=SEEDS).as_tensor("torch").cpu().numpy()
    ref = orm.pbvr(rays[:, :3], rays[:, 3:], ext, orm.constant_environment(rgb),
                   lambda x, w: orm.voxel_majorant(maj[..., 0], x, w), SEEDS, albedo=(0.8, 0.8, 0.8), g=0.3,
                   max_bounces=8)
    close = np.mean(np.all(np.abs(got - ref) <= 2e-5 + 1e-4 * np.abs(ref), axis=1))
    assert close >= 0.98, close
    assert rdv.device_status() == 0
