"""GPU parity of TensorSampler (rdv/maths/__init__.py:2050-2083) against the
oracle restatement (oracle/tensors.tensor_sampler, itself checked against
torch's grid_sample on CPU), alone and as the input encoding of a fused MLP
chain (sampler >> LinearFast ...). The sampler is fp32 arithmetic in the
reference's order: 1e-5; the chain runs float16 operands: 1e-2."""
import numpy as np
import pytest
import torch

from oracle import mlp as omlp
from oracle import tensors as oten

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rdv():
    import rdv_project_b200 as rdv
    return rdv


@pytest.mark.parametrize("shape", [(37, 5), (9, 13, 8), (6, 7, 5, 16), (32, 32, 32, 4)])
@pytest.mark.parametrize("clamp,aligned,linear", [(True, False, True), (False, True, True), (True, True, False),
                                                  (False, False, False)])
def test_sampler_matches_oracle(rdv, cuda_device, shape, clamp, aligned, linear):
    rng = np.random.default_rng(len(shape) * 7 + clamp + 2 * aligned + 4 * linear)
    t = rng.standard_normal(shape).astype(np.float32)
    in_dim = len(shape) - 1
    x = rng.uniform(-1.25, 1.25, size=(4000, in_dim)).astype(np.float32)
    s = rdv.TensorSampler(torch.from_numpy(t).to(cuda_device), clamp=clamp, aligned=aligned, linear=linear)
    got = s(torch.from_numpy(x).to(cuda_device)).as_tensor("torch").cpu().numpy()
    ref = oten.tensor_sampler(t, x, clamp, aligned, linear)
    nw, el = omlp.rel_errors(got, ref)
    assert nw <= 1e-5 and el <= 1e-5, (nw, el)


def test_sampler_feeds_fused_mlp(rdv, cuda_device):
    rng = np.random.default_rng(3)
    grid = rng.standard_normal((16, 16, 16, 16)).astype(np.float32)
    dims = [16, 64, 64, 4]
    layers = [{"W": (rng.standard_normal((dims[i + 1], dims[i])) * np.sqrt(2.0 / dims[i])).astype(np.float32),
               "b": (rng.standard_normal(dims[i + 1]) * 0.1).astype(np.float32), "math": "f16", "relu": i < 2}
              for i in range(3)]
    m = rdv.TensorSampler(torch.from_numpy(grid).to(cuda_device))
    for l in layers:
        m = m >> rdv.linear(torch.from_numpy(l["W"]).to(cuda_device), torch.from_numpy(l["b"]).to(cuda_device),
                            f16=True)
        if l["relu"]:
            m = m >> rdv.relu
    x = rng.uniform(-1, 1, size=(5000, 3)).astype(np.float32)
    got = m(rdv.wrap(torch.from_numpy(x).to(cuda_device))).as_tensor("torch").cpu().numpy()
    feats = oten.tensor_sampler(grid, x)
    ref = omlp.mlp_forward(feats, layers, tail_exact=True)
    nw, el = omlp.rel_errors(got, ref)
    assert nw <= 1e-2 and el <= 1e-2, (nw, el)
    assert got.shape == (5000, 4)


def test_sampler_shapes_and_empty(rdv, cuda_device):
    t = torch.randn(4, 5, 3, device=cuda_device)
    s = rdv.TensorSampler(t)
    assert (s.IN, s.OUT) == (2, 3)
    out = s(torch.zeros(0, 2, device=cuda_device)).as_tensor("torch")
    assert tuple(out.shape) == (0, 3)
    out = s(torch.zeros(2, 7, 2, device=cuda_device)).as_tensor("torch")
    assert tuple(out.shape) == (2, 7, 3)
    # the centre of a 1-cell-per-axis grid returns that cell
    one = torch.arange(6.0, device=cuda_device).reshape(1, 1, 6)
    v = rdv.TensorSampler(one)(torch.zeros(1, 2, device=cuda_device)).as_tensor("torch")
    assert torch.equal(v.cpu(), torch.arange(6.0).reshape(1, 6))
    assert rdv.device_status() == 0


# ------------------------------------------------------------- GridSampler
_GRID_PAIRS = ((1, 3), (2, 3), (3, 3), (4, 3), (3, 5))


@pytest.mark.parametrize("c", range(len(_GRID_PAIRS)))
def test_grid_sampler_bit_exact_vs_reference_fixture(rdv, cuda_device, golden, c):
    """GridSampler over a TensorGrid against the reference's own
    grid_sampler.h outputs (tests/golden/grid_sampler.npz): every (clamp,
    aligned, linear), IN 1..4, bit for bit (both round every product and
    sum separately in the same order)."""
    g = golden("grid_sampler.npz")
    t, x, ys = g[f"t{c}"], g[f"x{c}"], g[f"y{c}"]
    grid = rdv.TensorGrid(torch.from_numpy(t).to(cuda_device))
    for f in range(8):
        s = rdv.GridSampler(grid, clamp=bool(f & 1), aligned=bool(f & 2), linear=bool(f & 4))
        assert (s.IN, s.OUT) == _GRID_PAIRS[c]
        got = s(torch.from_numpy(x).to(cuda_device)).as_tensor("torch").cpu().numpy()
        np.testing.assert_array_equal(got, ys[f], err_msg=f"flags {f}")
    assert rdv.device_status() == 0


def test_grid_sampler_full_size_against_oracle(rdv, cuda_device):
    """A 64^3 x 8 grid at 2^22 points: bit-exact to the oracle on every 97th
    point; constant grids return the constant (partition of unity of the
    corner weights, up to rounding) wherever all corners are inside."""
    rng = np.random.default_rng(17)
    t = rng.standard_normal((64, 64, 64, 8)).astype(np.float32)
    x = rng.uniform(-1.05, 1.05, (1 << 22, 3)).astype(np.float32)
    dev_t = torch.from_numpy(t).to(cuda_device)
    xs = torch.from_numpy(x).to(cuda_device)
    for clamp, aligned in ((True, False), (False, True)):
        got = rdv.GridSampler(dev_t, clamp=clamp, aligned=aligned)(xs).as_tensor("torch")
        sub = np.arange(0, x.shape[0], 97)
        np.testing.assert_array_equal(got.cpu().numpy()[sub], oten.grid_sampler(t, x[sub], clamp, aligned))
    ones = torch.full((64, 64, 64, 2), 2.5, device=cuda_device)
    v = rdv.GridSampler(ones, clamp=True)(xs).as_tensor("torch").cpu().numpy()
    np.testing.assert_allclose(v, 2.5, rtol=1e-6)
    assert rdv.device_status() == 0


def test_grid_sampler_feeds_fused_mlp(rdv, cuda_device):
    """GridSampler >> LinearFast chain: the sampler launch, then the fused
    tensor-core MLP on its features."""
    rng = np.random.default_rng(5)
    grid = rng.standard_normal((8, 8, 8, 16)).astype(np.float32)
    dims = [16, 64, 4]
    layers = [{"W": (rng.standard_normal((dims[i + 1], dims[i])) * np.sqrt(2.0 / dims[i])).astype(np.float32),
               "b": (rng.standard_normal(dims[i + 1]) * 0.1).astype(np.float32), "math": "f16", "relu": i < 1}
              for i in range(2)]
    m = rdv.GridSampler(rdv.TensorGrid(torch.from_numpy(grid).to(cuda_device)), aligned=True)
    for l in layers:
        m = m >> rdv.linear(torch.from_numpy(l["W"]).to(cuda_device), torch.from_numpy(l["b"]).to(cuda_device),
                            f16=True)
        if l["relu"]:
            m = m >> rdv.relu
    x = rng.uniform(-1, 1, size=(5000, 3)).astype(np.float32)
    got = m(rdv.wrap(torch.from_numpy(x).to(cuda_device))).as_tensor("torch").cpu().numpy()
    ref = omlp.mlp_forward(oten.grid_sampler(grid, x, aligned=True), layers, tail_exact=True)
    nw, el = omlp.rel_errors(got, ref)
    assert nw <= 1e-2 and el <= 1e-2, (nw, el)
    empty = rdv.GridSampler(torch.from_numpy(grid).to(cuda_device))(torch.zeros(0, 3, device=cuda_device))
    assert tuple(empty.as_tensor("torch").shape) == (0, 16)


@pytest.mark.parametrize("entry", ["rdvb_grid_sampler", "rdvb_tensor_sampler"])
@pytest.mark.parametrize("flags", [(1, 0, 1), (0, 1, 1), (0, 0, 0), (1, 1, 0)])
def test_vec4_sampler_kernel_matches_per_channel_kernel(rdv, cuda_device, entry, flags):
    """3-D samplers with out % 4 == 0 and 16-byte aligned operands run the
    4-channel kernel (one thread per point and 4 channels, 16-byte corner
    loads); an output 4 bytes off alignment takes the per-channel kernel.
    Both restate the same per-channel arithmetic: equal bit for bit."""
    import rdv_project_b200._native as N
    clamp, aligned, linear = flags
    g = torch.Generator().manual_seed(sum(flags) + len(entry))
    grid = torch.randn(11, 7, 13, 12, generator=g).to(cuda_device)
    n = 30001
    x = (torch.rand(n, 3, generator=g) * 2.6 - 1.3).to(cuda_device)
    shape = N.int_array([11, 7, 13])
    fast = torch.empty(n, 12, device=cuda_device)
    slow_buf = torch.empty(n * 12 + 1, device=cuda_device)
    slow = slow_buf[1:].view(n, 12)
    fn = getattr(N.lib(), entry)
    for y in (fast, slow):
        N.check(fn(grid.data_ptr(), 3, shape, 12, x.data_ptr(), n, clamp, aligned, linear, y.data_ptr(),
                   torch.cuda.current_stream().cuda_stream), entry)
    torch.cuda.synchronize()
    assert torch.equal(fast, slow)
    ref = (oten.grid_sampler if entry == "rdvb_grid_sampler" else oten.tensor_sampler)(
        grid.cpu().numpy(), x.cpu().numpy(), bool(clamp), bool(aligned), bool(linear))
    nw, el = omlp.rel_errors(fast.cpu().numpy(), ref)
    assert nw <= 1e-5 and el <= 1e-5, (nw, el)
