"""GPU tests of the pipelined evaluators on one device: the host-streaming
pipeline (pieces copied in on a copy stream, kernels writing into the final
buffer, rows copied back on a second stream), the CTA cap of the persistent
MLP kernel, evaluate_into on buffer slices, and the aligned copy a
misaligned input gets. Each must give exactly what one ``m(x)`` call gives,
and that call meets the oracle (oracle/mlp.py)."""
import numpy as np
import pytest
import torch

from oracle import mlp as omlp

pytestmark = pytest.mark.gpu


def _layers(dims, seed=0):
    rng = np.random.default_rng(seed)
    return [{"W": (rng.standard_normal((dims[i + 1], dims[i])) * np.sqrt(2.0 / dims[i])).astype(np.float32),
             "b": (rng.standard_normal(dims[i + 1]) * 0.1).astype(np.float32), "math": "f16",
             "relu": i < len(dims) - 2} for i in range(len(dims) - 1)]


def _build(rdv, layers, dev):
    m = None
    for l in layers:
        lin = rdv.LinearFast(torch.from_numpy(l["W"]).to(dev), torch.from_numpy(l["b"]).to(dev))
        m = lin if m is None else m >> lin
        if l["relu"]:
            m = m >> rdv.relu
    return m


@pytest.mark.parametrize("n,chunks", [(128 * 300, 5), (128 * 300 + 45, 7), (1000, 16)])
def test_host_streaming_equals_one_call(cuda_device, n, chunks):
    import rdv_project_b200 as rdv
    from rdv_project_b200.sharding import sharded_map_overlapped

    layers = _layers([3, 64, 64, 64, 64, 4])
    m = _build(rdv, layers, cuda_device)
    x = torch.rand(n, 3, generator=torch.Generator().manual_seed(1)) * 2 - 1
    want = m(rdv.wrap(x.to(cuda_device))).as_tensor("torch").clone()
    x_pin = x.pin_memory()
    y_pin = torch.full((n, 4), float("nan")).pin_memory()
    out = torch.full((n, 4), float("nan"), device=cuda_device)
    for _ in range(2):  # the second call reuses the staging ring
        sharded_map_overlapped(m, x_host=x_pin, y_host=y_pin, out=out, chunks=chunks)
        torch.cuda.synchronize()
        assert torch.equal(out, want)
        assert torch.equal(y_pin, want.cpu())
    nw, el = omlp.rel_errors(want.cpu().numpy(), omlp.mlp_forward(x.numpy(), layers, tail_exact=True))
    assert nw <= 1e-2 and el <= 1e-2
    assert rdv.device_status() == 0


def test_device_input_slabs_and_cta_cap(cuda_device):
    import rdv_project_b200 as rdv
    from rdv_project_b200 import _native as N
    from rdv_project_b200.sharding import sharded_map_overlapped

    layers = _layers([32, 128, 128, 16], seed=2)
    m = _build(rdv, layers, cuda_device)
    n = 128 * 1000 + 77
    x = (torch.randn(n, 32, generator=torch.Generator().manual_seed(3))).to(cuda_device)
    want = m(rdv.wrap(x)).as_tensor("torch").clone()
    out = torch.empty(n, 16, device=cuda_device)
    sharded_map_overlapped(m, x, out=out, chunks=6)
    assert torch.equal(out, want)
    for cap in (1, 7, 100):
        prev = N.set_max_ctas(cap)
        try:
            got = m(rdv.wrap(x)).as_tensor("torch")
            torch.cuda.synchronize()
            assert torch.equal(got, want), cap
        finally:
            N.set_max_ctas(prev)
    assert rdv.device_status() == 0


def test_evaluate_into_slices_and_misaligned_input(cuda_device):
    import rdv_project_b200 as rdv
    from rdv_project_b200 import _native as N
    from rdv_project_b200.maps import evaluate_into

    layers = _layers([3, 64, 64, 4], seed=4)
    m = _build(rdv, layers, cuda_device)
    x = (torch.rand(4097, 3, generator=torch.Generator().manual_seed(5)) * 2 - 1).to(cuda_device)
    xs = x[1:]  # 12 bytes past the allocation: not 16-byte aligned
    assert xs.data_ptr() % 16 != 0
    want = m(rdv.wrap(xs.clone())).as_tensor("torch").clone()
    got = m(rdv.wrap(xs)).as_tensor("torch")
    assert torch.equal(got, want)
    out = torch.full((5000, 4), float("nan"), device=cuda_device)
    evaluate_into(m, xs, out[100:100 + 4096])
    assert torch.equal(out[100:4196], want)
    assert torch.isnan(out[:100]).all() and torch.isnan(out[4196:]).all()
    # the aligned copy is what the tensor-core kernel sees
    plan = next(iter(m._plans.values()))
    dims = N.int_array(plan.dims)
    flags = N.int_array(plan.flags)
    aligned = xs.clone()
    assert N.lib().rdvb_mlp_forward_path(aligned.data_ptr(), N.RDVB_F32, 4096, len(plan.dims) - 1, dims, flags,
                                         plan.packed.data_ptr(), out.data_ptr()) == N.RDVB_PATH_TENSOR_CORE
    assert N.lib().rdvb_mlp_forward_path(xs.data_ptr(), N.RDVB_F32, 4096, len(plan.dims) - 1, dims, flags,
                                         plan.packed.data_ptr(), out.data_ptr()) == N.RDVB_PATH_CUDA_CORE
    with pytest.raises(ValueError):
        evaluate_into(m, xs, out[:10])
