"""The allocation-free MLP entry point, rdvb_mlp_forward_static, through the
C ABI: on two calls in a row (different weights each time, so the library's
static weight image is rewritten) it must give the results of
rdvb_mlp_forward with a caller-packed buffer, and both must meet the oracle
(oracle/mlp.py, the reference's LinearFast / Linear arithmetic) within the
BASELINE tolerances; a run of calls must leave the device's free memory
unchanged. Collected last so it also runs after every other GPU test in the
same process."""
import numpy as np
import pytest
import torch

from oracle import mlp as omlp

pytestmark = pytest.mark.gpu


def _layers(dims, seed):
    g = torch.Generator().manual_seed(seed)
    Ws = [torch.randn(dims[i + 1], dims[i], generator=g) * (2.0 / dims[i]) ** 0.5 for i in range(len(dims) - 1)]
    bs = [torch.randn(dims[i + 1], generator=g) * 0.1 for i in range(len(dims) - 1)]
    return Ws, bs


def _existing(N, x, Ws, bs, dims, flags):
    lib = N.lib()
    n = len(Ws)
    packed = None
    nbytes = lib.rdvb_mlp_packed_bytes(n, N.int_array(dims))
    if nbytes > 0 and flags[0] & 3:
        packed = torch.empty(int(nbytes), dtype=torch.uint8, device=x.device)
        N.check(lib.rdvb_mlp_pack(n, N.int_array(dims), N.ptr_array([w.data_ptr() for w in Ws]),
                                  N.ptr_array([b.data_ptr() for b in bs]),
                                  N.RDVB_BF16 if (flags[0] & 3) == N.RDVB_MATH_BF16 else N.RDVB_F16,
                                  packed.data_ptr(), None), "rdvb_mlp_pack")
    y = torch.empty(x.shape[0], dims[-1], device=x.device)
    N.check(lib.rdvb_mlp_forward(x.data_ptr(), N.RDVB_F32, x.shape[0], n, N.int_array(dims),
                                 N.ptr_array([w.data_ptr() for w in Ws]), N.ptr_array([b.data_ptr() for b in bs]),
                                 N.int_array(flags), 0, 1, packed.data_ptr() if packed is not None else None,
                                 y.data_ptr(), None), "rdvb_mlp_forward")
    return y


def _static(N, x, Ws, bs, dims, flags):
    y = torch.empty(x.shape[0], dims[-1], device=x.device)
    N.check(N.lib().rdvb_mlp_forward_static(x.data_ptr(), N.RDVB_F32, x.shape[0], len(Ws), N.int_array(dims),
                                            N.ptr_array([w.data_ptr() for w in Ws]),
                                            N.ptr_array([b.data_ptr() for b in bs]), N.int_array(flags), 0, 1,
                                            y.data_ptr(), None), "rdvb_mlp_forward_static")
    return y


@pytest.mark.parametrize("dims,math_", [([32] + [128] * 8 + [16], 1), ([3, 64, 64, 4], 2), ([3, 64, 64, 64, 4], 0)])
def test_static_matches_caller_packed_two_calls_in_a_row(cuda_device, dims, math_):
    import rdv_project_b200._native as N

    flags = [math_ | (N.RDVB_LAYER_RELU if i < len(dims) - 2 else 0) for i in range(len(dims) - 1)]
    x_host = torch.rand(4096 + 7, dims[0], generator=torch.Generator().manual_seed(3)) * 2 - 1
    x = x_host.to(cuda_device)
    if math_:
        # the tensor-core kernel takes these chains, so the static image is written and read
        y_probe = torch.empty(x.shape[0], dims[-1], device=cuda_device)
        probe = torch.empty(256, dtype=torch.uint8, device=cuda_device)
        assert N.lib().rdvb_mlp_forward_path(x.data_ptr(), N.RDVB_F32, x.shape[0], len(dims) - 1,
                                             N.int_array(dims), N.int_array(flags), probe.data_ptr(),
                                             y_probe.data_ptr()) == N.RDVB_PATH_TENSOR_CORE
    tol = {0: 1e-5, 1: 1e-2, 2: 1e-2}[math_]
    for seed in (11, 12):  # second call: new weights, so the static image is rewritten
        Ws, bs = _layers(dims, seed)
        layers = [{"W": w.numpy(), "b": b.numpy(), "math": {0: "f32", 1: "f16", 2: "bf16"}[math_],
                   "relu": i < len(dims) - 2} for i, (w, b) in enumerate(zip(Ws, bs))]
        Ws = [w.to(cuda_device) for w in Ws]
        bs = [b.to(cuda_device) for b in bs]
        ref = _existing(N, x, Ws, bs, dims, flags)
        got = _static(N, x, Ws, bs, dims, flags)
        torch.cuda.synchronize()
        assert float((got - ref).abs().max()) <= 1e-6 * float(ref.abs().max())
        oracle = omlp.mlp_forward(x_host.numpy(), layers, tail_exact=True)
        for y in (got, ref):
            nw, el = omlp.rel_errors(y.cpu().numpy(), oracle)
            assert nw <= tol and el <= tol, (nw, el)
    import rdv_project_b200 as rdv

    assert rdv.device_status() == 0


def test_static_calls_allocate_nothing(cuda_device):
    """After a first call (which looks up the static array's address), more
    calls leave the device's free memory exactly where it was."""
    import rdv_project_b200._native as N

    dims = [3, 64, 64, 64, 4]
    flags = [N.RDVB_MATH_F16 | N.RDVB_LAYER_RELU] * 3 + [N.RDVB_MATH_F16]
    Ws, bs = _layers(dims, 21)
    Ws = [w.to(cuda_device) for w in Ws]
    bs = [b.to(cuda_device) for b in bs]
    x = (torch.rand(65536, 3, generator=torch.Generator().manual_seed(4)) * 2 - 1).to(cuda_device)
    y = torch.empty(65536, 4, device=cuda_device)
    args = (x.data_ptr(), N.RDVB_F32, 65536, 4, N.int_array(dims), N.ptr_array([w.data_ptr() for w in Ws]),
            N.ptr_array([b.data_ptr() for b in bs]), N.int_array(flags), 0, 1, y.data_ptr(), None)
    N.check(N.lib().rdvb_mlp_forward_static(*args), "rdvb_mlp_forward_static")
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda_device)
    for _ in range(5):
        N.check(N.lib().rdvb_mlp_forward_static(*args), "rdvb_mlp_forward_static")
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda_device)
    assert free1 == free0
    assert np.isfinite(y.cpu().numpy()).all()


def test_static_rejected_call_leaves_the_image(cuda_device):
    """A call rejected for its arguments returns before touching the static
    array: the next good call on the same weights still matches the
    caller-packed path."""
    import rdv_project_b200._native as N

    dims = [3, 64, 64, 4]
    flags = [N.RDVB_MATH_F16 | N.RDVB_LAYER_RELU] * 2 + [N.RDVB_MATH_F16]
    Ws, bs = _layers(dims, 31)
    Ws = [w.to(cuda_device) for w in Ws]
    bs = [b.to(cuda_device) for b in bs]
    x = (torch.rand(2048, 3, generator=torch.Generator().manual_seed(6)) * 2 - 1).to(cuda_device)
    first = _static(N, x, Ws, bs, dims, flags)
    y = torch.empty(2048, 4, device=cuda_device)
    rc = N.lib().rdvb_mlp_forward_static(x.data_ptr(), 9, 2048, 3, N.int_array(dims),
                                         N.ptr_array([w.data_ptr() for w in Ws]),
                                         N.ptr_array([b.data_ptr() for b in bs]), N.int_array(flags), 0, 1,
                                         y.data_ptr(), None)
    assert rc == N.RDVB_ERR_INVALID_ARG and "x_dtype" in N.last_error()
    again = _static(N, x, Ws, bs, dims, flags)
    torch.cuda.synchronize()
    assert torch.equal(first, again)


def test_static_capacity_limit(cuda_device):
    import rdv_project_b200._native as N

    lib = N.lib()
    assert lib.rdvb_mlp_static_capacity() == 256 * 1024
    dims = [128] * 11  # 10 layers of 128x128 float16: 320 KB of weights
    Ws, bs = _layers(dims, 5)
    Ws = [w.to(cuda_device) for w in Ws]
    bs = [b.to(cuda_device) for b in bs]
    y = torch.empty(64, 128, device=cuda_device)
    x = torch.zeros(64, 128, device=cuda_device)
    rc = lib.rdvb_mlp_forward_static(x.data_ptr(), N.RDVB_F32, 64, 10, N.int_array(dims),
                                     N.ptr_array([w.data_ptr() for w in Ws]), N.ptr_array([b.data_ptr() for b in bs]),
                                     N.int_array([N.RDVB_MATH_F16 | N.RDVB_LAYER_RELU] * 10), 0, 1, y.data_ptr(), None)
    assert rc == -2  # RDVB_ERR_UNSUPPORTED
    assert "holds at most" in N.last_error()
