"""GPU parity of the reference's tensor-core direct convolutions
(Conv2DTensorOpFast / Simple / Simple3x3 / Window3x3) and of the
resampling / concatenation tensor ops.

* Convolutions: against oracle/tensors.conv2d_staged (x and w rounded to
  float16, float64 sums) -- BASELINE's float16 tolerance 1e-2, normwise and
  elementwise, with a tighter 1e-4 asserted (the GPU sums exact products in
  fp32).
* Downsample2x / Upsample2x / Concat: bit-exact against the golden vectors
  the reference's own shader functions produced (tests/golden/resample.npz)
  and against the oracle on larger shapes.
"""
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


def _data(h, w, cin, cout, kh=3, kw=3, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(h * w, cin, generator=g)
    wt = torch.randn(kh, kw, cin, cout, generator=g) * (2.0 / (kh * kw * cin)) ** 0.5
    b = torch.randn(cout, generator=g) * 0.1
    return x, wt, b


@pytest.mark.parametrize("cls,kh,kw,h,w,cin,cout", [
    ("Conv2DTensorOpFast", 3, 3, 16, 16, 16, 32),
    ("Conv2DTensorOpFast", 5, 3, 8, 12, 32, 16),
    ("Conv2DTensorOpSimple", 3, 5, 16, 8, 16, 48),
    ("Conv2DTensorOpSimple3x3", 3, 3, 32, 32, 32, 32),
    ("Conv2DTensorOpSimple3x3", 3, 3, 8, 4, 16, 16),
    ("Conv2DTensorOpWindow3x3", 3, 3, 24, 16, 64, 32),
])
def test_staged_convolutions_match_oracle(rdv, cuda_device, cls, kh, kw, h, w, cin, cout):
    x, wt, b = _data(h, w, cin, cout, kh, kw)
    op = getattr(rdv, cls)(x.to(cuda_device), wt.to(cuda_device), b.to(cuda_device), h, w)
    got = op.as_type("torch").cpu().numpy()
    ref = oten.conv2d_staged(x.numpy(), wt.numpy(), b.numpy(), h, w, "f16")
    nw, el = omlp.rel_errors(got, ref)
    assert nw <= 1e-4 and el <= 1e-4, (nw, el)
    assert got.shape == (h * w, cout)


def test_fast_adds_bias_after_and_simple_seeds_it(rdv, cuda_device):
    """Same data through both bias conventions: equal within fp32 rounding."""
    x, wt, b = _data(16, 16, 16, 16, seed=3)
    a = rdv.Conv2DTensorOpFast(x.to(cuda_device), wt.to(cuda_device), b.to(cuda_device), 16, 16)
    s = rdv.Conv2DTensorOpSimple3x3(x.to(cuda_device), wt.to(cuda_device), b.to(cuda_device), 16, 16)
    torch.testing.assert_close(a.as_type("torch"), s.as_type("torch"), rtol=1e-5, atol=1e-5)


def test_conv_family_assertions(rdv, cuda_device):
    x, wt, b = _data(8, 8, 16, 16)
    with pytest.raises(AssertionError, match="must be a multiple of 32"):
        rdv.Conv2DTensorOpSimple3x3(torch.zeros(6 * 5, 16, device=cuda_device), wt.to(cuda_device),
                                    b.to(cuda_device), 6, 5)
    with pytest.raises(AssertionError, match="weight must be \\[3, 3"):
        rdv.Conv2DTensorOpSimple3x3(x.to(cuda_device), torch.zeros(5, 5, 16, 16, device=cuda_device),
                                    b.to(cuda_device), 8, 8)
    with pytest.raises(AssertionError, match="must be a multiple of 8"):
        rdv.Conv2DTensorOpWindow3x3(torch.zeros(12 * 8, 16, device=cuda_device), wt.to(cuda_device),
                                    b.to(cuda_device), 12, 8)
    with pytest.raises(AssertionError, match="must be at most 64"):
        rdv.Conv2DTensorOpWindow3x3(torch.zeros(64, 80, device=cuda_device),
                                    torch.zeros(3, 3, 80, 16, device=cuda_device), b.to(cuda_device), 8, 8)
    with pytest.raises(AssertionError, match="in_channels \\(8\\) must be a multiple of 16"):
        rdv.Conv2DTensorOpFast(torch.zeros(64, 8, device=cuda_device), torch.zeros(3, 3, 8, 16, device=cuda_device),
                               b.to(cuda_device), 8, 8)


def test_resample_and_concat_match_reference_golden(rdv, cuda_device, golden):
    g = golden("resample.npz")
    d = rdv.Downsample2xTensorOp(torch.from_numpy(g["down_x"]).to(cuda_device), 8, 12)
    assert np.array_equal(d.as_type("torch").cpu().numpy(), g["down_y"])
    u = rdv.Upsample2xTensorOp(torch.from_numpy(g["up_x"]).to(cuda_device), 4, 6)
    assert np.array_equal(u.as_type("torch").cpu().numpy(), g["up_y"])
    c = rdv.ConcatTensorOp(torch.from_numpy(g["cat_x1"]).to(cuda_device), torch.from_numpy(g["cat_x2"]).to(cuda_device))
    assert np.array_equal(c.as_type("torch").cpu().numpy(), g["cat_y"])


def test_resample_large_and_unet_style_chain(rdv, cuda_device):
    """Down -> conv -> up -> concat with the skip connection; every op
    against the oracle (bit-exact for the data movement), then an in-place
    edit of the input and evaluate_chain() over the two-upstream graph."""
    h, w, c = 64, 96, 16
    g = torch.Generator().manual_seed(5)
    x = torch.randn(h * w, c, generator=g).to(cuda_device)
    d = rdv.Downsample2xTensorOp(x, h, w)
    _, wt, b = _data(h // 2, w // 2, c, c, seed=6)
    conv = rdv.Conv2DTensorOpSimple3x3(d, wt.to(cuda_device), b.to(cuda_device), h // 2, w // 2)
    u = rdv.Upsample2xTensorOp(conv, h // 2, w // 2)
    cat = rdv.ConcatTensorOp(x, u)
    xd = oten.downsample2x(x.cpu().numpy(), h, w)
    assert np.array_equal(d.as_type("torch").cpu().numpy(), xd)
    ref_conv = oten.conv2d_staged(xd, wt.numpy(), b.numpy(), h // 2, w // 2)
    nw, el = omlp.rel_errors(conv.as_type("torch").cpu().numpy(), ref_conv)
    assert nw <= 1e-4 and el <= 1e-4
    assert np.array_equal(u.as_type("torch").cpu().numpy(), oten.upsample2x(conv.as_type("torch").cpu().numpy(),
                                                                           h // 2, w // 2))
    assert np.array_equal(cat.as_type("torch").cpu().numpy(),
                          oten.concat(x.cpu().numpy(), u.as_type("torch").cpu().numpy()))
    x.mul_(-0.5)
    cat.evaluate_chain()
    xd2 = oten.downsample2x(x.cpu().numpy(), h, w)
    conv2 = oten.conv2d_staged(xd2, wt.numpy(), b.numpy(), h // 2, w // 2)
    got = cat.as_type("torch").cpu().numpy()
    assert np.array_equal(got[:, :c], x.cpu().numpy())
    nw, el = omlp.rel_errors(got[:, c:], oten.upsample2x(conv2, h // 2, w // 2))
    assert nw <= 1e-4 and el <= 1e-4
    assert rdv.device_status() == 0


def _tc_conv(N, x, wt, b, n, h, w, operand):
    cin, cout = wt.shape[2], wt.shape[3]
    kh, kw = wt.shape[0], wt.shape[1]
    lib = N.lib()
    nbytes = lib.rdvb_conv_tc_packed_bytes(kh, kw, cin, cout)
    assert nbytes > 0
    wp = torch.empty(int(nbytes), dtype=torch.uint8, device=x.device)
    N.check(lib.rdvb_conv_tc_pack(wt.data_ptr(), kh, kw, cin, cout, operand, wp.data_ptr(), None), "pack")
    y = torch.full((n * h * w, cout), float("nan"), device=x.device)
    N.check(lib.rdvb_conv2d_tc(x.data_ptr(), N.RDVB_F16 if x.dtype == torch.float16 else N.RDVB_F32, n, h, w, cin,
                               cout, kh, kw, wp.data_ptr(), operand, b.data_ptr(), y.data_ptr(), None), "conv_tc")
    return y


@pytest.mark.parametrize("n,h,w,cin,cout,kh,kw,operand", [
    (1, 160, 160, 16, 16, 3, 3, "f16"),    # 200 blocks: several per CTA, both accumulator halves
    (2, 37, 53, 64, 128, 3, 3, "f16"),     # ragged last block, two images
    (3, 24, 24, 32, 32, 5, 5, "bf16"),     # 25 taps, bfloat16 operands
    (1, 64, 64, 48, 256, 1, 1, "f16"),     # 1x1, widest output
])
def test_tensor_core_conv_matches_oracle(rdv, cuda_device, n, h, w, cin, cout, kh, kw, operand):
    import rdv_project_b200._native as N
    from oracle import winograd as owg
    from oracle.mlp import stage

    g = torch.Generator().manual_seed(n * 100 + cin)
    x = torch.randn(n * h * w, cin, generator=g)
    wt = torch.randn(kh, kw, cin, cout, generator=g) * (2.0 / (kh * kw * cin)) ** 0.5
    b = torch.randn(cout, generator=g) * 0.1
    op = N.RDVB_F16 if operand == "f16" else N.RDVB_BF16
    xd, wd, bd = x.to(cuda_device), wt.to(cuda_device), b.to(cuda_device)  # alive while the kernels run
    y = _tc_conv(N, xd, wd, bd, n, h, w, op)
    torch.cuda.synchronize()
    xs = stage(x.numpy(), operand).reshape(n, h, w, cin)
    ref = owg.conv2d_direct(xs, stage(wt.numpy(), operand), b.numpy()).reshape(n * h * w, cout)
    got = y.cpu().numpy()
    assert not np.isnan(got).any()
    nw, el = omlp.rel_errors(got, ref)
    assert nw <= 1e-4 and el <= 1e-4, (nw, el)
    # the CUDA-core kernel on the same staged operands agrees to fp32 rounding
    if operand == "f16" and n == 1:
        y2 = torch.empty_like(y)
        N.check(N.lib().rdvb_conv2d_direct_staged(
            xd.data_ptr(), N.RDVB_F32, n, h, w, cin, cout, kh, kw, wd.data_ptr(), bd.data_ptr(), N.RDVB_MATH_F16, 0,
            y2.data_ptr(), None), "staged")
        torch.testing.assert_close(y, y2, rtol=2e-5, atol=2e-5)
    assert rdv.device_status() == 0


def test_shapes_outside_tensor_core_limits_take_cuda_cores(rdv, cuda_device):
    import rdv_project_b200._native as N

    assert N.lib().rdvb_conv_tc_packed_bytes(3, 3, 96, 32) == 0   # cin > 64
    assert N.lib().rdvb_conv_tc_packed_bytes(7, 7, 16, 16) == 0   # 49 taps
    x, wt, b = _data(16, 16, 96, 32, seed=9)
    op = rdv.Conv2DTensorOpFast(x.to(cuda_device), wt.to(cuda_device), b.to(cuda_device), 16, 16)
    ref = oten.conv2d_staged(x.numpy(), wt.numpy(), b.numpy(), 16, 16, "f16")
    nw, el = omlp.rel_errors(op.as_type("torch").cpu().numpy(), ref)
    assert nw <= 1e-4 and el <= 1e-4


@pytest.mark.parametrize("n,h,w,cout,kh,kw", [
    (1, 40, 48, 64, 3, 3),      # whole 8x16 blocks
    (2, 37, 53, 128, 3, 3),     # ragged blocks at the bottom and right edges, two images
    (1, 24, 32, 32, 5, 5),      # 25 taps, halo of 2
    (3, 9, 17, 256, 1, 1),      # 1x1, widest output, one-row-deep blocks
])
def test_tma_fed_conv_matches_oracle_and_staging_kernel(rdv, cuda_device, monkeypatch, n, h, w, cout, kh, kw):
    """float16 input with 64 channels and float16 operands runs the TMA-fed
    kernel (input boxes loaded by the copy engine, border zero-filled); it
    must agree with the oracle and with the staging kernel on the same data."""
    import rdv_project_b200._native as N
    from oracle import winograd as owg
    from oracle.mlp import stage

    cin = 64
    g = torch.Generator().manual_seed(h * 1000 + w)
    x = torch.randn(n * h * w, cin, generator=g).half()
    wt = torch.randn(kh, kw, cin, cout, generator=g) * (2.0 / (kh * kw * cin)) ** 0.5
    b = torch.randn(cout, generator=g) * 0.1
    xd, wd, bd = x.to(cuda_device), wt.to(cuda_device), b.to(cuda_device)
    launches = N.launch_count()
    y = _tc_conv(N, xd, wd, bd, n, h, w, N.RDVB_F16)
    torch.cuda.synchronize()
    ref = owg.conv2d_direct(x.float().numpy().reshape(n, h, w, cin), stage(wt.numpy(), "f16"),
                            b.numpy()).reshape(n * h * w, cout)
    got = y.cpu().numpy()
    assert not np.isnan(got).any()
    nw, el = omlp.rel_errors(got, ref)
    assert nw <= 1e-4 and el <= 1e-4, (nw, el)
    monkeypatch.setenv("RDVB_CONV_TMA", "0")
    y2 = _tc_conv(N, xd, wd, bd, n, h, w, N.RDVB_F16)
    torch.cuda.synchronize()
    torch.testing.assert_close(y, y2, rtol=2e-5, atol=2e-5)
    assert N.launch_count() > launches
    assert rdv.device_status() == 0
