"""GPU parity of the Winograd F(2x2,3x3) operator and the direct convolution.

Checks, all through the C ABI (librdvb.so):
* the filter transform is bit-identical to the reference's own torch helper
  (golden fixture from rdv/domain/nn.py:525-538);
* the fused kernel matches the oracle with the same float16 staging of U and
  V at fp32 level (TIGHT: only the fp32 summation order differs), and the
  float64 direct convolution within BASELINE's float16 tolerance (1e-2,
  normwise and elementwise, oracle.mlp.rel_errors);
* the reference-layout TensorOperation forms reproduce the reference's direct
  convolution shader output (golden, compiled from conv2d_tensor_op.h);
* multi-block / partial-block / odd-size / every channel combination, and
  the BASELINE config-3 size (8x256x256x64) against the on-device fp32
  direct convolution.
"""
import numpy as np
import pytest
import torch

from oracle import mlp as omlp
from oracle import winograd as owg

pytestmark = pytest.mark.gpu

TOL_F16 = 1e-2   # BASELINE: float16 operands, fp32 accumulation
TOL_F32 = 1e-5   # BASELINE: fp32
TIGHT = 2e-5     # GPU vs the identically staged oracle


@pytest.fixture(scope="module")
def rdv():
    import rdv_project_b200 as rdv
    return rdv


def _weights(rng, cin, cout, bias_scale=0.1):
    w = (rng.standard_normal((3, 3, cin, cout)) * np.sqrt(2.0 / (9 * cin))).astype(np.float32)
    b = (rng.standard_normal(cout) * bias_scale).astype(np.float32)
    return w, b


def _oracle_staged(x, w, b):
    """Staged-oracle Winograd for any H, W: zero-extends odd sizes to whole
    2x2 tiles (the extra row/column is the 'same' padding) and crops."""
    n, h, wd, c = x.shape
    H2, W2 = h + (h & 1), wd + (wd & 1)
    xp = np.zeros((n, H2, W2, c), dtype=np.float32)
    xp[:, :h, :wd] = x
    return owg.conv3x3_winograd(xp, w, b, "F2x2", staged=True)[:, :h, :wd]


def _check(y, ref, tol):
    nw, el = omlp.rel_errors(np.asarray(y, dtype=np.float64), np.asarray(ref, dtype=np.float64))
    assert nw <= tol and el <= tol, (nw, el)
    return nw, el


def test_filter_transform_bit_exact_vs_reference_helper(rdv, cuda_device, golden):
    g = golden("winograd.npz")
    U = rdv._winograd_transform_weight(torch.from_numpy(g["w"]), 16, 32)
    assert U.dtype == torch.float16 and U.shape == (16 * 16 * 32,)
    np.testing.assert_array_equal(U.cpu().numpy().view(np.uint16), g["U"].view(np.uint16))


@pytest.mark.parametrize("cin,cout", [(16, 16), (16, 32), (32, 16), (48, 48), (64, 64), (64, 32), (32, 64)])
@pytest.mark.parametrize("xdt", ["f32", "f16"])
def test_winograd_matches_oracle(rdv, cuda_device, cin, cout, xdt):
    rng = np.random.default_rng(cin * 100 + cout)
    x = rng.standard_normal((2, 12, 20, cin)).astype(np.float32)
    if xdt == "f16":
        x = x.astype(np.float16).astype(np.float32)
    w, b = _weights(rng, cin, cout)
    conv = rdv.Conv3x3Winograd(torch.from_numpy(w), torch.from_numpy(b))
    xt = torch.from_numpy(x).to(cuda_device)
    if xdt == "f16":
        xt = xt.half()
    y = conv(xt).cpu().numpy()
    _check(y, _oracle_staged(x, w, b), TIGHT)
    _check(y, owg.conv3x3_direct(x, w, b), TOL_F16)
    assert rdv.device_status() == 0


@pytest.mark.parametrize("shape", [(1, 15, 17), (3, 1, 1), (1, 2, 2), (2, 7, 4), (1, 33, 1)])
def test_winograd_odd_and_tiny_images(rdv, cuda_device, shape):
    n, h, wd = shape
    rng = np.random.default_rng(h * 31 + wd)
    x = rng.standard_normal((n, h, wd, 32)).astype(np.float32)
    w, b = _weights(rng, 32, 16)
    y = rdv.Conv3x3Winograd(torch.from_numpy(w), torch.from_numpy(b))(torch.from_numpy(x).to(cuda_device))
    y = y.cpu().numpy()
    _check(y, _oracle_staged(x, w, b), TIGHT)
    _check(y, owg.conv3x3_direct(x, w, b), TOL_F16)


def test_winograd_many_blocks_per_cta(rdv, cuda_device):
    # 8*64*64 = 32768 tiles = 256 blocks of 128: more blocks than SMs, so
    # CTAs loop over blocks and the TMEM/V rings wrap many times
    rng = np.random.default_rng(7)
    x = rng.standard_normal((8, 128, 128, 16)).astype(np.float16).astype(np.float32)
    w, b = _weights(rng, 16, 16)
    conv = rdv.Conv3x3Winograd(torch.from_numpy(w), torch.from_numpy(b))
    y = conv(torch.from_numpy(x).to(cuda_device).half()).cpu().numpy()
    _check(y, _oracle_staged(x, w, b), TIGHT)
    assert rdv.device_status() == 0


def test_winograd_float16_output(rdv, cuda_device):
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.standard_normal((2, 16, 16, 64)).astype(np.float32)).to(cuda_device).half()
    w, b = _weights(rng, 64, 64)
    conv = rdv.Conv3x3Winograd(torch.from_numpy(w), torch.from_numpy(b))
    y32 = conv(x)
    y16 = conv(x, out_dtype=torch.float16)
    assert y16.dtype == torch.float16
    torch.testing.assert_close(y16.float(), y32.half().float(), rtol=0, atol=0)


def test_reference_layout_ops_vs_reference_shader(rdv, cuda_device, golden):
    g = golden("tensor_ops.npz")
    x, w, b, y_ref = g["conv_x"], g["conv_w"], g["conv_b"], g["conv_y"]
    wino = rdv.Conv2DTensorOpWinograd3x3(torch.from_numpy(x), torch.from_numpy(w), torch.from_numpy(b), 16, 16)
    y = wino.as_type("torch").cpu().numpy()
    assert y.shape == (256, 32)
    _check(y, y_ref, TOL_F16)
    direct = rdv.Conv2DTensorOp(torch.from_numpy(x), torch.from_numpy(w), torch.from_numpy(b), 16, 16)
    _check(direct.as_type("torch").cpu().numpy(), y_ref, TOL_F32)


@pytest.mark.parametrize("k", [(1, 1), (3, 3), (5, 5), (3, 1), (2, 2)])
@pytest.mark.parametrize("xdt", ["f32", "f16"])
def test_direct_conv_vs_oracle(rdv, cuda_device, k, xdt):
    rng = np.random.default_rng(k[0] * 10 + k[1])
    x = rng.standard_normal((2, 9, 11, 24)).astype(np.float32)
    if xdt == "f16":
        x = x.astype(np.float16).astype(np.float32)
    w = (rng.standard_normal((k[0], k[1], 24, 16)) * 0.2).astype(np.float32)
    b = rng.standard_normal(16).astype(np.float32)
    xt = torch.from_numpy(x).to(cuda_device)
    y = rdv.conv2d_direct(xt.half() if xdt == "f16" else xt, torch.from_numpy(w), torch.from_numpy(b))
    _check(y.cpu().numpy(), owg.conv2d_direct(x, w, b), TOL_F32)


def test_evaluate_chain_sees_in_place_input_edit(rdv, cuda_device):
    rng = np.random.default_rng(11)
    x = torch.from_numpy(rng.standard_normal((64, 16)).astype(np.float32)).to(cuda_device)
    w, b = _weights(rng, 16, 16)
    op = rdv.Conv2DTensorOpWinograd3x3(x, torch.from_numpy(w), torch.from_numpy(b), 8, 8)
    first = op.as_type("torch").clone()
    x.mul_(2.0)
    op.evaluate_chain()
    second = op.as_type("torch")
    torch.testing.assert_close(second - torch.from_numpy(b).to(cuda_device),
                               2.0 * (first - torch.from_numpy(b).to(cuda_device)), rtol=2e-3, atol=2e-3)


def test_config3_full_size_vs_direct(rdv, cuda_device):
    # x [8, 256, 256, 64] float16 ~N(0,1), Kaiming-normal
    # weights, zero bias, fp32 output; compared against a direct convolution:
    # the oracle's float64 one (conv2d_tensor_op.h:21-87 semantics) on output
    # rows 0-31 of images 0 and 7, and the on-device fp32 one on every pixel
    g = torch.Generator().manual_seed(0)
    x_host = torch.randn((8, 256, 256, 64), generator=g).half()
    x = x_host.to(cuda_device)
    w = torch.randn((64, 64, 3, 3), generator=torch.Generator().manual_seed(1000)) * np.sqrt(2.0 / 576)
    w33io = w.permute(2, 3, 1, 0).contiguous()
    conv = rdv.Conv3x3Winograd(w33io, torch.zeros(64))
    y = conv(x)
    y_host = y.cpu().numpy()
    for img in (0, 7):
        band = owg.conv3x3_direct(x_host[img:img + 1, :33].float().numpy(), w33io.numpy(), np.zeros(64))[0, :32]
        _check(y_host[img, :32], band, TOL_F16)
    ref = rdv.conv2d_direct(x, w33io, torch.zeros(64))
    torch.cuda.synchronize()
    d = (y.double() - ref.double()).abs()
    nw = (d.max() / ref.double().abs().max()).item()
    el = (d / (ref.double().abs() + ref.double().pow(2).mean().sqrt())).max().item()
    assert nw <= TOL_F16 and el <= TOL_F16, (nw, el)
    assert rdv.device_status() == 0


def test_errors_and_empty(rdv, cuda_device):
    import rdv_project_b200._native as N
    lib = N.lib()
    assert lib.rdvb_winograd_packed_bytes(N.RDVB_WINOGRAD_F2X2, 64, 64) == 16 * 64 * 128
    assert lib.rdvb_winograd_packed_bytes(N.RDVB_WINOGRAD_F2X2, 80, 64) == 0
    assert lib.rdvb_winograd_packed_bytes(N.RDVB_WINOGRAD_F4X4, 64, 64) == 36 * 64 * 64 * 4
    dummy = torch.zeros(1 << 16, device=cuda_device)
    # n = 0: nothing to do, no launch
    before = N.launch_count()
    N.check(lib.rdvb_conv3x3_winograd(dummy.data_ptr(), N.RDVB_F32, 0, 8, 8, 16, 16, dummy.data_ptr(),
                                      N.RDVB_WINOGRAD_F2X2, None, dummy.data_ptr(), N.RDVB_F32, None), "empty")
    assert N.launch_count() == before
    rc = lib.rdvb_conv3x3_winograd(dummy.data_ptr(), N.RDVB_F32, 1, 8, 8, 16, 16, dummy.data_ptr(),
                                   7, None, dummy.data_ptr(), N.RDVB_F32, None)
    assert rc == -1 and "variant" in N.last_error()
    rc = lib.rdvb_conv3x3_winograd(dummy.data_ptr(), N.RDVB_F32, 1, 8, 8, 24, 16, dummy.data_ptr(),
                                   N.RDVB_WINOGRAD_F2X2, None, dummy.data_ptr(), N.RDVB_F32, None)
    assert rc == -2 and "multiples of 16" in N.last_error()
    rc = lib.rdvb_conv3x3_winograd(dummy.data_ptr() + 4, N.RDVB_F32, 1, 8, 8, 16, 16, dummy.data_ptr(),
                                   N.RDVB_WINOGRAD_F2X2, None, dummy.data_ptr(), N.RDVB_F32, None)
    assert rc == -1 and "aligned" in N.last_error()
    with pytest.raises(AssertionError, match=r"H \(15\) must be even"):
        rdv.Conv2DTensorOpWinograd3x3(torch.zeros(15 * 8, 16), torch.zeros(3, 3, 16, 16), torch.zeros(16), 15, 8)
    with pytest.raises(AssertionError, match=r"in_channels \(80\) must be at most 64"):
        rdv.Conv2DTensorOpWinograd3x3(torch.zeros(64, 80), torch.zeros(3, 3, 80, 16), torch.zeros(16), 8, 8)


@pytest.mark.parametrize("shape,cout", [((3, 37, 61), 64), ((1, 1, 1), 64), ((2, 17, 31), 32),
                                        ((8, 128, 128), 64), ((1, 33, 100), 48)])
def test_tma_fed_kernel_equals_global_load_kernel(rdv, cuda_device, monkeypatch, shape, cout):
    """float16 input with 64 channels takes the TMA-fed kernel (the block's
    input halo as one box, zero-filled at the border): the same transform
    arithmetic and GEMMs as the global-load kernel, so the outputs are
    bit-identical; both agree with the oracle. (8, 128, 128): 320 blocks,
    more than one per CTA, so the input box and the U ring wrap."""
    n, h, wd = shape
    rng = np.random.default_rng(h * 7 + wd + cout)
    x = rng.standard_normal((n, h, wd, 64)).astype(np.float16).astype(np.float32)
    w, b = _weights(rng, 64, cout)
    conv = rdv.Conv3x3Winograd(torch.from_numpy(w), torch.from_numpy(b))
    xt = torch.from_numpy(x).to(cuda_device).half()
    y_tma = conv(xt)
    y16_tma = conv(xt, out_dtype=torch.float16)
    monkeypatch.setenv("RDVB_WINO_TMA", "0")
    y_ref = conv(xt)
    y16_ref = conv(xt, out_dtype=torch.float16)
    torch.cuda.synchronize()
    assert torch.equal(y_tma, y_ref)
    assert torch.equal(y16_tma, y16_ref)
    if n * h * wd <= 20000:
        _check(y_tma.cpu().numpy(), _oracle_staged(x, w, b), TIGHT)
    assert rdv.device_status() == 0


@pytest.mark.parametrize("c", [16, 48])
def test_reference_winograd_op_vs_reference_coopmat(rdv, cuda_device, golden, c):
    """Conv2DTensorOpWinograd3x3 against the reference's own
    cooperative-matrix body executed on the CPU (tests/golden/coopmat.npz):
    same float16 staging of U and V, so only the fp32 summation order
    differs -- within the tight Winograd bound."""
    g = golden("coopmat.npz")
    x = torch.from_numpy(g[f"wino{c}_x"].reshape(256, c))
    w = torch.from_numpy(g[f"wino{c}_w"].astype(np.float32))
    b = torch.from_numpy(g[f"wino{c}_b"])
    op = rdv.Conv2DTensorOpWinograd3x3(x, w, b, 16, 16)
    y = op.as_type("torch").cpu().numpy().reshape(16, 16, c)
    _check(y, g[f"wino{c}_y"], TIGHT)
