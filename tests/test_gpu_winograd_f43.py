"""GPU parity of the Winograd F(4x4,3x3) path (a B200 extension: the
reference operator is F(2x2,3x3) only), through the C ABI (librdvb.so).
F(4x4) keeps every operand fp32 (float16 U and V would reach ~1.3e-2 of the
output at 64 channels, above the 1e-2 tolerance):

* the filter transform U = G g G^T (fp32) against the oracle's
  (oracle/winograd.py filter_transform, same Toom-Cook matrices);
* the convolution against the oracle's float64 Winograd (same transforms,
  exact arithmetic): normwise TIGHT_F43_NW, elementwise TIGHT_F43_EL -- the
  kernel's fp32 rounding only; a wrong tile, position or constant gives
  errors of order 1;
* the convolution against the float64 direct convolution, elementwise
  within TIGHT_F43_EL too (well inside the float16 tolerance 1e-2);
* channels off the 16 grid, partial 4x4 tiles at the bottom/right edges,
  CTAs that walk several blocks of tiles, both tile-block sizes (8 tiles,
  or 4 when 128 + 128 channels need the shared memory), float16 input and
  output, and the argument checks.
"""
import numpy as np
import pytest
import torch

from oracle import mlp as omlp
from oracle import winograd as owg

pytestmark = pytest.mark.gpu

TIGHT_F43_NW = 2e-5
TIGHT_F43_EL = 2e-4


@pytest.fixture(scope="module")
def rdv():
    import rdv_project_b200 as rdv
    return rdv


def _weights(rng, cin, cout):
    w = (rng.standard_normal((3, 3, cin, cout)) * np.sqrt(2.0 / (9 * cin))).astype(np.float32)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    return w, b


def _oracle_f43(x, w, b):
    """Staged F(4x4) oracle for any H, W: zero-extends to whole 4x4 tiles (the
    extra rows/columns read as the 'same' padding) and crops."""
    n, h, wd, c = x.shape
    H4, W4 = -(-h // 4) * 4, -(-wd // 4) * 4
    xp = np.zeros((n, H4, W4, c), dtype=np.float32)
    xp[:, :h, :wd] = x
    return owg.conv3x3_winograd(xp, w, b, "F4x4", staged=False)[:, :h, :wd]


def _errors(y, ref):
    return omlp.rel_errors(np.asarray(y, dtype=np.float64), np.asarray(ref, dtype=np.float64))


def test_f4x4_filter_transform_vs_oracle(rdv, cuda_device):
    import rdv_project_b200.conv as C
    rng = np.random.default_rng(11)
    w, _ = _weights(rng, 24, 40)
    u, _ = C._filter_transform(torch.from_numpy(w).to(cuda_device), 24, 40, plain=True, packed=False,
                               variant="F4x4")
    assert u.dtype == torch.float32 and u.shape == (36 * 24 * 40,)
    ref = owg.filter_transform(w, "F4x4").reshape(-1)
    np.testing.assert_allclose(u.cpu().numpy(), ref, rtol=2e-6, atol=1e-8)


@pytest.mark.parametrize("cin,cout,xdt,shape", [
    (16, 32, "f32", (2, 12, 16)),
    (64, 64, "f16", (1, 16, 20)),
    (24, 40, "f32", (1, 13, 18)),   # channels off the 16 grid, partial tiles
    (3, 5, "f16", (2, 5, 7)),
    (128, 16, "f32", (1, 8, 8)),
    (128, 128, "f16", (2, 9, 11)),   # 4-tile blocks
    (16, 128, "f16", (1, 4, 4)),
    (32, 16, "f32", (3, 1, 1)),
])
def test_f4x4_matches_oracle(rdv, cuda_device, cin, cout, xdt, shape):
    n, h, wd = shape
    rng = np.random.default_rng(cin * 1000 + cout + h)
    x = rng.standard_normal((n, h, wd, cin)).astype(np.float32)
    if xdt == "f16":
        x = x.astype(np.float16).astype(np.float32)
    w, b = _weights(rng, cin, cout)
    conv = rdv.Conv3x3Winograd(torch.from_numpy(w), torch.from_numpy(b), variant="F4x4")
    xt = torch.from_numpy(x).to(cuda_device)
    if xdt == "f16":
        xt = xt.half()
    y = conv(xt).cpu().numpy()
    nw, el = _errors(y, _oracle_f43(x, w, b))
    assert nw <= TIGHT_F43_NW and el <= TIGHT_F43_EL, (nw, el)
    nw, el = _errors(y, owg.conv3x3_direct(x, w, b))
    assert nw <= TIGHT_F43_NW and el <= TIGHT_F43_EL, (nw, el)
    assert rdv.device_status() == 0


def test_f4x4_many_blocks_per_cta_and_f16_output(rdv, cuda_device):
    # 8 * 32 * 32 = 8192 tiles = 1024 blocks of 8: several blocks per CTA
    rng = np.random.default_rng(5)
    x = rng.standard_normal((8, 128, 128, 16)).astype(np.float16).astype(np.float32)
    w, b = _weights(rng, 16, 16)
    conv = rdv.Conv3x3Winograd(torch.from_numpy(w), torch.from_numpy(b), variant="F4x4")
    xt = torch.from_numpy(x).to(cuda_device).half()
    y = conv(xt)
    y16 = conv(xt, out_dtype=torch.float16)
    torch.cuda.synchronize()
    ref = _oracle_f43(x, w, b)
    nw, el = _errors(y.cpu().numpy(), ref)
    assert nw <= TIGHT_F43_NW and el <= TIGHT_F43_EL, (nw, el)
    # the float16 output is the fp32 result rounded once
    assert torch.equal(y16, y.half())
    assert rdv.device_status() == 0


def test_f4x4_errors_and_empty(rdv, cuda_device):
    import rdv_project_b200._native as N
    lib = N.lib()
    assert lib.rdvb_winograd_packed_bytes(N.RDVB_WINOGRAD_F4X4, 24, 40) == 36 * 24 * 40 * 4
    assert lib.rdvb_winograd_packed_bytes(N.RDVB_WINOGRAD_F4X4, 129, 16) == 0
    dummy = torch.zeros(1 << 16, device=cuda_device)
    before = N.launch_count()
    N.check(lib.rdvb_conv3x3_winograd(dummy.data_ptr(), N.RDVB_F32, 0, 8, 8, 16, 16, dummy.data_ptr(),
                                      N.RDVB_WINOGRAD_F4X4, None, dummy.data_ptr(), N.RDVB_F32, None), "empty")
    assert N.launch_count() == before
    rc = lib.rdvb_conv3x3_winograd(dummy.data_ptr(), N.RDVB_F32, 1, 8, 8, 200, 16, dummy.data_ptr(),
                                   N.RDVB_WINOGRAD_F4X4, None, dummy.data_ptr(), N.RDVB_F32, None)
    assert rc == -2 and "F4X4" in N.last_error()
    rc = lib.rdvb_conv3x3_winograd(dummy.data_ptr() + 2, N.RDVB_F32, 1, 8, 8, 16, 16, dummy.data_ptr(),
                                   N.RDVB_WINOGRAD_F4X4, None, dummy.data_ptr(), N.RDVB_F32, None)
    assert rc == -1 and "aligned" in N.last_error()
    with pytest.raises(ValueError, match="variant"):
        rdv.Conv3x3Winograd(torch.zeros(3, 3, 16, 16), variant="F6x6")
