"""The C ABI on CPU: librdvb.so loads and exports every function that
include/rdvb.h declares, and the entry points that need no device (sizes,
version, argument validation) behave as declared. No kernel is launched."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    from rdv_project_b200.csrc import build as b

    b.build()  # compiles in-tree when missing or stale (nvcc cross-compiles, no GPU needed)
    import rdv_project_b200._native as N

    return N.lib()


def declared_functions():
    text = open(os.path.join(ROOT, "include", "rdvb.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rdvb_\w+)\s*\(", text)))


def test_header_declares_the_path(lib):
    names = declared_functions()
    for required in ["rdvb_mlp_forward", "rdvb_mlp_pack", "rdvb_conv3x3_winograd", "rdvb_winograd_filter_transform",
                     "rdvb_raymarch_render", "rdvb_camera_rays", "rdvb_last_error", "rdvb_device_status"]:
        assert required in names


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    import rdv_project_b200._native as N

    # the Python binding types every exported entry point
    assert set(N.SIGNATURES) >= set(declared_functions())


def test_host_only_entry_points(lib):
    import rdv_project_b200._native as N

    assert lib.rdvb_version() >= 100
    assert lib.rdvb_launch_count() >= 0
    # packed-weight size: per layer n_pad * ceil(k_pad/64) * 128 bytes (1 KB aligned), then fp32 biases
    dims = N.int_array([32] + [128] * 8 + [16])
    size = lib.rdvb_mlp_packed_bytes(9, dims)
    expect_w = 128 * 1 * 128 + 7 * 128 * 2 * 128 + 16 * 2 * 128
    assert size == expect_w + (128 * 8 + 16) * 4
    assert lib.rdvb_mlp_packed_bytes(1, N.int_array([300, 4])) == 0  # too wide for the tensor-core kernel
    assert lib.rdvb_winograd_packed_bytes(N.RDVB_WINOGRAD_F2X2, 64, 64) == 16 * 64 * 128
    assert lib.rdvb_winograd_packed_bytes(N.RDVB_WINOGRAD_F2X2, 48, 80) == 0
    assert lib.rdvb_raymarch_workspace_bytes(1920, 1080) == 256 + 1920 * 1080 * 4


def test_validation_before_any_device_work(lib):
    import rdv_project_b200._native as N

    rc = lib.rdvb_mlp_forward(None, N.RDVB_F32, 16, 0, N.int_array([3, 4]), None, None, N.int_array([0]), 0, 0,
                              None, None, None)
    assert rc == -1 and "n_layers" in N.last_error()
    rc = lib.rdvb_mlp_forward(None, 7, 16, 1, N.int_array([3, 4]), None, None, N.int_array([0]), 0, 0, None, None,
                              None)
    assert rc == -1 and "x_dtype" in N.last_error()
    rc = lib.rdvb_conv3x3_winograd(None, N.RDVB_F16, 1, 8, 8, 64, 64, None, N.RDVB_WINOGRAD_F4X4, None, None,
                                   N.RDVB_F32, None)
    assert rc == -2 and "F4X4" in N.last_error()
    rc = lib.rdvb_raymarch_render(N.float_array([3, 0.5, 0, 0, 0, 0, 0, 1, 0]), 8, 8, 0.0, 0.0, 64, 3,
                                  N.int_array([3, 64, 64, 4]), N.int_array([5, 5, 1]), None, 0, 8, None, 0, None,
                                  None)
    assert rc == -2 and "n_samples" in N.last_error()
