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
                     "rdvb_raymarch_render", "rdvb_camera_rays", "rdvb_camera_rays_jittered", "rdvb_last_error",
                     "rdvb_device_status"]:
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
    rc = lib.rdvb_conv3x3_winograd(None, N.RDVB_F16, 1, 8, 8, 200, 64, None, N.RDVB_WINOGRAD_F4X4, None, None,
                                   N.RDVB_F32, None)
    assert rc == -2 and "F4X4" in N.last_error()
    rc = lib.rdvb_conv3x3_winograd(None, N.RDVB_F16, 1, 8, 8, 24, 40, None, N.RDVB_WINOGRAD_F4X4, None, None,
                                   N.RDVB_F32, None)
    assert rc == -1 and "NULL" in N.last_error()
    assert lib.rdvb_winograd_packed_bytes(N.RDVB_WINOGRAD_F4X4, 24, 40) == 36 * 24 * 40 * 4
    assert lib.rdvb_winograd_packed_bytes(N.RDVB_WINOGRAD_F4X4, 0, 40) == 0
    rc = lib.rdvb_raymarch_render(N.float_array([3, 0.5, 0, 0, 0, 0, 0, 1, 0]), 8, 8, 0.0, 0.0, 64, 3,
                                  N.int_array([3, 64, 64, 4]), N.int_array([5, 5, 1]), None, 0, 8, None, 0, None,
                                  None)
    assert rc == -2 and "n_samples" in N.last_error()


def test_ratio_tracking_validation_before_any_device_work(lib):
    import rdv_project_b200._native as N

    dims, flags = N.int_array([3, 16, 1]), N.int_array([1, 1])
    seeds = N.uint32_array([1, 2, 3, 4])
    vox = N.RDVB_MAJORANT_VOXEL
    rc = lib.rdvb_transmittance_rt(None, 4, None, 1.0, None, N.int_array([2, 2, 0]), vox, seeds, 0, None, 2, dims, None,
                                   None, flags, 0, None, 256, None, None)
    assert rc == -1 and "weights" in N.last_error()
    w = N.ptr_array([1, 1])
    rc = lib.rdvb_transmittance_rt(None, 4, None, 1.0, None, N.int_array([2, 2, 0]), vox, seeds, 0, None, 2, dims, w, w,
                                   flags, 0, None, 256, None, None)
    assert rc == -1 and "majorant_dims" in N.last_error()
    rc = lib.rdvb_transmittance_rt(None, 4, None, 1.0, None, N.int_array([2, 2, 2]), vox, None, 0, None, 2, dims, w, w,
                                   flags, 0, None, 256, None, None)
    assert rc == -1 and "seeds" in N.last_error()
    rc = lib.rdvb_transmittance_rt(None, 4, None, 1.0, None, N.int_array([2, 2, 2]), vox, seeds, 0, None, 2,
                                   N.int_array([3, 16, 2]), w, w, flags, 0, None, 256, None, None)
    assert rc == -1 and "3 -> 1" in N.last_error()
    rc = lib.rdvb_transmittance_rt(None, 4, None, 1.0, None, N.int_array([2, 2, 2]), vox, seeds, -1, None, 2, dims, w, w,
                                   flags, 0, None, 256, None, None)
    assert rc == -1 and "draws_before" in N.last_error()
    rc = lib.rdvb_transmittance_rt(None, 4, None, 1.0, None, N.int_array([2, 2, 2]), 7, seeds, 0, None, 2, dims, w, w,
                                   flags, 0, None, 256, None, None)
    assert rc == -1 and "majorant_kind" in N.last_error()
    # nothing to do: no device needed
    for kind in (N.RDVB_MAJORANT_VOXEL, N.RDVB_MAJORANT_SPHERE):
        assert lib.rdvb_transmittance_rt(None, 0, None, 1.0, None, N.int_array([2, 2, 2]), kind, seeds, 0, None, 2, dims,
                                         w, w, flags, 0, None, 256, None, None) == 0


def _pbvr(lib, N, *, n=4, kind=0, albedo=(1.0, 1.0, 1.0), g=0.0, max_bounces=4, env_kind=0, env_rgb=(1, 1, 1),
          env_dims=(4, 8), env_flags=0, seeds=(1, 2, 3, 4), dims=(3, 16, 1), w=(1, 1)):
    return lib.rdvb_pbvr(None, n, None, None, N.int_array([2, 2, 2]), kind,
                         N.float_array(albedo) if albedo is not None else None, g, max_bounces, env_kind,
                         N.float_array(env_rgb) if env_rgb is not None else None, None,
                         N.int_array(env_dims) if env_dims is not None else None, env_flags,
                         N.uint32_array(seeds) if seeds is not None else None, 0, None, len(dims) - 1,
                         N.int_array(dims), N.ptr_array(w), N.ptr_array(w), N.int_array([1] * (len(dims) - 1)), 0,
                         None, 256, None, None)


def test_pbvr_validation_before_any_device_work(lib):
    """rdvb_pbvr checks its arguments on the host, before any device work;
    a call without rays succeeds without a device."""
    import rdv_project_b200._native as N

    assert _pbvr(lib, N, n=0) == 0
    assert _pbvr(lib, N, n=0, kind=N.RDVB_MAJORANT_SPHERE, env_kind=N.RDVB_ENV_EQUIRECT, env_rgb=None) == 0
    cases = [
        (dict(kind=3), "majorant_kind"),
        (dict(seeds=None), "seeds"),
        (dict(dims=(3, 16, 3)), "3 -> 1"),
        (dict(albedo=None, n=0), "albedo"),
        (dict(max_bounces=-1, n=0), "max_bounces"),
        (dict(g=float("nan"), n=0), "g must be finite"),
        (dict(env_kind=5, n=0), "env_kind"),
        (dict(env_rgb=None, n=0), "env_rgb"),
        (dict(env_kind=N.RDVB_ENV_EQUIRECT, env_dims=None, n=0), "env_dims"),
        (dict(env_kind=N.RDVB_ENV_EQUIRECT, env_dims=(0, 8), n=0), "env_dims"),
        (dict(env_kind=N.RDVB_ENV_EQUIRECT, env_flags=8, n=0), "env_flags"),
        (dict(env_kind=N.RDVB_ENV_EQUIRECT), "rays, majorant and out"),
    ]
    for kw, msg in cases:
        rc = _pbvr(lib, N, **kw)
        assert rc == -1 and msg in N.last_error(), (kw, rc, N.last_error())
    assert lib.rdvb_xr_project(None, 0, None, None) == 0
    assert lib.rdvb_xr_project(None, -1, None, None) == -1
    assert lib.rdvb_xr_project(None, 3, None, None) == -1 and "aligned" in N.last_error()


def test_volume_nodes_host_side():
    """Argument handling of the volume nodes that needs no device: seeds as
    the reference draws them, majorant wrapping, TensorGrid shapes."""
    import torch

    import rdv_project_b200 as rdv
    from rdv_project_b200 import volumes

    for _ in range(50):
        s = volumes._draw_seeds()
        assert len(s) == 4 and all(128 <= v < (1 << 30) for v in s)
    g = rdv.TensorGrid(torch.ones(4, 5, 6, 1))
    assert (g.IN, g.OUT, g.shape) == (3, 1, [4, 5, 6])
    f = volumes._as_majorant_field(torch.ones(2, 2, 2, 1))
    assert isinstance(f, rdv.VoxelMajorantField) and f.grid.shape == [2, 2, 2]
    assert volumes._as_majorant_field(f) is f
    with pytest.raises(AssertionError, match="Grid\\[3, 1\\]"):
        rdv.VoxelMajorantField(torch.ones(4, 4, 2))
    with pytest.raises(NotImplementedError):
        volumes._as_majorant_field(3.0)
    ext = rdv.linear(torch.randn(1, 3), torch.zeros(1))
    node = rdv.RatiotrackingTransmittance(ext, torch.ones(1, 1, 1, 1), density_scale=2.0)
    assert node.IN == 6 and node.OUT == 1 and node.density_scale == 2.0
    assert not hasattr(node, "step_size")


def test_forward_path_reasons_without_a_device(lib):
    """rdvb_mlp_forward_path names why a chain would run on the CUDA cores;
    every case here is decided from the arguments alone."""
    import rdv_project_b200._native as N

    dims = N.int_array([3, 64, 64, 4])
    f16 = N.int_array([N.RDVB_MATH_F16 | N.RDVB_LAYER_RELU] * 2 + [N.RDVB_MATH_F16])
    good_x, good_p, good_y = 0x10000, 0x20000, 0x30000

    def path(x, flags, packed, y, d=dims, n=3, rows=4096):
        return lib.rdvb_mlp_forward_path(x, N.RDVB_F32, rows, n, d, flags, packed, y)

    assert path(good_x, N.int_array([0, 0, 0]), good_p, good_y) == N.RDVB_PATH_CUDA_CORE
    assert "fp32" in N.last_error()
    mixed = N.int_array([N.RDVB_MATH_F16, N.RDVB_MATH_BF16, N.RDVB_MATH_F16])
    assert path(good_x, mixed, good_p, good_y) == N.RDVB_PATH_CUDA_CORE and "mixes" in N.last_error()
    assert path(good_x, f16, None, good_y) == N.RDVB_PATH_CUDA_CORE and "packed" in N.last_error()
    assert path(good_x, f16, good_p + 16, good_y) == N.RDVB_PATH_CUDA_CORE and "256-byte" in N.last_error()
    # x[1:] of a 3-wide fp32 tensor: 12 bytes past an aligned base
    assert path(good_x + 12, f16, good_p, good_y) == N.RDVB_PATH_CUDA_CORE
    assert "x is not 16-byte aligned" in N.last_error()
    assert path(good_x, f16, good_p, good_y + 2) == N.RDVB_PATH_CUDA_CORE and "y is not" in N.last_error()
    wide = N.int_array([3, 200, 4])
    assert path(good_x, f16, good_p, good_y, d=wide, n=2) == N.RDVB_PATH_CUDA_CORE
    assert "width above 128" in N.last_error()
    assert path(good_x, f16, good_p, good_y, rows=31) == N.RDVB_PATH_CUDA_CORE and "32 rows" in N.last_error()
    assert lib.rdvb_mlp_forward_path(good_x, 9, 4096, 3, dims, f16, good_p, good_y) == N.RDVB_ERR_INVALID_ARG


def test_max_ctas_setting(lib):
    import rdv_project_b200._native as N

    assert lib.rdvb_get_max_ctas() == 0
    assert N.set_max_ctas(100) == 0
    assert lib.rdvb_get_max_ctas() == 100
    assert N.set_max_ctas(0) == 100
    assert lib.rdvb_set_max_ctas(-1) == N.RDVB_ERR_INVALID_ARG and "max_ctas" in N.last_error()
    assert lib.rdvb_get_max_ctas() == 0


def test_grid_sampler_validation(lib):
    import rdv_project_b200._native as N

    shape = N.int_array([4, 4, 4, 4, 4])
    assert lib.rdvb_grid_sampler(None, 3, shape, 2, None, 0, 1, 0, 1, None, None) == 0
    assert lib.rdvb_grid_sampler(None, 5, shape, 2, None, 4, 1, 0, 1, None, None) == -2
    assert "in_dim" in N.last_error()
    assert lib.rdvb_grid_sampler(None, 3, N.int_array([4, 0, 4]), 2, None, 4, 1, 0, 1, None, None) == -1
    assert lib.rdvb_grid_sampler(None, 3, shape, 0, None, 4, 1, 0, 1, None, None) == -1
    assert lib.rdvb_grid_sampler(None, 3, shape, 2, None, 4, 1, 0, 1, None, None) == -1
    assert "must not be NULL" in N.last_error()


def test_pbvrt_validation(lib):
    import rdv_project_b200._native as N

    def call(n=0, variant=0, albedo=(1, 1, 1), light=(0, 1, 0), intensity=(1, 1, 1), g=0.0, mb=4, scale=1.0):
        return lib.rdvb_pbvrt(None, n, None, scale, None, N.int_array([2, 2, 2]), 0,
                              N.float_array(albedo) if albedo else None, g, mb,
                              N.float_array(light) if light else None, N.float_array(intensity) if intensity else None,
                              variant, 0, N.float_array([1, 1, 1]), None, N.int_array([1, 1]), 0,
                              None, 0, N.uint32_array([1, 2, 3, 4]), 0, None, 2, N.int_array([3, 16, 1]), N.ptr_array([1, 1]),
                              N.ptr_array([1, 1]), N.int_array([1, 1]), 0, None, 256, None, None)

    assert call() == 0
    assert call(variant=N.RDVB_PBVR_NEE, intensity=None) == 0     # NEE reads no light intensity
    for kw, msg in ((dict(variant=3), "variant"), (dict(albedo=None), "albedo"), (dict(light=None), "light"),
                    (dict(intensity=None), "light_intensity"), (dict(mb=-1), "max_bounces"),
                    (dict(scale=float("inf")), "finite"), (dict(light=(0, 0, 0)), "nonzero")):
        assert call(**kw) == -1 and msg in N.last_error(), (kw, N.last_error())


def test_extinction_encoding_validation(lib):
    """A sampler in front of a volume node's chain (rdvb_encoding): checked
    on the host; with it the chain maps features -> 1, or is empty."""
    import ctypes
    import rdv_project_b200._native as N

    def rm(enc, n_layers, dims, n=0):
        return lib.rdvb_transmittance_rm(None, n, None, 0.01, 1.0, ctypes.byref(enc) if enc is not None else None,
                                         n_layers, N.int_array(dims), N.ptr_array([1] * max(n_layers, 1)),
                                         N.ptr_array([1] * max(n_layers, 1)), N.int_array([1] * max(n_layers, 1)), 0,
                                         None, 256, None, None)

    e = N.Encoding()
    e.kind, e.grid, e.features, e.flags = N.RDVB_ENCODING_GRID_SAMPLER, 256, 4, N.RDVB_SAMPLER_LINEAR
    for k in range(3):
        e.dims[k] = 8
    assert rm(e, 1, [4, 1]) == 0              # sampler (4 features) >> Linear 4 -> 1
    assert rm(e, 0, [4]) == -1 and "4 -> 1" in N.last_error()
    e.features = 1
    assert rm(e, 0, [1]) == 0                 # the sampled density is the extinction
    assert rm(None, 0, [3]) == -1 and "n_layers" in N.last_error()
    e.kind = 9
    assert rm(e, 0, [1]) == -1 and "encoding kind" in N.last_error()
    e.kind, e.dims[1] = N.RDVB_ENCODING_TENSOR_SAMPLER, 0
    assert rm(e, 0, [1]) == -1 and "encoding dims" in N.last_error()
    e.dims[1], e.flags = 8, 16
    assert rm(e, 0, [1]) == -1 and "flag" in N.last_error()


def test_pbvr_env_validation(lib):
    import rdv_project_b200._native as N

    def call(levels=4, dens=None, n=0):
        return lib.rdvb_pbvrt(None, n, None, 1.0, None, N.int_array([2, 2, 2]), 0, N.float_array([1, 1, 1]), 0.0, 4,
                              None, None, N.RDVB_PBVR_ENV, 0, N.float_array([1, 1, 1]), None, N.int_array([1, 1]), 0,
                              dens, levels, N.uint32_array([1, 2, 3, 4]), 0, None, 2, N.int_array([3, 16, 1]),
                              N.ptr_array([1, 1]), N.ptr_array([1, 1]), N.int_array([1, 1]), 0, None, 256, None, None)

    assert call() == 0                                      # no light direction or intensity needed
    assert call(levels=0) == -1 and "env_levels" in N.last_error()
    assert call(levels=13) == -1 and "env_levels" in N.last_error()


def test_peer_copy_and_ipc_validation(lib):
    """The peer copy and the IPC helpers check their arguments before
    touching a device."""
    import ctypes

    import rdv_project_b200._native as N

    rc = lib.rdvb_peer_copy(None, None, 9, 16, None)
    assert rc == -1 and "n_dst" in N.last_error()
    rc = lib.rdvb_peer_copy(None, None, 1, -1, None)
    assert rc == -1 and "bytes" in N.last_error()
    rc = lib.rdvb_peer_copy(None, N.ptr_array([0]), 1, 16, None)
    assert rc == -1 and "NULL" in N.last_error()
    assert lib.rdvb_peer_copy(None, None, 0, 16, None) == 0  # nothing to copy
    ptr = ctypes.c_void_p()
    assert lib.rdvb_ipc_alloc(0, ctypes.byref(ptr), None) == -1
    assert lib.rdvb_ipc_open(None, ctypes.byref(ptr)) == -1
    assert lib.rdvb_ipc_free(None) == 0 and lib.rdvb_ipc_close(None) == 0
    assert N.RDVB_IPC_HANDLE_BYTES == 64 and N.RDVB_MAX_PEERS == 7


def test_multicast_copy_validation(lib):
    import rdv_project_b200._native as N

    rc = lib.rdvb_multicast_copy(None, 0, 24, 16, None)
    assert rc == -1 and "multiple of 16" in N.last_error()
    rc = lib.rdvb_multicast_copy(None, 0, 32, 16, None)
    assert rc == -1 and "NULL" in N.last_error()
    assert lib.rdvb_multicast_copy(None, 0, 0, 16, None) == 0
