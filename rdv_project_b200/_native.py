"""ctypes binding of librdvb.so (the C ABI declared in include/rdvb.h).

The library is built in-tree by ``rdv_project_b200.csrc.build`` (or
``__graft_entry__.build()``). There is no fallback: if the library is missing
or cannot be loaded every operator raises, so a CUDA-less or unbuilt
environment can never silently compute something else.
"""
from __future__ import annotations

import ctypes
import os
import threading

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "librdvb.so")
_lib = None
_lock = threading.Lock()

RDVB_OK = 0
RDVB_F32, RDVB_F16, RDVB_BF16 = 0, 1, 2
RDVB_MATH_F32, RDVB_MATH_F16, RDVB_MATH_BF16 = 0, 1, 2
RDVB_LAYER_RELU = 4
RDVB_WINOGRAD_F2X2, RDVB_WINOGRAD_F4X4 = 0, 1
RDVB_PATH_CUDA_CORE, RDVB_PATH_TENSOR_CORE = 0, 1
RDVB_MAJORANT_VOXEL, RDVB_MAJORANT_SPHERE = 0, 1
RDVB_ENV_CONSTANT, RDVB_ENV_EQUIRECT = 0, 1
RDVB_SAMPLER_CLAMP, RDVB_SAMPLER_ALIGNED, RDVB_SAMPLER_LINEAR = 1, 2, 4
RDVB_PBVRT, RDVB_PBVR_NEE, RDVB_PBVR_ENV = 0, 1, 2
RDVB_ENCODING_TENSOR_SAMPLER, RDVB_ENCODING_GRID_SAMPLER = 1, 2
RDVB_IPC_HANDLE_BYTES = 64
RDVB_MAX_PEERS = 7

_c_int, _c_i64, _vp, _c_u32, _c_f = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float

# name -> (restype, argtypes); the exported surface of include/rdvb.h
SIGNATURES = {
    "rdvb_version": (_c_int, []),
    "rdvb_launch_count": (_c_i64, []),
    "rdvb_last_error": (ctypes.c_char_p, []),
    "rdvb_device_status": (_c_int, [_c_int, ctypes.POINTER(_c_u32)]),
    "rdvb_mlp_packed_bytes": (_c_i64, [_c_int, _vp]),
    "rdvb_mlp_pack": (_c_int, [_c_int, _vp, _vp, _vp, _c_int, _vp, _vp]),
    "rdvb_mlp_forward": (_c_int, [_vp, _c_int, _c_i64, _c_int, _vp, _vp, _vp, _vp, _c_int, _c_int, _vp, _vp, _vp]),
    "rdvb_peer_copy": (_c_int, [_vp, _vp, _c_int, _c_i64, _vp]),
    "rdvb_multicast_copy": (_c_int, [_vp, ctypes.c_uint64, _c_i64, _c_int, _vp]),
    "rdvb_ipc_alloc": (_c_int, [_c_i64, ctypes.POINTER(_vp), _vp]),
    "rdvb_ipc_free": (_c_int, [_vp]),
    "rdvb_ipc_open": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "rdvb_ipc_close": (_c_int, [_vp]),
    "rdvb_mlp_static_capacity": (_c_i64, []),
    "rdvb_mlp_forward_static": (_c_int, [_vp, _c_int, _c_i64, _c_int, _vp, _vp, _vp, _vp, _c_int, _c_int, _vp, _vp]),
    "rdvb_mlp_forward_path": (_c_int, [_vp, _c_int, _c_i64, _c_int, _vp, _vp, _vp, _vp]),
    "rdvb_set_max_ctas": (_c_int, [_c_int]),
    "rdvb_get_max_ctas": (_c_int, []),
    "rdvb_relu": (_c_int, [_vp, _vp, _c_i64, _vp]),
    "rdvb_winograd_packed_bytes": (_c_i64, [_c_int, _c_int, _c_int]),
    "rdvb_winograd_filter_transform": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _vp]),
    "rdvb_conv3x3_winograd": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_int, _vp, _vp,
                                       _c_int, _vp]),
    "rdvb_conv2d_direct": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _vp,
                                    _vp, _vp]),
    "rdvb_conv2d_direct_staged": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                           _vp, _vp, _c_int, _c_int, _vp, _vp]),
    "rdvb_conv_tc_packed_bytes": (_c_i64, [_c_int, _c_int, _c_int, _c_int]),
    "rdvb_conv_tc_pack": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _vp]),
    "rdvb_conv2d_tc": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_int,
                                _vp, _vp, _vp]),
    "rdvb_tensor_sampler": (_c_int, [_vp, _c_int, _vp, _c_int, _vp, _c_i64, _c_int, _c_int, _c_int, _vp, _vp]),
    "rdvb_downsample2x": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp]),
    "rdvb_upsample2x": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp]),
    "rdvb_concat_channels": (_c_int, [_vp, _c_int, _vp, _c_int, _c_i64, _vp, _vp]),
    "rdvb_camera_rays": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_f, _c_f, _vp, _vp]),
    "rdvb_camera_rays_jittered": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_f, _c_f, _vp, _vp, _vp]),
    "rdvb_raymarch_workspace_bytes": (_c_i64, [_c_int, _c_int]),
    "rdvb_raymarch_render": (_c_int, [_vp, _c_int, _c_int, _c_f, _c_f, _c_int, _c_int, _vp, _vp, _vp, _c_int, _c_int,
                                      _vp, ctypes.c_size_t, _vp, _vp]),
    "rdvb_transmittance_workspace_bytes": (_c_i64, [_c_i64, _c_int, _vp, _vp]),
    "rdvb_transmittance_rm": (_c_int, [_vp, _c_i64, _vp, _c_f, _c_f, _vp, _c_int, _vp, _vp, _vp, _vp, _c_int, _vp,
                                       ctypes.c_size_t, _vp, _vp]),
    "rdvb_transmittance_rt": (_c_int, [_vp, _c_i64, _vp, _c_f, _vp, _vp, _c_int, _vp, _c_int, _vp, _c_int, _vp, _vp,
                                       _vp, _vp, _c_int, _vp, ctypes.c_size_t, _vp, _vp]),
    "rdvb_xr_project": (_c_int, [_vp, _c_i64, _vp, _vp]),
    "rdvb_pbvrt": (_c_int, [_vp, _c_i64, _vp, _c_f, _vp, _vp, _c_int, _vp, _c_f, _c_int, _vp, _vp, _c_int, _c_int,
                            _vp, _vp, _vp, _c_int, _vp, _c_int, _vp, _c_int, _vp, _c_int, _vp, _vp, _vp, _vp,
                            _c_int, _vp, ctypes.c_size_t, _vp, _vp]),
    "rdvb_grid_sampler": (_c_int, [_vp, _c_int, _vp, _c_int, _vp, _c_i64, _c_int, _c_int, _c_int, _vp, _vp]),
    "rdvb_pbvr": (_c_int, [_vp, _c_i64, _vp, _vp, _vp, _c_int, _vp, _c_f, _c_int, _c_int, _vp, _vp, _vp, _c_int,
                           _vp, _c_int, _vp, _c_int, _vp, _vp, _vp, _vp, _c_int, _vp, ctypes.c_size_t, _vp, _vp]),
}


class Encoding(ctypes.Structure):
    """rdvb_encoding: a sampler of a dense 3-D grid in front of a volume
    node's extinction chain."""
    _fields_ = [("kind", _c_int), ("grid", _vp), ("dims", _c_int * 3), ("features", _c_int), ("flags", _c_int)]


class RdvbError(RuntimeError):
    """A librdvb call returned an error status."""


def library_path() -> str:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(_LIB_PATH):
                    raise RdvbError(
                        f"{_LIB_PATH} is missing: build the CUDA extension first "
                        "(python -m rdv_project_b200.csrc.build, or __graft_entry__.build())")
                handle = ctypes.CDLL(_LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name, None)
                    if fn is None:
                        continue
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().rdvb_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc != RDVB_OK:
        raise RdvbError(f"{what} failed ({rc}): {last_error()}")


RDVB_ERR_INVALID_ARG, RDVB_ERR_UNSUPPORTED, RDVB_ERR_CUDA, RDVB_ERR_DEVICE_STATUS = -1, -2, -3, -4


def device_status(clear: bool = True) -> int:
    """Synchronizes the device and returns the bounded-wait status word
    (0 = healthy; bits name the wait that expired)."""
    v = _c_u32(0)
    rc = lib().rdvb_device_status(1 if clear else 0, ctypes.byref(v))
    if rc != RDVB_ERR_DEVICE_STATUS:
        check(rc, "rdvb_device_status")
    return int(v.value)


def launch_count() -> int:
    return int(lib().rdvb_launch_count())


def set_max_ctas(n: int) -> int:
    """Caps the persistent tensor-core MLP kernel at n CTAs (0 = one per SM)
    for later launches; returns the previous cap."""
    prev = int(lib().rdvb_get_max_ctas())
    check(lib().rdvb_set_max_ctas(int(n)), "rdvb_set_max_ctas")
    return prev


def int_array(values):
    arr = (_c_int * len(values))()
    for i, v in enumerate(values):
        arr[i] = int(v)
    return arr


def float_array(values):
    arr = (_c_f * len(values))()
    for i, v in enumerate(values):
        arr[i] = float(v)
    return arr


def uint32_array(values):
    arr = (_c_u32 * len(values))()
    for i, v in enumerate(values):
        arr[i] = int(v) & 0xFFFFFFFF
    return arr


def ptr_array(ptrs):
    arr = (_vp * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = int(p)
    return arr
