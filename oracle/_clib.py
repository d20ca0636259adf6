"""ctypes loaders for the oracle's C libraries (test infrastructure only)."""
from __future__ import annotations

import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_shaders.so")
REF_COOPMAT_LIB = os.path.join(HERE, "_ref", "libref_coopmat.so")
REF_PBVR_LIB = os.path.join(HERE, "_ref", "libref_pbvr.so")
REF_SAMPLERS_LIB = os.path.join(HERE, "_ref", "libref_samplers.so")
# The reference checkout: $RDV_REFERENCE_ROOT, else a checkout named
# `reference` beside this repository.
REFERENCE_ROOT = os.environ.get("RDV_REFERENCE_ROOT") or os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                                      "reference")

_oracle = None
_ref = None
_ref_cm = None
_ref_pbvr = None
_ref_samplers = None


def build_oracle(verbose: bool = False) -> None:
    """make -C oracle (C restatement) and, when the reference checkout is
    present, make -C oracle ref (reference shader functions)."""
    out = None if verbose else subprocess.DEVNULL
    subprocess.check_call(["make", "-s", "-C", HERE], stdout=out)
    if os.path.isdir(os.path.join(REFERENCE_ROOT, "src", "rdv", "shaders")):
        subprocess.check_call(["make", "-s", "-C", HERE, "ref", f"REF={REFERENCE_ROOT}"], stdout=out)


def oracle_lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_LIB):
            build_oracle()
        lib = ctypes.CDLL(ORACLE_LIB)
        lib.oracle_mlp_forward.restype = None
        lib.oracle_mlp_forward.argtypes = [
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
        ]
        lib.oracle_round.restype = None
        lib.oracle_round.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
        _oracle = lib
    return _oracle


def ref_lib_available() -> bool:
    if os.path.exists(REF_LIB):
        return True
    if os.path.isdir(os.path.join(REFERENCE_ROOT, "src", "rdv", "shaders")):
        try:
            build_oracle()
        except (OSError, subprocess.CalledProcessError):
            return False
        return os.path.exists(REF_LIB)
    return False


def ref_lib() -> ctypes.CDLL:
    """The reference's own scalar shader functions (see ref_shim/)."""
    global _ref
    if _ref is None:
        if not ref_lib_available():
            raise FileNotFoundError(
                f"{REF_LIB} is missing and the reference checkout is not present to build it")
        lib = ctypes.CDLL(REF_LIB)
        vp, lg, i32, f32 = ctypes.c_void_p, ctypes.c_long, ctypes.c_int, ctypes.c_float
        lib.ref_mlp_c1.argtypes = [vp, lg, vp, vp, vp]
        lib.ref_mlp_small.argtypes = [vp, lg, vp, vp, vp]
        lib.ref_linear_tensor_op_16_24.argtypes = [vp, i32, vp, vp, vp]
        lib.ref_relu_tensor_op.argtypes = [vp, i32, i32, vp]
        lib.ref_conv2d_tensor_op_3x3_16_32_16x16.argtypes = [vp, vp, vp, vp]
        lib.ref_winograd_fwd.argtypes = [vp, vp]
        lib.ref_winograd_inv.argtypes = [vp, vp]
        lib.ref_transmittance_rm.argtypes = [f32, f32, vp, vp, f32, f32, f32]
        lib.ref_transmittance_rm.restype = f32
        lib.ref_random_sequence.argtypes = [vp, i32, i32, vp]
        lib.ref_random_sequence.restype = None
        lib.ref_transmittance_rt.argtypes = [f32, f32, vp, i32, i32, i32, vp, i32, vp, vp, f32, f32]
        lib.ref_transmittance_rt.restype = f32
        lib.ref_downsample2x.argtypes = [vp, i32, i32, i32, vp]
        lib.ref_upsample2x.argtypes = [vp, i32, i32, i32, vp]
        lib.ref_concat.argtypes = [vp, i32, vp, i32, i32, vp]
        for name in ("ref_mlp_c1", "ref_mlp_small", "ref_linear_tensor_op_16_24", "ref_relu_tensor_op",
                     "ref_conv2d_tensor_op_3x3_16_32_16x16", "ref_winograd_fwd", "ref_winograd_inv",
                     "ref_downsample2x", "ref_upsample2x", "ref_concat"):
            getattr(lib, name).restype = None
        _ref = lib
    return _ref


def ref_coopmat_lib() -> ctypes.CDLL:
    """The reference's cooperative-matrix (float16) code paths executed on
    the CPU (ref_shim/ref_coopmat.cpp)."""
    global _ref_cm
    if _ref_cm is None:
        if not os.path.exists(REF_COOPMAT_LIB) and not ref_lib_available():
            raise FileNotFoundError(
                f"{REF_COOPMAT_LIB} is missing and the reference checkout is not present to build it")
        lib = ctypes.CDLL(REF_COOPMAT_LIB)
        vp, lg, i32 = ctypes.c_void_p, ctypes.c_long, ctypes.c_int
        for name in ("ref_cm_mlp_c5", "ref_cm_mlp_c2"):
            getattr(lib, name).argtypes = [vp, lg, vp, vp, vp]
        for name in ("ref_cm_small_32_48", "ref_cm_small_64_32", "ref_cm_simple_32_64", "ref_cm_fast_32_64",
                     "ref_cm_mine_32_48"):
            getattr(lib, name).argtypes = [vp, i32, vp, vp, vp]
        for name in ("ref_cm_winograd_16", "ref_cm_winograd_48"):
            getattr(lib, name).argtypes = [vp, vp, vp, vp]
        for name in ("ref_cm_mlp_c5", "ref_cm_mlp_c2", "ref_cm_small_32_48", "ref_cm_small_64_32",
                     "ref_cm_simple_32_64", "ref_cm_fast_32_64", "ref_cm_mine_32_48", "ref_cm_winograd_16",
                     "ref_cm_winograd_48"):
            getattr(lib, name).restype = None
        _ref_cm = lib
    return _ref_cm


def ref_pbvr_lib() -> ctypes.CDLL:
    """The reference's PBVR body and Henyey-Greenstein sampler compiled as
    C++ (ref_shim/ref_pbvr.cpp)."""
    global _ref_pbvr
    if _ref_pbvr is None:
        if not os.path.exists(REF_PBVR_LIB) and not ref_lib_available():
            raise FileNotFoundError(
                f"{REF_PBVR_LIB} is missing and the reference checkout is not present to build it")
        lib = ctypes.CDLL(REF_PBVR_LIB)
        vp, lg, i32, f32 = ctypes.c_void_p, ctypes.c_long, ctypes.c_int, ctypes.c_float
        lib.ref_pbvr.argtypes = [f32, f32, i32, vp, i32, i32, i32, vp, vp, vp, f32, i32, vp, vp, lg, vp]
        lib.ref_pbvr.restype = None
        lib.ref_pbvrt.argtypes = [i32, f32, f32, i32, vp, i32, i32, i32, vp, vp, vp, vp, vp, f32, f32, i32, vp, vp,
                                  lg, vp]
        lib.ref_pbvrt.restype = None
        lib.ref_pbvr_env.argtypes = [f32, f32, i32, vp, i32, i32, i32, vp, vp, vp, vp, i32, f32, f32, i32, vp, vp,
                                     lg, vp]
        lib.ref_pbvr_env.restype = None
        lib.ref_hg_phase_sample.argtypes = [vp, i32, i32, vp, f32, vp]
        lib.ref_hg_phase_sample.restype = None
        _ref_pbvr = lib
    return _ref_pbvr


def ref_samplers_lib() -> ctypes.CDLL:
    """The reference's GridSampler body compiled as C++
    (ref_shim/ref_samplers.cpp)."""
    global _ref_samplers
    if _ref_samplers is None:
        if not os.path.exists(REF_SAMPLERS_LIB) and not ref_lib_available():
            raise FileNotFoundError(
                f"{REF_SAMPLERS_LIB} is missing and the reference checkout is not present to build it")
        lib = ctypes.CDLL(REF_SAMPLERS_LIB)
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        lib.ref_grid_sampler.argtypes = [i32, i32, vp, vp, i32, i32, i32, vp, ctypes.c_long, vp]
        lib.ref_grid_sampler.restype = i32
        _ref_samplers = lib
    return _ref_samplers


def ptr(a) -> int:
    """Address of a C-contiguous numpy array."""
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def ptr_array(arrays) -> ctypes.Array:
    arr = (ctypes.c_void_p * len(arrays))()
    for i, a in enumerate(arrays):
        arr[i] = ptr(a)
    return arr
