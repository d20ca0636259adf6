"""B200-native implementation of Rendervous's data-parallel hot path.

Drop-in for the reference's (rdv) operator API on this path::

    import rdv_project_b200 as rdv
    mlp = rdv.linear(W1, b1, f16=True) >> rdv.relu >> rdv.linear(W2, b2, f16=True)
    y = mlp(rdv.wrap(x)).as_tensor('torch')

Every operator launches hand-written sm_100a kernels from the in-tree
``_lib/librdvb.so`` (C ABI in ``include/rdvb.h``); there is no CPU fallback.
"""
from .core import (RDVObject, wrap, profiling, reset_submit_times, profiling_submit_times)
from .maps import (Map, Identity, X, ReLU, relu, Linear, LinearFast, LinearFastBF16, linear, Composite, TensorSampler,
                   GridSampler, Constant, XRProject, dir2xr)
from .tensor_ops import (TensorOperation, ReLUTensorOp, LinearTensorOp, LinearTensorOpFast, LinearTensorOpMine,
                         LinearTensorOpSimple, LinearTensorOpSmall, Downsample2xTensorOp, Upsample2xTensorOp,
                         ConcatTensorOp)
from .conv import (Conv2DTensorOp, Conv2DTensorOpFast, Conv2DTensorOpSimple, Conv2DTensorOpSimple3x3,
                   Conv2DTensorOpWindow3x3, Conv2DTensorOpWinograd3x3, Conv3x3Winograd, conv2d_direct,
                   _winograd_transform_weight)
from .rendering import Cameras, VolumeRenderer
from .volumes import (RaymarchingTransmittance, RatiotrackingTransmittance, TensorGrid, VoxelMajorantField,
                      SphereMajorantField, PBVR, PBVRT, PBVR_NEE, PBVR_ENV, XREnvironmentSampler)
from ._native import RdvbError, device_status

__all__ = [
    "RDVObject", "wrap", "profiling", "reset_submit_times", "profiling_submit_times",
    "Map", "Identity", "X", "ReLU", "relu", "Linear", "LinearFast", "LinearFastBF16", "linear", "Composite",
    "TensorSampler", "GridSampler", "Constant", "XRProject", "dir2xr",
    "TensorOperation", "ReLUTensorOp", "LinearTensorOp", "LinearTensorOpFast", "LinearTensorOpMine",
    "LinearTensorOpSimple", "LinearTensorOpSmall", "Downsample2xTensorOp", "Upsample2xTensorOp", "ConcatTensorOp",
    "Conv2DTensorOp", "Conv2DTensorOpFast", "Conv2DTensorOpSimple", "Conv2DTensorOpSimple3x3",
    "Conv2DTensorOpWindow3x3", "Conv2DTensorOpWinograd3x3", "Conv3x3Winograd", "conv2d_direct",
    "Cameras", "VolumeRenderer", "RaymarchingTransmittance", "RatiotrackingTransmittance", "TensorGrid",
    "VoxelMajorantField", "SphereMajorantField", "PBVR", "PBVRT", "PBVR_NEE", "PBVR_ENV", "XREnvironmentSampler",
    "RdvbError", "device_status",
]
