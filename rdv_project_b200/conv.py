"""3x3 convolution operators (the reference's conv TensorOperations,
rdv/domain/nn.py:414-469 and 1002-1087) and a batched NHWC Winograd
operator.

* ``Conv2DTensorOp(x, weight, bias, H, W)``: 'same', stride-1 KHxKW
  convolution in exact fp32 (CUDA cores) -> rdvb_conv2d_direct.
* ``Conv2DTensorOpFast`` / ``Conv2DTensorOpSimple`` / ``Conv2DTensorOpSimple3x3``
  / ``Conv2DTensorOpWindow3x3(x, weight, bias, H, W)`` (nn.py:608-999): the
  reference's tensor-core direct convolutions -- x and weight rounded to
  float16, fp32 accumulation, the bias seeding the accumulator (Simple*,
  Window3x3) or added after (Fast) -> rdvb_conv2d_direct_staged, with each
  op's own shape assertions.
* ``Conv2DTensorOpWinograd3x3(x, weight, bias, H, W)``: Winograd F(2x2,3x3)
  -> rdvb_winograd_filter_transform (once, at construction, like the
  reference's ``_winograd_transform_weight``) + rdvb_conv3x3_winograd.
  Same inputs, layouts and assertion messages as the reference, except
  that in/out channels may go up to 64 (reference: 48, a limit of its 48 KB
  shared-memory budget) and (H/2)*(W/2) need not be a multiple of 32 (the
  reference's workgroup size; the B200 kernel masks partial blocks).
* ``Conv3x3Winograd(weight, bias)``: the same kernel on batched NHWC
  tensors ``[N, H, W, CIN]`` (float32 or float16, any H/W), output float32
  or float16 -- the form the BASELINE config-3 workload uses.
* ``_winograd_transform_weight(weight, in_channels, out_channels)``: the
  reference's helper (nn.py:525-538), computed on the device; returns the
  flat float16 ``[16 * CIN * COUT]`` buffer.

Inputs of the TensorOperation forms are ``[H*W, channels]`` row-major
(channels-last, H*W flattened), weights ``[3, 3, CIN, COUT]``.
"""
from __future__ import annotations

import torch

from . import _native as N
from .core import RDVObject, _timed, current_device, stream_handle, wrap
from .tensor_ops import TensorOperation, _as_op_input, _f32_view, _max_subgroups

_DTYPES = {torch.float32: N.RDVB_F32, torch.float16: N.RDVB_F16}
MAX_WINOGRAD_CHANNELS = 64


def _dev_f32(t) -> torch.Tensor:
    t = t._tensor if isinstance(t, RDVObject) else torch.as_tensor(t)
    return t.to(device=current_device(), dtype=torch.float32).contiguous()


_VARIANTS = {"F2x2": (N.RDVB_WINOGRAD_F2X2, 16), "F4x4": (N.RDVB_WINOGRAD_F4X4, 36)}


def _variant(name: str) -> int:
    if name not in _VARIANTS:
        raise ValueError(f"Winograd variant must be one of {sorted(_VARIANTS)} (got {name!r})")
    return _VARIANTS[name][0]


def _filter_transform(w33io: torch.Tensor, cin: int, cout: int, plain: bool, packed: bool, variant: str = "F2x2"):
    lib = N.lib()
    code = _variant(variant)
    positions = _VARIANTS[variant][1]
    u_dtype = torch.float32 if variant == "F4x4" else torch.float16   # F(4x4) keeps U fp32
    u_plain = torch.empty(positions * cin * cout, dtype=u_dtype, device=w33io.device) if plain else None
    u_packed = None
    if packed:
        nbytes = lib.rdvb_winograd_packed_bytes(code, cin, cout)
        if nbytes <= 0:
            raise N.RdvbError(f"no packed Winograd {variant} operand for cin={cin}, cout={cout}")
        u_packed = torch.empty(int(nbytes), dtype=torch.uint8, device=w33io.device)
    N.check(lib.rdvb_winograd_filter_transform(
        w33io.data_ptr(), cin, cout, code,
        u_plain.data_ptr() if plain else None, u_packed.data_ptr() if packed else None, stream_handle()),
        "rdvb_winograd_filter_transform")
    return u_plain, u_packed


def _winograd_transform_weight(weight, in_channels: int, out_channels: int) -> torch.Tensor:
    """U = G g G^T of a [3, 3, CIN, COUT] weight, fp32 arithmetic, stored
    float16 as a flat [16][CIN][COUT] buffer (rdv/domain/nn.py:525-538)."""
    w = _dev_f32(weight)
    assert tuple(w.shape) == (3, 3, in_channels, out_channels), "weight must be [3, 3, in_channels, out_channels]"
    u_plain, _ = _filter_transform(w, in_channels, out_channels, plain=True, packed=False)
    return u_plain


def _launch_winograd(x: torch.Tensor, n: int, h: int, w: int, cin: int, cout: int, u_packed: torch.Tensor,
                     bias, y: torch.Tensor, variant: str = "F2x2") -> None:
    N.check(N.lib().rdvb_conv3x3_winograd(
        x.data_ptr(), _DTYPES[x.dtype], n, h, w, cin, cout, u_packed.data_ptr(), _variant(variant),
        bias.data_ptr() if bias is not None else None, y.data_ptr(), _DTYPES[y.dtype], stream_handle()),
        "rdvb_conv3x3_winograd")


class Conv2DTensorOp(TensorOperation):
    """'same'-padded, stride-1 KHxKW convolution in exact fp32
    (rdv/domain/nn.py:414-469, rdv/shaders/tensors/conv2d_tensor_op.h)."""

    def __init__(self, x, weight, bias, H: int, W: int) -> None:
        data, shape, upstream = _as_op_input(x)
        assert len(shape) == 2, "Conv2DTensorOp requires a 2D (H*W, in_channels) input"
        hw, in_channels = shape
        assert hw == H * W, f"H*W ({H * W}) must match x's own row count ({hw})"
        weight = weight if isinstance(weight, RDVObject) else wrap(weight)
        bias = bias if isinstance(bias, RDVObject) else wrap(bias)
        assert len(weight.shape) == 4, "weight must be [KH, KW, in_channels, out_channels]"
        kh, kw, weight_in_channels, out_channels = weight.shape
        assert weight_in_channels == in_channels, "weight's own in_channels must match x's own trailing dim"
        assert tuple(bias.shape) == (out_channels,), "bias must be [out_channels]"
        assert in_channels % 8 == 0, f"in_channels ({in_channels}) must be a multiple of 8"
        assert out_channels % 8 == 0, f"out_channels ({out_channels}) must be a multiple of 8"
        self.KH, self.KW, self.CIN, self.COUT, self.H, self.W = kh, kw, in_channels, out_channels, H, W
        self.x_buf = data
        self.weight = weight
        self.bias = bias
        self._upstream = upstream
        super().__init__([hw, out_channels])

    def _run(self):
        x = _f32_view(self.x_buf)
        w = _f32_view(self.weight)
        b = _f32_view(self.bias)
        y = self._result._tensor
        N.check(N.lib().rdvb_conv2d_direct(
            x.data_ptr(), N.RDVB_F32, 1, self.H, self.W, self.CIN, self.COUT, self.KH, self.KW, w.data_ptr(),
            b.data_ptr(), y.data_ptr(), stream_handle()), "rdvb_conv2d_direct")


class _StagedConv(TensorOperation):
    """Shared body of the reference's tensor-core direct convolutions:
    x [H*W, in_channels], weight [KH, KW, in_channels, out_channels], bias
    [out_channels]; x and weight rounded to float16, fp32 accumulation over
    (kh, kw, cin). Runs as a tcgen05 implicit GEMM (rdvb_conv2d_tc) when
    the shape fits it, else on the CUDA cores (rdvb_conv2d_direct_staged,
    the bias seeding the accumulator or added after as the op does)."""

    _TILE_ROWS = 32
    _TILE_COLS = 16
    _bias_first = True
    _name = "Conv2DTensorOp"

    def _check(self, x, weight, bias, H, W, fixed_3x3=False):
        data, shape, upstream = _as_op_input(x)
        assert len(shape) == 2, f"{self._name} requires a 2D (H*W, in_channels) input"
        hw, in_channels = shape
        assert hw == H * W, f"H*W ({H * W}) must match x's own row count ({hw})"
        weight = weight if isinstance(weight, RDVObject) else wrap(weight)
        bias = bias if isinstance(bias, RDVObject) else wrap(bias)
        if fixed_3x3:
            assert tuple(weight.shape[:2]) == (3, 3), "weight must be [3, 3, in_channels, out_channels]"
        else:
            assert len(weight.shape) == 4, "weight must be [KH, KW, in_channels, out_channels]"
        kh, kw, weight_in_channels, out_channels = weight.shape
        assert weight_in_channels == in_channels, "weight's own in_channels must match x's own trailing dim"
        assert tuple(bias.shape) == (out_channels,), "bias must be [out_channels]"
        return data, upstream, hw, in_channels, out_channels, kh, kw, weight, bias

    def _setup(self, data, upstream, hw, cin, cout, kh, kw, weight, bias, H, W):
        self.KH, self.KW, self.CIN, self.COUT, self.H, self.W = kh, kw, cin, cout, H, W
        self.x_buf = data
        self.weight = weight
        self.bias = bias
        self._upstream = upstream
        TensorOperation.__init__(self, [hw, cout])

    def _packed(self, w: torch.Tensor):
        """float16 weight image of the tensor-core kernel (re-packed after an
        in-place weight edit), or None when the shape is outside its limits."""
        lib = N.lib()
        nbytes = lib.rdvb_conv_tc_packed_bytes(self.KH, self.KW, self.CIN, self.COUT)
        if nbytes <= 0:
            return None
        key = (w.data_ptr(), self.weight._tensor._version)
        if getattr(self, "_wpack_key", None) != key:
            if getattr(self, "_wpack", None) is None:
                self._wpack = torch.empty(int(nbytes), dtype=torch.uint8, device=w.device)
            N.check(lib.rdvb_conv_tc_pack(w.data_ptr(), self.KH, self.KW, self.CIN, self.COUT, N.RDVB_F16,
                                          self._wpack.data_ptr(), stream_handle()), "rdvb_conv_tc_pack")
            self._wpack_key = key
        return self._wpack

    def _run(self):
        x = _f32_view(self.x_buf)
        w = _f32_view(self.weight)
        b = _f32_view(self.bias)
        y = self._result._tensor
        wpack = self._packed(w)
        if wpack is not None:
            # tcgen05 implicit GEMM: fp32 accumulation from zero, bias in the
            # epilogue (equal to the bias-seeded sum within fp32 rounding)
            N.check(N.lib().rdvb_conv2d_tc(
                x.data_ptr(), N.RDVB_F32, 1, self.H, self.W, self.CIN, self.COUT, self.KH, self.KW,
                wpack.data_ptr(), N.RDVB_F16, b.data_ptr(), y.data_ptr(), stream_handle()), "rdvb_conv2d_tc")
            return
        # shapes outside the tensor-core kernel's limits (cin > 64, cout > 256,
        # more taps than fit shared memory): the same arithmetic on CUDA cores
        N.check(N.lib().rdvb_conv2d_direct_staged(
            x.data_ptr(), N.RDVB_F32, 1, self.H, self.W, self.CIN, self.COUT, self.KH, self.KW, w.data_ptr(),
            b.data_ptr(), N.RDVB_MATH_F16, int(self._bias_first), y.data_ptr(), stream_handle()),
            "rdvb_conv2d_direct_staged")


class Conv2DTensorOpFast(_StagedConv):
    """'same'-padded, stride-1 KHxKW convolution with float16 operands and
    fp32 accumulation, bias added after the sum (rdv/domain/nn.py:608-666,
    rdv/shaders/tensors/conv2d_tensor_op_fast.h)."""

    _bias_first = False
    _name = "Conv2DTensorOpFast"

    def __init__(self, x, weight, bias, H: int, W: int) -> None:
        data, up, hw, cin, cout, kh, kw, weight, bias = self._check(x, weight, bias, H, W)
        assert cin % 16 == 0, f"in_channels ({cin}) must be a multiple of 16"
        assert cout % 16 == 0, f"out_channels ({cout}) must be a multiple of 16"
        self._setup(data, up, hw, cin, cout, kh, kw, weight, bias, H, W)


class Conv2DTensorOpSimple(_StagedConv):
    """'same'-padded, stride-1 KHxKW convolution with float16 operands, the
    fp32 accumulator seeded with the bias (rdv/domain/nn.py:669-754,
    rdv/shaders/tensors/conv2d_tensor_op_simple.h)."""

    _name = "Conv2DTensorOpSimple"

    def __init__(self, x, weight, bias, H: int, W: int) -> None:
        data, up, hw, cin, cout, kh, kw, weight, bias = self._check(x, weight, bias, H, W)
        assert hw % 32 == 0, f"H*W ({hw}) must be a multiple of 32"
        assert cin % 16 == 0, f"in_channels ({cin}) must be a multiple of 16"
        assert cout % 16 == 0, f"out_channels ({cout}) must be a multiple of 16"
        self._setup(data, up, hw, cin, cout, kh, kw, weight, bias, H, W)


class Conv2DTensorOpSimple3x3(_StagedConv):
    """'same'-padded, stride-1 3x3 convolution with float16 operands, the
    fp32 accumulator seeded with the bias (rdv/domain/nn.py:757-848,
    rdv/shaders/tensors/conv2d_tensor_op_simple3x3.h)."""

    _name = "Conv2DTensorOpSimple3x3"

    def __init__(self, x, weight, bias, H: int, W: int) -> None:
        data, up, hw, cin, cout, kh, kw, weight, bias = self._check(x, weight, bias, H, W, fixed_3x3=True)
        assert hw % 32 == 0, f"H*W ({hw}) must be a multiple of 32"
        assert cin % 16 == 0, f"in_channels ({cin}) must be a multiple of 16"
        assert cout % 16 == 0, f"out_channels ({cout}) must be a multiple of 16"
        # the reference's subgroups-per-tile choice (nn.py:830-838); the B200
        # kernel does not use it
        tap_k = 9 * cin
        self.SPT = _max_subgroups(fixed_bytes=32 * tap_k * 2, per_subgroup_bytes=16 * tap_k * 2,
                                  divides=lambda s: cout % (16 * s) == 0)
        self._setup(data, up, hw, cin, cout, kh, kw, weight, bias, H, W)


class Conv2DTensorOpWindow3x3(_StagedConv):
    """'same'-padded, stride-1 3x3 convolution over 8x8 output windows with
    float16 operands, the fp32 accumulator seeded with the bias
    (rdv/domain/nn.py:851-999, rdv/shaders/tensors/conv2d_tensor_op_window3x3.h).
    The reference's separate zero-padding pass into a temporary buffer is not
    needed here: the kernel skips taps outside the image."""

    _TILE_ROWS = 1
    _TILE_COLS = 16
    _WIN = 8
    _name = "Conv2DTensorOpWindow3x3"

    def __init__(self, x, weight, bias, H: int, W: int) -> None:
        data, up, hw, cin, cout, kh, kw, weight, bias = self._check(x, weight, bias, H, W, fixed_3x3=True)
        assert H % self._WIN == 0, f"H ({H}) must be a multiple of {self._WIN}"
        assert W % self._WIN == 0, f"W ({W}) must be a multiple of {self._WIN}"
        assert cin % 16 == 0, f"in_channels ({cin}) must be a multiple of 16"
        assert cout % 16 == 0, f"out_channels ({cout}) must be a multiple of 16"
        assert cin <= 64, f"in_channels ({cin}) must be at most 64 (see this op's own docstring)"
        fetch = self._WIN + 2
        shared_bytes = (fetch * fetch * cin + 16 * 9 * cin) * 2 + 64 * 16 * 2 + 64 * 16 * 4
        assert shared_bytes <= 49152, f"in_channels ({cin}) needs {shared_bytes} bytes of shared memory (48KB budget)"
        self._setup(data, up, hw, cin, cout, kh, kw, weight, bias, H, W)


class Conv2DTensorOpWinograd3x3(TensorOperation):
    """'same'-padded, stride-1 3x3 convolution via Winograd F(2x2, 3x3)
    (rdv/domain/nn.py:1002-1087). The weight is transformed once, at
    construction, into U = G g G^T (float16); later in-place weight edits are
    not seen, as in the reference."""

    _TILE_ROWS = 1
    _TILE_COLS = 16

    def __init__(self, x, weight, bias, H: int, W: int) -> None:
        data, shape, upstream = _as_op_input(x)
        assert len(shape) == 2, "Conv2DTensorOpWinograd3x3 requires a 2D (H*W, in_channels) input"
        hw, in_channels = shape
        assert hw == H * W, f"H*W ({H * W}) must match x's own row count ({hw})"
        weight = weight if isinstance(weight, RDVObject) else wrap(weight)
        bias = bias if isinstance(bias, RDVObject) else wrap(bias)
        assert tuple(weight.shape[:2]) == (3, 3), "weight must be [3, 3, in_channels, out_channels]"
        _, _, weight_in_channels, out_channels = weight.shape
        assert weight_in_channels == in_channels, "weight's own in_channels must match x's own trailing dim"
        assert tuple(bias.shape) == (out_channels,), "bias must be [out_channels]"
        assert H % 2 == 0, f"H ({H}) must be even"
        assert W % 2 == 0, f"W ({W}) must be even"
        assert in_channels % 16 == 0, f"in_channels ({in_channels}) must be a multiple of 16"
        assert out_channels % 16 == 0, f"out_channels ({out_channels}) must be a multiple of 16"
        assert in_channels <= MAX_WINOGRAD_CHANNELS, \
            f"in_channels ({in_channels}) must be at most {MAX_WINOGRAD_CHANNELS} (see this op's own docstring)"
        assert out_channels <= MAX_WINOGRAD_CHANNELS, \
            f"out_channels ({out_channels}) must be at most {MAX_WINOGRAD_CHANNELS} (see this op's own docstring)"
        self.CIN, self.COUT, self.H, self.W = in_channels, out_channels, H, W
        self.x_buf = data
        self.bias = bias
        self._upstream = upstream
        w32 = _f32_view(weight)
        self.weight_u, self._u_packed = _filter_transform(w32, in_channels, out_channels, plain=True, packed=True)
        super().__init__([hw, out_channels])

    def _run(self):
        x = _f32_view(self.x_buf)
        b = _f32_view(self.bias)
        _launch_winograd(x, 1, self.H, self.W, self.CIN, self.COUT, self._u_packed, b, self._result._tensor)


class Conv3x3Winograd:
    """Batched NHWC 'same' 3x3 convolution via Winograd:
    ``Conv3x3Winograd(weight[3,3,CIN,COUT], bias[COUT] | None, variant="F2x2")``,
    then ``conv(x[N,H,W,CIN], out_dtype=torch.float32, out=None)``. x may
    be float32 or float16.

    variant "F2x2": the fused tcgen05 kernel, channels multiples of 16 up to
    64 (the reference operator's transform). variant "F4x4": F(4x4,3x3) on
    CUDA cores with fp32 operands, channels 1..128 (a B200 extension; with
    float16 U and V its error would exceed the 1e-2 tolerance)."""

    def __init__(self, weight, bias=None, variant: str = "F2x2") -> None:
        w = _dev_f32(weight)
        assert w.dim() == 4 and tuple(w.shape[:2]) == (3, 3), "weight must be [3, 3, in_channels, out_channels]"
        self.cin, self.cout = int(w.shape[2]), int(w.shape[3])
        _variant(variant)
        self.variant = variant
        self.bias = _dev_f32(bias) if bias is not None else None
        if self.bias is not None:
            assert tuple(self.bias.shape) == (self.cout,), "bias must be [out_channels]"
        _, self.u_packed = _filter_transform(w, self.cin, self.cout, plain=False, packed=True, variant=variant)

    def __call__(self, x, out_dtype=torch.float32, out: torch.Tensor | None = None) -> torch.Tensor:
        x = x._tensor if isinstance(x, RDVObject) else x
        assert x.dim() == 4 and x.shape[3] == self.cin, f"x must be [N, H, W, {self.cin}]"
        assert x.dtype in _DTYPES, "x must be float32 or float16"
        if x.device != current_device() or not x.is_contiguous():
            x = x.to(current_device()).contiguous()
        n, h, w, _ = (int(v) for v in x.shape)
        if out is None:
            out = torch.empty((n, h, w, self.cout), dtype=out_dtype, device=x.device)
        assert out.shape == (n, h, w, self.cout) and out.dtype in _DTYPES and out.is_contiguous()
        with _timed():
            _launch_winograd(x, n, h, w, self.cin, self.cout, self.u_packed, self.bias, out, self.variant)
        return out


def conv2d_direct(x: torch.Tensor, weight, bias=None) -> torch.Tensor:
    """fp32 'same' direct convolution of NHWC x [N, H, W, CIN] (float32 or
    float16) with weight [KH, KW, CIN, COUT]: the on-device check of the
    Winograd path."""
    w = _dev_f32(weight)
    b = _dev_f32(bias) if bias is not None else None
    x = x.to(current_device()).contiguous()
    n, h, wd, cin = (int(v) for v in x.shape)
    kh, kw, wcin, cout = (int(v) for v in w.shape)
    assert wcin == cin, "weight's own in_channels must match x's own trailing dim"
    y = torch.empty((n, h, wd, cout), dtype=torch.float32, device=x.device)
    with _timed():
        N.check(N.lib().rdvb_conv2d_direct(
            x.data_ptr(), _DTYPES[x.dtype], n, h, wd, cin, cout, kh, kw, w.data_ptr(),
            b.data_ptr() if b is not None else None, y.data_ptr(), stream_handle()), "rdvb_conv2d_direct")
    return y
