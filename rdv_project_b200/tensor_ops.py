"""Self-materialising 2-D tensor operations (the reference's TensorOperation
family, rdv/maths/__init__.py:1251-1430 and rdv/domain/nn.py).

Each operation validates its inputs with the reference's assertion messages,
allocates its own fp32 ``result`` ``[rows, channels]`` on the device and
dispatches eagerly in ``__init__``; ``evaluate()`` re-dispatches over the
same result buffer, ``evaluate_chain()`` re-dispatches the op and every
upstream op in dependency order, ``as_type(backend)`` returns the result.
Inputs are aliased, so an in-place edit of a leaf tensor followed by
``evaluate_chain()`` recomputes the pipeline, as in the reference.

Operators and the kernels behind them:

* ``ReLUTensorOp`` -> rdvb_relu.
* ``LinearTensorOp`` (exact fp32) and ``LinearTensorOp{Fast,Mine,Simple,Small}``
  (float16 operands, fp32 accumulate) -> rdvb_mlp_forward with one layer;
  the float16 ones run on the tcgen05 kernel. ``LinearTensorOpSimple``
  converts its weight to float16 once at construction (nn.py:1297,
  ``_cast_fp16``), so like the reference it does not see later in-place
  weight edits; the others re-read the fp32 weight when it has changed.
* Convolutions live in ``conv.py``.
"""
from __future__ import annotations

import torch

from . import _native as N
from .core import RDVObject, _timed, current_device, stream_handle, wrap

BLOCK_ROWS = 4
BLOCK_CHANNELS = 8


def _max_subgroups(fixed_bytes, per_subgroup_bytes, divides, budget=49152, cap=32):
    """Largest power-of-two subgroup count whose shared-memory footprint fits
    the reference hardware's 48 KB budget (rdv/domain/nn.py:504-519). Kept
    only so the reference's divisibility assertions (LinearTensorOpSimple's
    out_features multiple of 16*SPT) read the same; the B200 kernels do not
    use it."""
    spt = 1
    while spt * 2 <= cap and fixed_bytes + (spt * 2) * per_subgroup_bytes <= budget and divides(spt * 2):
        spt *= 2
    return spt


class TensorOperation:
    _TILE_ROWS = BLOCK_ROWS
    _TILE_COLS = BLOCK_CHANNELS
    _shape = None
    _upstream = None
    _extra_upstreams = ()

    def __init__(self, shape):
        cls = type(self)
        assert len(shape) == 2, "TensorOperation only supports 2D (rows, channels) shapes"
        assert shape[0] % cls._TILE_ROWS == 0, f"rows ({shape[0]}) must be a multiple of {cls._TILE_ROWS}"
        assert shape[1] % cls._TILE_COLS == 0, f"channels ({shape[1]}) must be a multiple of {cls._TILE_COLS}"
        self._shape = list(shape)
        self.shape = list(shape)
        dev = current_device()
        self.result = RDVObject(torch.empty(self._shape, dtype=torch.float32, device=dev))
        self._output_t = self.result
        self.evaluate()

    def as_type(self, backend):
        return self._output_t.as_tensor(backend).reshape(self._shape)

    def evaluate(self):
        with _timed():
            self._run()

    def evaluate_chain(self):
        ops = []
        _collect_tensor_ops(self, set(), ops)
        for op in ops:
            op.evaluate()

    def _run(self):  # pragma: no cover - abstract
        raise NotImplementedError


def _as_op_input(x):
    """(data, shape, upstream) for an op input: another TensorOperation's
    result, or raw data (wrapped, aliased when already on the device)
    (rdv/maths/__init__.py:1402-1415)."""
    if isinstance(x, TensorOperation):
        return x.result, list(x._shape), x
    data = x if isinstance(x, RDVObject) else wrap(x)
    return data, list(data.shape), None


def _collect_tensor_ops(node, seen_ids, out):
    if id(node) in seen_ids:
        return
    if node._upstream is not None:
        _collect_tensor_ops(node._upstream, seen_ids, out)
    for up in node._extra_upstreams:
        _collect_tensor_ops(up, seen_ids, out)
    seen_ids.add(id(node))
    out.append(node)


def _f32_view(obj: RDVObject) -> torch.Tensor:
    t = obj._tensor
    dev = current_device()
    if t.device != dev or t.dtype != torch.float32 or not t.is_contiguous():
        t = t.to(device=dev, dtype=torch.float32).contiguous()
    return t


class ReLUTensorOp(TensorOperation):
    """f(x) = max(x, 0) (rdv/domain/nn.py:362-374)."""

    def __init__(self, x) -> None:
        data, shape, upstream = _as_op_input(x)
        self.x_buf = data
        self._upstream = upstream
        super().__init__(shape)

    def _run(self):
        x = _f32_view(self.x_buf)
        y = self.result._tensor
        N.check(N.lib().rdvb_relu(x.data_ptr(), y.data_ptr(), y.numel(), stream_handle()), "rdvb_relu")


class _LinearOpBase(TensorOperation):
    _math = N.RDVB_MATH_F32
    _name = "LinearTensorOp"
    _precast = False

    def _check_linear(self, x, weight, bias):
        data, shape, upstream = _as_op_input(x)
        assert len(shape) == 2, f"{self._name} requires a 2D (BATCH, in_features) input"
        batch, in_features = shape
        weight = weight if isinstance(weight, RDVObject) else wrap(weight)
        bias = bias if isinstance(bias, RDVObject) else wrap(bias)
        assert len(weight.shape) == 2, "weight must be [out_features, in_features]"
        out_features, weight_in_features = weight.shape
        assert weight_in_features == in_features, "weight's own in_features must match x's own trailing dim"
        assert tuple(bias.shape) == (out_features,), "bias must be [out_features]"
        return data, batch, in_features, out_features, weight, bias, upstream

    def _setup(self, data, weight, bias, upstream, batch, out_features):
        self.x_buf = data
        self.weight = weight
        self.bias = bias
        self._upstream = upstream
        self._packed = None
        self._packed_key = None
        if self._precast:
            self._prepare_weights(force=True)
        super().__init__([batch, out_features])

    def _prepare_weights(self, force=False):
        W = _f32_view(self.weight)
        b = _f32_view(self.bias)
        if self._precast and self._packed is not None:
            return self._W32, self._b32
        self._W32, self._b32 = W, b
        if self._math == N.RDVB_MATH_F32:
            return W, b
        key = (W.data_ptr(), self.weight._tensor._version, b.data_ptr(), self.bias._tensor._version)
        if not force and self._packed is not None and key == self._packed_key:
            return W, b
        lib = N.lib()
        dims = N.int_array([W.shape[1], W.shape[0]])
        nbytes = lib.rdvb_mlp_packed_bytes(1, dims)
        if nbytes > 0:
            if self._packed is None:
                self._packed = torch.empty(int(nbytes), dtype=torch.uint8, device=W.device)
            N.check(lib.rdvb_mlp_pack(1, dims, N.ptr_array([W.data_ptr()]), N.ptr_array([b.data_ptr()]),
                                      N.RDVB_F16, self._packed.data_ptr(), stream_handle()), "rdvb_mlp_pack")
            if self._precast:
                # the fp32 fallback path must see the same (construction-time) values
                self._W32 = W.clone()
                self._b32 = b.clone()
        self._packed_key = key
        return self._W32, self._b32

    def _run(self):
        W, b = self._prepare_weights()
        x = _f32_view(self.x_buf)
        y = self.result._tensor
        rc = N.lib().rdvb_mlp_forward(
            x.data_ptr(), N.RDVB_F32, x.shape[0], 1, N.int_array([W.shape[1], W.shape[0]]),
            N.ptr_array([W.data_ptr()]), N.ptr_array([b.data_ptr()]), N.int_array([self._math]), 0, 0,
            self._packed.data_ptr() if self._packed is not None else None, y.data_ptr(), stream_handle())
        N.check(rc, "rdvb_mlp_forward")


class LinearTensorOp(_LinearOpBase):
    """Exact fp32 y = W @ x + b (rdv/domain/nn.py:377-411)."""

    _math = N.RDVB_MATH_F32
    _name = "LinearTensorOp"

    def __init__(self, x, weight, bias) -> None:
        data, batch, inf, outf, weight, bias, up = self._check_linear(x, weight, bias)
        assert inf % 8 == 0, f"in_features ({inf}) must be a multiple of 8"
        assert outf % 8 == 0, f"out_features ({outf}) must be a multiple of 8"
        self._setup(data, weight, bias, up, batch, outf)


class LinearTensorOpFast(_LinearOpBase):
    """float16-operand y = W @ x + b (rdv/domain/nn.py:541-605)."""

    _math = N.RDVB_MATH_F16
    _name = "LinearTensorOpFast"
    _TILE_ROWS = 32 * 2
    _TILE_COLS = 16 * 2

    def __init__(self, x, weight, bias) -> None:
        data, batch, inf, outf, weight, bias, up = self._check_linear(x, weight, bias)
        assert batch % self._TILE_ROWS == 0, f"batch ({batch}) must be a multiple of {self._TILE_ROWS}"
        assert inf % 16 == 0, f"in_features ({inf}) must be a multiple of 16"
        assert outf % self._TILE_COLS == 0, f"out_features ({outf}) must be a multiple of {self._TILE_COLS}"
        self._setup(data, weight, bias, up, batch, outf)


class LinearTensorOpMine(_LinearOpBase):
    """float16-operand y = W @ x + b (rdv/domain/nn.py:1153-1201)."""

    _math = N.RDVB_MATH_F16
    _name = "LinearTensorOpMine"
    _TILE_ROWS = 32
    _TILE_COLS = 16

    def __init__(self, x, weight, bias) -> None:
        data, batch, inf, outf, weight, bias, up = self._check_linear(x, weight, bias)
        assert batch % 32 == 0, f"batch ({batch}) must be a multiple of 32"
        assert inf % 16 == 0, f"in_features ({inf}) must be a multiple of 16"
        assert outf % 16 == 0, f"out_features ({outf}) must be a multiple of 16"
        self._setup(data, weight, bias, up, batch, outf)


class LinearTensorOpSimple(_LinearOpBase):
    """float16-operand y = W @ x + b with the weight cast to float16 once at
    construction (rdv/domain/nn.py:1204-1300)."""

    _math = N.RDVB_MATH_F16
    _name = "LinearTensorOpSimple"
    _TILE_ROWS = 32
    _TILE_COLS = 16
    _precast = True

    def __init__(self, x, weight, bias) -> None:
        data, batch, inf, outf, weight, bias, up = self._check_linear(x, weight, bias)
        assert batch % 32 == 0, f"batch ({batch}) must be a multiple of 32"
        assert inf % 16 == 0, f"in_features ({inf}) must be a multiple of 16"
        spt = _max_subgroups(fixed_bytes=32 * inf * 2, per_subgroup_bytes=16 * inf * 2,
                             divides=lambda s: outf % (16 * s) == 0)
        out_tile = 16 * spt
        assert outf % out_tile == 0, f"out_features ({outf}) must be a multiple of {out_tile}"
        self._setup(data, weight, bias, up, batch, outf)


class LinearTensorOpSmall(_LinearOpBase):
    """float16-operand y = W @ x + b for in/out_features <= 128
    (rdv/domain/nn.py:1303-1411)."""

    _math = N.RDVB_MATH_F16
    _name = "LinearTensorOpSmall"
    _TILE_ROWS = 32
    _TILE_COLS = 16

    def __init__(self, x, weight, bias) -> None:
        data, batch, inf, outf, weight, bias, up = self._check_linear(x, weight, bias)
        assert batch % 32 == 0, f"batch ({batch}) must be a multiple of 32"
        assert inf % 16 == 0, f"in_features ({inf}) must be a multiple of 16"
        assert outf % 16 == 0, f"out_features ({outf}) must be a multiple of 16"
        assert inf <= 128, f"in_features ({inf}) must be at most 128 (see this op's own docstring)"
        assert outf <= 128, f"out_features ({outf}) must be at most 128 (see this op's own docstring)"
        self._setup(data, weight, bias, up, batch, outf)
