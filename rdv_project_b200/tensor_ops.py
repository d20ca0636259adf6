"""Self-materialising 2-D tensor operations (the reference's TensorOperation
family, rdv/maths/__init__.py:1251-1430 and rdv/domain/nn.py).

Each operation validates its inputs with the reference's assertion messages,
allocates its own fp32 ``result`` ``[rows, channels]`` on the device and
dispatches eagerly in ``__init__``; ``evaluate()`` re-dispatches over the
same result buffer, ``evaluate_chain()`` re-dispatches the op and every
upstream op in dependency order, ``as_type(backend)`` returns the result.
Inputs are aliased, so an in-place edit of a leaf tensor followed by
``evaluate_chain()`` recomputes the pipeline, as in the reference.

``evaluate_chain()`` runs each maximal run of linear / ReLU ops that feed
only one another and share one arithmetic (all exact fp32, or all float16
operands fitting the tensor-core kernel) as ONE fused rdvb_mlp_forward
launch: the run's last op gets its result, the ops inside the run are
marked stale and materialise on first use (``result``, ``as_type``, a
downstream ``evaluate()`` or their own ``evaluate_chain()``). The fused
launch computes the same values as the per-op dispatches: the fp32
accumulator + bias of each layer is rounded once to the next layer's
float16 operand either way (ReLU first), and exact fp32 layers keep their
summation order.

Operators and the kernels behind them:

* ``ReLUTensorOp`` -> rdvb_relu.
* ``LinearTensorOp`` (exact fp32) and ``LinearTensorOp{Fast,Mine,Simple,Small}``
  (float16 operands, fp32 accumulate) -> rdvb_mlp_forward with one layer;
  the float16 ones run on the tcgen05 kernel. ``LinearTensorOpSimple``
  converts its weight to float16 once at construction (nn.py:1297,
  ``_cast_fp16``), so like the reference it does not see later in-place
  weight edits; the others re-read the fp32 weight when it has changed.
* ``Downsample2xTensorOp(x, H, W)`` (2x2 average pool), ``Upsample2xTensorOp(x,
  H, W)`` (nearest 2x), ``ConcatTensorOp(g1, g2)`` (channel concat)
  -> rdvb_downsample2x / rdvb_upsample2x / rdvb_concat_channels.
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
    _stale = False

    def __init__(self, shape):
        cls = type(self)
        assert len(shape) == 2, "TensorOperation only supports 2D (rows, channels) shapes"
        assert shape[0] % cls._TILE_ROWS == 0, f"rows ({shape[0]}) must be a multiple of {cls._TILE_ROWS}"
        assert shape[1] % cls._TILE_COLS == 0, f"channels ({shape[1]}) must be a multiple of {cls._TILE_COLS}"
        self._shape = list(shape)
        self.shape = list(shape)
        dev = current_device()
        self._result = RDVObject(torch.empty(self._shape, dtype=torch.float32, device=dev))
        self._output_t = self._result
        self.evaluate()

    @property
    def result(self) -> RDVObject:
        if self._stale:
            self.evaluate_chain()
        return self._result

    def as_type(self, backend):
        if self._stale:
            self.evaluate_chain()
        return self._output_t.as_tensor(backend).reshape(self._shape)

    def evaluate(self):
        for up in (self._upstream, *self._extra_upstreams):
            if up is not None and up._stale:
                up.evaluate_chain()
        with _timed():
            self._run()
        self._stale = False

    def evaluate_chain(self):
        ops = []
        _collect_tensor_ops(self, set(), ops)
        with _timed():
            _run_chain_fused(ops, self)

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


def _fusable(op) -> bool:
    return isinstance(op, (_LinearOpBase, ReLUTensorOp))


def _linear_math(run):
    maths = {op._math for op in run if isinstance(op, _LinearOpBase)}
    return maths.pop() if len(maths) == 1 else None


def _tc_eligible(dims) -> bool:
    return N.lib().rdvb_mlp_packed_bytes(len(dims) - 1, N.int_array(dims)) > 0


def _run_chain_fused(ops, final) -> None:
    """Dispatches `ops` (dependency order) with each fusable run as one
    launch; see the module docstring."""
    consumers = {id(op): 0 for op in ops}
    for op in ops:
        for up in (op._upstream, *op._extra_upstreams):
            if up is not None and id(up) in consumers:
                consumers[id(up)] += 1
    i = 0
    while i < len(ops):
        run = [ops[i]]
        if _fusable(ops[i]):
            j = i
            while j + 1 < len(ops):
                a, b = ops[j], ops[j + 1]
                if not (_fusable(b) and b._upstream is a and not b._extra_upstreams and consumers[id(a)] == 1
                        and a is not final):
                    break
                cand = run + [b]
                if _linear_math(cand) is None and any(isinstance(o, _LinearOpBase) for o in cand):
                    break
                run = cand
                j += 1
        if not _launch_fused(run):
            for op in run:
                op._run()
                op._stale = False
        i += len(run)


def _launch_fused(run) -> bool:
    """One rdvb_mlp_forward for a run of >= 2 ops holding >= 1 linear op;
    False when the run is dispatched op by op instead."""
    linears = [op for op in run if isinstance(op, _LinearOpBase)]
    if len(run) < 2 or not linears or len(linears) > 16:
        return False
    input_relu = 0
    layers = []  # [op, relu_after]
    for op in run:
        if isinstance(op, _LinearOpBase):
            layers.append([op, False])
        elif layers:
            layers[-1][1] = True
        else:
            input_relu = 1
    math = _linear_math(run)
    dims = [layers[0][0].weight.shape[1]] + [op.weight.shape[0] for op, _ in layers]
    if math != N.RDVB_MATH_F32 and not _tc_eligible(dims):
        return False  # would run on the CUDA cores with a different summation order
    first = run[0]
    x = _f32_view(first.x_buf)
    Ws, bs = [], []
    for op, _ in layers:
        W, b = op._prepare_weights()
        Ws.append(W)
        bs.append(b)
    flags = [op._math | (N.RDVB_LAYER_RELU if relu else 0) for op, relu in layers]
    last = run[-1]
    packed = None
    if math != N.RDVB_MATH_F32:
        key = tuple((w.data_ptr(), w._version, b.data_ptr(), b._version) for w, b in zip(Ws, bs))
        cache = last.__dict__.setdefault("_fused_pack", {})
        packed = cache.get(key)
        if packed is None:
            lib = N.lib()
            nbytes = lib.rdvb_mlp_packed_bytes(len(layers), N.int_array(dims))
            packed = torch.empty(int(nbytes), dtype=torch.uint8, device=x.device)
            N.check(lib.rdvb_mlp_pack(len(layers), N.int_array(dims), N.ptr_array([w.data_ptr() for w in Ws]),
                                      N.ptr_array([b.data_ptr() for b in bs]), N.RDVB_F16, packed.data_ptr(),
                                      stream_handle()), "rdvb_mlp_pack")
            cache.clear()
            cache[key] = packed
    y = last._result._tensor
    N.check(N.lib().rdvb_mlp_forward(
        x.data_ptr(), N.RDVB_F32, x.shape[0], len(layers), N.int_array(dims),
        N.ptr_array([w.data_ptr() for w in Ws]), N.ptr_array([b.data_ptr() for b in bs]), N.int_array(flags),
        input_relu, 0, packed.data_ptr() if packed is not None else None, y.data_ptr(), stream_handle()),
        "rdvb_mlp_forward")
    for op in run[:-1]:
        op._stale = True
    last._stale = False
    return True


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
        y = self._result._tensor
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
        y = self._result._tensor
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


class Downsample2xTensorOp(TensorOperation):
    """2x2 average pool, stride 2, over a flattened [H*W, C] input
    (rdv/domain/nn.py:1090-1107, rdv/shaders/tensors/downsample2x_tensor_op.h)."""

    def __init__(self, x, H: int, W: int) -> None:
        data, shape, upstream = _as_op_input(x)
        assert len(shape) == 2, "Downsample2xTensorOp requires a 2D (H*W, C) input"
        hw, channels = shape
        assert hw == H * W, f"H*W ({H * W}) must match x's own row count ({hw})"
        assert H % 2 == 0 and W % 2 == 0, "Downsample2xTensorOp requires even H and W"
        self.x_buf = data
        self.H_in, self.W_in = H, W
        self.W = W // 2  # output width
        self._upstream = upstream
        super().__init__([(H // 2) * (W // 2), channels])

    def _run(self):
        x = _f32_view(self.x_buf)
        y = self._result._tensor
        N.check(N.lib().rdvb_downsample2x(x.data_ptr(), self.H_in, self.W_in, y.shape[1], y.data_ptr(),
                                          stream_handle()), "rdvb_downsample2x")


class Upsample2xTensorOp(TensorOperation):
    """Nearest-neighbour 2x upsample over a flattened [H*W, C] input
    (rdv/domain/nn.py:1110-1124, rdv/shaders/tensors/upsample2x_tensor_op.h)."""

    def __init__(self, x, H: int, W: int) -> None:
        data, shape, upstream = _as_op_input(x)
        assert len(shape) == 2, "Upsample2xTensorOp requires a 2D (H*W, C) input"
        hw, channels = shape
        assert hw == H * W, f"H*W ({H * W}) must match x's own row count ({hw})"
        self.x_buf = data
        self.H_in, self.W_in = H, W
        self.W = W * 2  # output width
        self._upstream = upstream
        super().__init__([(H * 2) * (W * 2), channels])

    def _run(self):
        x = _f32_view(self.x_buf)
        y = self._result._tensor
        N.check(N.lib().rdvb_upsample2x(x.data_ptr(), self.H_in, self.W_in, y.shape[1], y.data_ptr(),
                                        stream_handle()), "rdvb_upsample2x")


class ConcatTensorOp(TensorOperation):
    """Channel concat of two ops/tensors sharing the H*W leading dim
    (rdv/domain/nn.py:1127-1150, rdv/shaders/tensors/concat_tensor_op.h)."""

    def __init__(self, g1, g2) -> None:
        data1, shape1, up1 = _as_op_input(g1)
        data2, shape2, up2 = _as_op_input(g2)
        assert len(shape1) == 2 and len(shape2) == 2, "ConcatTensorOp requires 2D (H*W, C) inputs"
        assert shape1[0] == shape2[0], "g1/g2 must share the same H*W leading dim"
        assert shape1[1] % 8 == 0, f"g1's own channels ({shape1[1]}) must be a multiple of 8"
        assert shape2[1] % 8 == 0, f"g2's own channels ({shape2[1]}) must be a multiple of 8"
        self.x1_buf = data1
        self.x2_buf = data2
        self.C1 = shape1[1]
        self._upstream = up1
        self._extra_upstreams = (up2,) if up2 is not None else ()
        super().__init__([shape1[0], shape1[1] + shape2[1]])

    def _run(self):
        x1 = _f32_view(self.x1_buf)
        x2 = _f32_view(self.x2_buf)
        y = self._result._tensor
        N.check(N.lib().rdvb_concat_channels(x1.data_ptr(), x1.shape[1], x2.data_ptr(), x2.shape[1], y.shape[0],
                                             y.data_ptr(), stream_handle()), "rdvb_concat_channels")
