"""Map algebra of the hot path: Linear / LinearFast / ReLU / Identity and
their ``>>`` composition, evaluated as ONE fused kernel launch.

Reference surface mirrored (same names, argument meaning and assertion
messages):

* ``linear(weight, bias, f16=False)`` -> ``LinearFast`` if f16 else ``Linear``
  (rdv/domain/nn.py:99-104); ``_LinearBase.__init__`` checks
  (nn.py:34-41): weight ``[out_features, in_features]`` (PyTorch nn.Linear
  layout), bias ``[out_features]``.
* ``ReLU`` / ``relu`` (nn.py:107-119) and ``Identity`` / ``X``
  (rdv/maths/__init__.py:1671-1687): generic maps whose width is bound by
  whatever they are composed with.
* ``m1 >> m2`` (maths/__init__.py:1489-1498): ``Composite(m2, m1)``, i.e.
  f(g(x)) with g = m1; Identity operands are dropped; ``Composite`` asserts
  "g's OUT must match f's IN - g's output is f's input." (:1722-1723).
* ``m(x)`` (maths/__init__.py:1451-1487): one row per leading index of x,
  output ``[..., OUT]`` float32, the output buffer allocated once per
  (instance, shape) and reused by later calls with the same shape.

Evaluation lowers the composed chain to an affine-layer list and calls
``rdvb_mlp_forward`` once: all-LinearFast chains run on the tcgen05 fused
kernel (float16 operands, fp32 accumulate and bias, like
rdv/shaders/maps/linear_fast.h), chains containing exact ``Linear`` layers on
the CUDA-core kernel (rdv/shaders/maps/linear.h arithmetic). A trailing
partial 32-row group evaluates in exact fp32, as the reference's
cooperative-matrix path falls back when its 32-lane workgroup is not full
(linear_fast.h:44,102-108).
"""
from __future__ import annotations

import torch

from . import _native as N
from .core import RDVObject, _timed, current_device, stream_handle, wrap


class Map:
    """Pointwise row map with input width IN and output width OUT (None while
    generic)."""

    IN = None
    OUT = None

    # -- composition -------------------------------------------------------
    def __rshift__(self, m):
        if not isinstance(m, Map):
            return NotImplemented
        return _compose(m, self)

    def __rrshift__(self, other):
        return NotImplemented

    def __lshift__(self, m):
        if not isinstance(m, Map):
            return NotImplemented
        return _compose(self, m)

    # -- generic binding ------------------------------------------------------
    def _bind(self, in_size=None, out_size=None) -> "Map":
        """Concrete version of this map for the given widths (a generic map
        returns a bound copy; a concrete one returns itself)."""
        return self

    def _ops(self):
        return [self]

    @property
    def __is_generic__(self) -> bool:
        return self.IN is None or self.OUT is None

    # -- evaluation ------------------------------------------------------------
    def __call__(self, *args, **kwargs):
        if len(args) != 1:
            raise TypeError("a Map is called with exactly one input tensor")
        x, = args
        in_size = x.shape[-1]
        m = self
        if self.__is_generic__:
            m = self._bind(in_size=in_size)
            if m.__is_generic__:
                raise RuntimeError("Generic arguments could not be deduced from input data. You must explicitly cast.")
        assert in_size == m.IN, f"input's last dimension ({in_size}) must match the map's IN ({m.IN})"
        return _evaluate(m, self, x)


class Identity(Map):
    """f(x) = x."""

    def __init__(self, size=None):
        self.IN = size
        self.OUT = size

    def _bind(self, in_size=None, out_size=None):
        size = in_size if in_size is not None else out_size
        if self.IN is not None or size is None:
            return self
        return Identity(size)


X = Identity()


class ReLU(Map):
    """f(x) = max(x, 0), elementwise (rdv/shaders/maps/relu.h)."""

    def __init__(self, size=None):
        self.IN = size
        self.OUT = size

    def _bind(self, in_size=None, out_size=None):
        size = in_size if in_size is not None else out_size
        if self.IN is not None or size is None:
            return self
        return ReLU(size)


relu = ReLU()


class _LinearBase(Map):
    """y = W @ x + b; weight [OUT, IN] (PyTorch nn.Linear layout), bias [OUT]."""

    _math = N.RDVB_MATH_F32
    __next_id__ = 0

    def __init__(self, weight, bias) -> None:
        weight = weight if isinstance(weight, RDVObject) else wrap(weight)
        bias = bias if isinstance(bias, RDVObject) else wrap(bias)
        assert len(weight.shape) == 2, "weight must be [out_features, in_features]"
        out_features, in_features = weight.shape
        assert tuple(bias.shape) == (out_features,), "bias must be [out_features]"
        self.IN = in_features
        self.OUT = out_features
        self.weight = weight
        self.bias = bias
        cls = type(self)
        self.id = cls.__next_id__
        cls.__next_id__ += 1

    def _fp32(self, obj: RDVObject, dev) -> torch.Tensor:
        t = obj._tensor
        if t.device != dev or t.dtype != torch.float32 or not t.is_contiguous():
            t = t.to(device=dev, dtype=torch.float32).contiguous()
        return t


class Linear(_LinearBase):
    """Exact fp32 linear layer (rdv/shaders/maps/linear.h)."""

    _math = N.RDVB_MATH_F32
    __next_id__ = 0


class LinearFast(_LinearBase):
    """Linear layer on the tensor cores: float16 operands, fp32 accumulation,
    fp32 bias (rdv/shaders/maps/linear_fast.h)."""

    _math = N.RDVB_MATH_F16
    __next_id__ = 0


class LinearFastBF16(_LinearBase):
    """bfloat16-operand variant of LinearFast (B200 extension; the reference
    has float16 only)."""

    _math = N.RDVB_MATH_BF16
    __next_id__ = 0


def linear(weight, bias, f16: bool = False):
    """`x >> linear(weight, bias)` - Linear (default, exact fp32) or, with
    f16=True, LinearFast (tensor-core matmul, float16 operands)."""
    return (LinearFast if f16 else Linear)(weight, bias)


class TensorSampler(Map):
    """Multilinear (linear=True) or nearest lookup of a dense fp32 tensor
    t [D0, ..., D(IN-1), OUT] at points in [-1, 1]^IN
    (rdv/maths/__init__.py:2050-2083, rdv/shaders/samplers/tensor_sampler.h):
    clamp clamps out-of-range corners (else they contribute 0), aligned ties
    -1/+1 to the first/last cell centres (else to the outer edges), as
    torch's grid_sample. IN is 1, 2 or 3. Composed before a Linear chain
    (``sampler >> mlp``) it is the chain's input encoding: one sampler
    launch, then the fused MLP on its output."""

    def __init__(self, t, clamp: bool = True, aligned: bool = False, linear: bool = True) -> None:
        t = t if isinstance(t, RDVObject) else wrap(t)
        n = len(t.shape)
        assert 2 <= n <= 4, "TensorSampler supports 1- to 3-dimensional grids (a [D0, ..., OUT] tensor)"
        self.t = t
        self.IN = n - 1
        self.OUT = t.shape[n - 1]
        self.clamp = 1 if clamp else 0
        self.aligned = 1 if aligned else 0
        self.linear = 1 if linear else 0

    def _sample(self, x2d: torch.Tensor, y2d: torch.Tensor) -> None:
        t = self.t._tensor
        if t.device != x2d.device or t.dtype != torch.float32 or not t.is_contiguous():
            t = t.to(device=x2d.device, dtype=torch.float32).contiguous()
        N.check(N.lib().rdvb_tensor_sampler(
            t.data_ptr(), self.IN, N.int_array(list(t.shape[:self.IN])), self.OUT, x2d.data_ptr(), x2d.shape[0],
            self.clamp, self.aligned, self.linear, y2d.data_ptr(), stream_handle()), "rdvb_tensor_sampler")

    def __call__(self, *args, **kwargs):
        if len(args) != 1:
            raise TypeError("a Map is called with exactly one input tensor")
        x, = args
        xt = x._tensor if isinstance(x, RDVObject) else wrap(x)._tensor
        assert xt.shape[-1] == self.IN, f"input's last dimension ({xt.shape[-1]}) must match the map's IN ({self.IN})"
        dev = current_device()
        x2d = xt.reshape(-1, self.IN).to(device=dev, dtype=torch.float32).contiguous()
        out = torch.empty(list(xt.shape[:-1]) + [self.OUT], dtype=torch.float32, device=dev)
        with _timed():
            if x2d.shape[0]:
                self._sample(x2d, out.view(-1, self.OUT))
        return RDVObject(out)


class GridSampler(Map):
    """Multilinear (linear=True) or nearest lookup of a grid at points in
    [-1, 1]^IN (rdv/maths/__init__.py:2018-2047,
    rdv/shaders/samplers/grid_sampler.h): clamp clamps out-of-range corners
    (else they are skipped), aligned ties -1/+1 to the first/last cell
    centres (else to the outer edges). ``g`` is a dense grid: a TensorGrid
    (rdv_project_b200.volumes) or its tensor [D0, ..., D(IN-1), OUT], IN 1
    to 4 -> rdvb_grid_sampler. Its position and corner arithmetic is the
    GridSampler's, not the TensorSampler's, so the two round differently on
    the same tensor, as in the reference. Composed before a Linear chain
    (``sampler >> mlp``) it is the chain's input encoding, like the
    TensorSampler."""

    def __init__(self, g, clamp: bool = True, aligned: bool = False, linear: bool = True) -> None:
        data = getattr(g, "data", g)     # a TensorGrid holds its tensor in .data
        t = data if isinstance(data, RDVObject) else wrap(data)
        n = len(t.shape)
        assert 2 <= n <= 5, "GridSampler supports 1- to 4-dimensional grids (a [D0, ..., OUT] tensor)"
        self.g = g
        self.t = t
        self.IN = n - 1
        self.OUT = t.shape[n - 1]
        self.clamp = 1 if clamp else 0
        self.aligned = 1 if aligned else 0
        self.linear = 1 if linear else 0

    def _sample(self, x2d: torch.Tensor, y2d: torch.Tensor) -> None:
        t = self.t._tensor
        if t.device != x2d.device or t.dtype != torch.float32 or not t.is_contiguous():
            t = t.to(device=x2d.device, dtype=torch.float32).contiguous()
        N.check(N.lib().rdvb_grid_sampler(
            t.data_ptr(), self.IN, N.int_array(list(t.shape[:self.IN])), self.OUT, x2d.data_ptr(), x2d.shape[0],
            self.clamp, self.aligned, self.linear, y2d.data_ptr(), stream_handle()), "rdvb_grid_sampler")

    def __call__(self, *args, **kwargs):
        return TensorSampler.__call__(self, *args, **kwargs)


class Constant(Map):
    """f(x) = data for every x (rdv/maths/__init__.py:1659-1668,
    rdv/shaders/maps/constant.h): OUT = data's last dimension, IN generic.
    PBVR takes a Constant[3, 3] as a uniform environment."""

    def __init__(self, data, in_size=None) -> None:
        t = data._tensor if isinstance(data, RDVObject) else torch.as_tensor(data, dtype=torch.float32)
        self.data = t.reshape(-1).to(torch.float32)
        self.IN = in_size
        self.OUT = int(self.data.numel())

    def _bind(self, in_size=None, out_size=None):
        if self.IN is not None or in_size is None:
            return self
        return Constant(self.data, in_size)

    def __call__(self, *args, **kwargs):
        if len(args) != 1:
            raise TypeError("a Map is called with exactly one input tensor")
        xt = _device_tensor(args[0])
        dev = current_device()
        out = self.data.to(dev).expand(list(xt.shape[:-1]) + [self.OUT]).contiguous()
        return RDVObject(out)


class XRProject(Map):
    """Map[3, 2]: a direction's equirectangular coordinates
    (rdv/domain/rendering.py:150-160, rdv/shaders/rendering/xr_project.h,
    dir2xr of rdv/shaders/libraries/math_library.h:265-276):
    (atan(w.x, w.z) / pi, asin(clamp(w.y, -1, 1)) * 2 / pi) ->
    rdvb_xr_project. ``XRProject() >> TensorSampler(image [H, W, C])`` looks
    an environment image up by direction (PBVR's environment)."""

    IN = 3
    OUT = 2

    def _project(self, x2d: torch.Tensor, y2d: torch.Tensor) -> None:
        N.check(N.lib().rdvb_xr_project(x2d.data_ptr(), x2d.shape[0], y2d.data_ptr(), stream_handle()),
                "rdvb_xr_project")


dir2xr = XRProject()


class Composite(Map):
    """f(g(x)); g's OUT must match f's IN."""

    def __init__(self, f: Map, g: Map) -> None:
        assert g.OUT == f.IN, "g's OUT must match f's IN - g's output is f's input."
        self.f = f
        self.g = g
        self.IN = g.IN
        self.OUT = f.OUT
        self._out_cache = {}
        self._pack_cache = {}

    def _ops(self):
        return self.g._ops() + self.f._ops()

    def _bind(self, in_size=None, out_size=None):
        if not self.__is_generic__:
            return self
        g = self.g._bind(in_size=in_size) if self.g.IN is None else self.g
        f = self.f
        if f.IN is None and g.OUT is not None:
            f = f._bind(in_size=g.OUT)
        if g.OUT is None and f.IN is not None:
            g = g._bind(out_size=f.IN)
        if f is self.f and g is self.g:
            return self
        return Composite(f, g)


def _compose(f: Map, g: Map) -> Map:
    """f(g(x)), binding whichever side is still generic to the other's width."""
    if g.OUT is not None and f.IN is None:
        f = f._bind(in_size=g.OUT)
    if f.IN is not None and g.OUT is None:
        g = g._bind(out_size=f.IN)
    if isinstance(g, Identity):
        return f
    if isinstance(f, Identity):
        return g
    return Composite(f, g)


# ---------------------------------------------------------------- lowering
def _lower(m: Map):
    """Composed map -> (input_relu, [linear layers], [relu after each])."""
    input_relu = False
    layers = []
    relus = []
    for op in m._ops():
        if isinstance(op, (TensorSampler, GridSampler, XRProject)):
            raise NotImplementedError(f"a {type(op).__name__} must come first in the chain (its input encoding)")
        if isinstance(op, _LinearBase):
            layers.append(op)
            relus.append(False)
        elif isinstance(op, ReLU):
            if layers:
                relus[-1] = True
            else:
                input_relu = True
        elif isinstance(op, Identity):
            continue
        else:
            raise NotImplementedError(f"{type(op).__name__} is not part of the fused MLP path")
    return input_relu, layers, relus


def _weights_key(layers):
    return tuple((l.weight._tensor.data_ptr(), l.weight._tensor._version,
                  l.bias._tensor.data_ptr(), l.bias._tensor._version) for l in layers)


class _ChainPlan:
    """Per-device lowered chain: an optional leading TensorSampler (the
    input encoding), fp32 weight views, flags and (for float16/bfloat16
    chains) the packed tensor-core weight image."""

    def __init__(self, m: Map, dev):
        ops = m._ops()
        self.project = ops[0] if ops and isinstance(ops[0], XRProject) else None
        if self.project is not None:
            ops = ops[1:]
        self.prologue = ops[0] if ops and isinstance(ops[0], (TensorSampler, GridSampler)) else None
        if self.prologue is not None:
            ops = ops[1:]
        rest = _compose_ops(ops)
        self.input_relu, self.layers, self.relus = _lower(rest) if rest is not None else (False, [], [])
        self.dev = dev
        first = self.prologue.OUT if self.prologue is not None else (2 if self.project is not None else m.IN)
        self.dims = [first] + [l.OUT for l in self.layers]
        self.flags = [l._math | (N.RDVB_LAYER_RELU if r else 0) for l, r in zip(self.layers, self.relus)]
        self.packed = None
        self.packed_key = None
        self.operand = None
        maths = {l._math for l in self.layers}
        if len(maths) == 1 and next(iter(maths)) != N.RDVB_MATH_F32:
            self.operand = N.RDVB_F16 if next(iter(maths)) == N.RDVB_MATH_F16 else N.RDVB_BF16

    def refresh(self):
        Ws = [l._fp32(l.weight, self.dev) for l in self.layers]
        bs = [l._fp32(l.bias, self.dev) for l in self.layers]
        self.Ws, self.bs = Ws, bs
        if self.operand is None or not self.layers:
            return
        key = _weights_key(self.layers)
        if self.packed is not None and key == self.packed_key:
            return
        lib = N.lib()
        dims = N.int_array(self.dims)
        nbytes = lib.rdvb_mlp_packed_bytes(len(self.layers), dims)
        if nbytes <= 0:
            return
        if self.packed is None or self.packed.numel() < nbytes:
            self.packed = torch.empty(int(nbytes), dtype=torch.uint8, device=self.dev)
        N.check(lib.rdvb_mlp_pack(len(self.layers), dims, N.ptr_array([w.data_ptr() for w in Ws]),
                                  N.ptr_array([b.data_ptr() for b in bs]), self.operand, self.packed.data_ptr(),
                                  stream_handle()), "rdvb_mlp_pack")
        self.packed_key = key


_DTYPES = {torch.float32: N.RDVB_F32, torch.float16: N.RDVB_F16, torch.bfloat16: N.RDVB_BF16}


def _compose_ops(ops):
    """Composite of the ops (applied first to last), or None if empty."""
    m = None
    for op in ops:
        m = op if m is None else Composite(op, m)
    return m


def run_chain(plan: _ChainPlan, x2d: torch.Tensor, y2d: torch.Tensor, tail_exact: bool) -> None:
    """Launches the lowered chain on [rows, IN] -> [rows, OUT] (device tensors)."""
    plan.refresh()
    rows = x2d.shape[0]
    if rows == 0:
        return
    if plan.project is not None:
        xs = x2d if x2d.dtype == torch.float32 else x2d.float()
        last = plan.prologue is None and not plan.layers and not plan.input_relu
        coords = y2d if last else torch.empty(rows, 2, dtype=torch.float32, device=x2d.device)
        plan.project._project(xs.contiguous(), coords)
        if last:
            return
        x2d = coords
    if plan.prologue is not None:
        feats = torch.empty(rows, plan.prologue.OUT, dtype=torch.float32, device=x2d.device)
        xs = x2d if x2d.dtype == torch.float32 else x2d.float()
        plan.prologue._sample(xs.contiguous(), feats if plan.layers or plan.input_relu else y2d)
        if not plan.layers and not plan.input_relu:
            return
        x2d = feats
    if not plan.layers:
        if plan.input_relu:
            N.check(N.lib().rdvb_relu(x2d.data_ptr(), y2d.data_ptr(), x2d.numel(), stream_handle()), "rdvb_relu")
        else:
            y2d.copy_(x2d)
        return
    lib = N.lib()
    n = len(plan.layers)
    rc = lib.rdvb_mlp_forward(
        x2d.data_ptr(), _DTYPES[x2d.dtype], rows, n, N.int_array(plan.dims),
        N.ptr_array([w.data_ptr() for w in plan.Ws]), N.ptr_array([b.data_ptr() for b in plan.bs]),
        N.int_array(plan.flags), int(plan.input_relu), int(tail_exact),
        plan.packed.data_ptr() if plan.packed is not None else None,
        y2d.data_ptr(), stream_handle())
    N.check(rc, "rdvb_mlp_forward")


def _device_tensor(x) -> torch.Tensor:
    return x._tensor if isinstance(x, RDVObject) else wrap(x)._tensor


def _as_rows(m: Map, xt: torch.Tensor) -> torch.Tensor:
    """xt as a contiguous [rows, IN] tensor. The tensor-core kernel reads x
    with 16-byte bulk copies; a misaligned view (a row slice such as x[1:] of
    a 3-wide fp32 tensor) is copied to an aligned buffer instead of sending
    the chain to the CUDA cores."""
    if xt.dtype not in _DTYPES:
        xt = xt.to(torch.float32)
    x2d = xt.reshape(-1, m.IN)
    if not x2d.is_contiguous() or x2d.data_ptr() % 16:
        x2d = x2d.contiguous() if not x2d.is_contiguous() else x2d.clone()
    return x2d


def _plan_of(m: Map, owner: Map, dev) -> _ChainPlan:
    plans = owner.__dict__.setdefault("_plans", {})
    pkey = (dev.index, m.IN)
    plan = plans.get(pkey)
    if plan is None:
        plan = _ChainPlan(m, dev)
        plans[pkey] = plan
    return plan


def _bound(m: Map, in_size: int) -> Map:
    b = m._bind(in_size=in_size) if m.__is_generic__ else m
    if b.__is_generic__:
        raise RuntimeError("Generic arguments could not be deduced from input data. You must explicitly cast.")
    assert in_size == b.IN, f"input's last dimension ({in_size}) must match the map's IN ({b.IN})"
    return b


def _evaluate(m: Map, owner: Map, x):
    dev = current_device()
    xt = _device_tensor(x)
    x2d = _as_rows(m, xt)
    lead = list(xt.shape[:-1])
    cache = owner.__dict__.setdefault("_out_cache", {})
    key = (dev.index, tuple(lead), m.OUT)
    out = cache.get(key)
    if out is None:
        out = RDVObject(torch.empty(lead + [m.OUT], dtype=torch.float32, device=dev))
        cache[key] = out
    plan = _plan_of(m, owner, dev)
    with _timed():
        run_chain(plan, x2d, out._tensor.view(-1, m.OUT), tail_exact=True)
    return out


def evaluate_into(m: Map, x, out: torch.Tensor) -> torch.Tensor:
    """m(x) written into `out` (a [rows, OUT] fp32 view on the current
    device, e.g. a slice of a larger buffer) instead of the map's cached
    output object; the same launches and results as ``m(x)``. Used by the
    sharded and host-streaming evaluators, which place each chunk's rows
    straight into the final buffer."""
    dev = current_device()
    xt = _device_tensor(x)
    b = _bound(m, xt.shape[-1])
    x2d = _as_rows(b, xt)
    y2d = out.view(-1, b.OUT)
    if y2d.dtype != torch.float32 or y2d.device != dev or y2d.shape[0] != x2d.shape[0]:
        raise ValueError(f"out must be a float32 [{x2d.shape[0]}, {b.OUT}] tensor on {dev}")
    plan = _plan_of(b, m, dev)
    with _timed():
        run_chain(plan, x2d, y2d, tail_exact=True)
    return out
