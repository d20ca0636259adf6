"""Volume nodes of the hot path.

``RaymarchingTransmittance(extinction, transform=None, step_size=0.002,
density_scale=1.0)`` mirrors rdv/domain/volumes.py:124-141: a ``Map[6, 1]``
from a ray (origin, direction) to the transmittance of the fixed-step
absorption march through the node's [-1, 1]^3 box
(rdv/shaders/volumes/raymarching_transmittance.h:1-21,
raymarching_transmittance_trait.h:1-14). ``extinction`` is a ``Map[3, 1]``
(the reference casts it so, volumes.py:16) built from ``Linear`` /
``LinearFast`` / ``ReLU``; ``transform`` is the node's ``mat4x3`` (four
columns: the 3x3 part, then the origin; default identity). Calling the node on
rays ``[..., 6]`` returns ``[..., 1]`` float32 (rdvb_transmittance_rm): exact
fp32 chains march one ray per CUDA thread like the reference's loop;
float16 / bfloat16 (LinearFast) chains evaluate the steps in 128-step chunks
with the fused tensor-core MLP kernel.

``RatiotrackingTransmittance(extinction, majorant, transform=None,
density_scale=1.0)`` mirrors rdv/domain/volumes.py:144-170: the same
``Map[6, 1]`` estimated by majorant-based ratio tracking with Russian
roulette (rdv/shaders/volumes/ratiotracking_transmittance.h and
ratiotracking_transmittance_trait.h), one CUDA thread per ray
(rdvb_transmittance_rt). ``majorant`` is a ``VoxelMajorantField`` (or, as
in the reference's ``_as_majorant_field``, a bare ``TensorGrid`` / tensor
``[D, H, W, 1]`` wrapped as one). Each call draws fresh generator seeds, as
the reference does per dispatch; ``node(rays, seeds=(s0, s1, s2, s3))``
fixes them for a reproducible estimate.

``Cameras(...) >> node`` composes a camera grid with either node; calling the
composition returns ``[num_cameras, height, width, 1]``.
"""
from __future__ import annotations

import ctypes
import random as _random

import torch

from . import _native as N
from .core import RDVObject, _timed, current_device, stream_handle, wrap
from .maps import Composite, Constant, GridSampler, Map, TensorSampler, XRProject, _lower

_IDENTITY = (1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0)


def _mat4x3(transform) -> tuple:
    """12 floats, column-major (the reference's mat4x3 constructor order)."""
    if transform is None:
        return _IDENTITY
    t = torch.as_tensor(transform, dtype=torch.float64).detach().cpu()
    if t.shape == (4, 3):      # four columns of vec3
        t = t.reshape(-1)
    assert t.numel() == 12, "transform must be a mat4x3 (12 values, column-major)"
    return tuple(float(v) for v in t.reshape(-1))


def _split_encoding(extinction: Map):
    """(leading TensorSampler / GridSampler of a 3-D grid or None, the rest
    of the chain or None): the sampler becomes the kernels' input encoding."""
    ops = extinction._ops()
    if ops and isinstance(ops[0], (TensorSampler, GridSampler)):
        smp = ops[0]
        assert smp.IN == 3, "a volume's extinction encoding samples a 3-D grid"
        rest = None
        for op in ops[1:]:
            rest = op if rest is None else Composite(op, rest)
        return smp, rest
    return None, extinction


def _encoding(smp, dev):
    """rdvb_encoding of a sampler (its grid kept alive on the struct)."""
    t = smp.t._tensor
    if t.device != dev or t.dtype != torch.float32 or not t.is_contiguous():
        t = t.to(device=dev, dtype=torch.float32).contiguous()
    e = N.Encoding()
    e.kind = N.RDVB_ENCODING_GRID_SAMPLER if isinstance(smp, GridSampler) else N.RDVB_ENCODING_TENSOR_SAMPLER
    e.grid = t.data_ptr()
    for k in range(3):
        e.dims[k] = int(t.shape[k])
    e.features = int(t.shape[3])
    e.flags = ((N.RDVB_SAMPLER_CLAMP if smp.clamp else 0) | (N.RDVB_SAMPLER_ALIGNED if smp.aligned else 0) |
               (N.RDVB_SAMPLER_LINEAR if smp.linear else 0))
    e._keep = t
    return e


def _enc_arg(st):
    return ctypes.byref(st["enc"]) if st["enc"] is not None else None


class RaymarchingTransmittance(Map):
    """Map[6, 1]: ray -> transmittance through the extinction field."""

    IN = 6
    OUT = 1

    def __init__(self, extinction: Map, transform=None, step_size: float = 0.002, density_scale: float = 1.0):
        ext = extinction
        if ext.__is_generic__:
            ext = ext._bind(in_size=3, out_size=1)
        assert ext.IN == 3 and ext.OUT == 1, "extinction must be a Map[3, 1]"
        self.extinction = ext
        self.step_size = float(step_size)
        self.transform = _mat4x3(transform)
        self.density_scale = float(density_scale)
        self._state = {}

    def _ops(self):
        raise NotImplementedError("RaymarchingTransmittance is evaluated by its own kernel, not a fused MLP chain")

    def _device_state(self, dev):
        st = self._state.get(dev.index)
        if st is None:
            sampler, rest = _split_encoding(self.extinction)
            input_relu, layers, relus = _lower(rest) if rest is not None else (False, [], [])
            if not layers and sampler is None:
                raise NotImplementedError("the extinction needs at least one Linear layer or a sampler")
            if sampler is not None and not layers:
                assert sampler.OUT == 1, "a sampler alone as the extinction must have OUT = 1"
            st = {
                "input_relu": int(input_relu),
                "layers": layers,
                "dims": [sampler.OUT if sampler is not None else 3] + [l.OUT for l in layers],
                "flags": [l._math | (N.RDVB_LAYER_RELU if r else 0) for l, r in zip(layers, relus)],
                "sampler": sampler,
                "ws": None,
            }
            self._state[dev.index] = st
        st["W"] = [l._fp32(l.weight, dev) for l in st["layers"]]
        st["b"] = [l._fp32(l.bias, dev) for l in st["layers"]]
        st["enc"] = _encoding(st["sampler"], dev) if st["sampler"] is not None else None
        return st

    def __call__(self, rays):
        dev = current_device()
        rt = rays._tensor if isinstance(rays, RDVObject) else wrap(rays)._tensor
        assert rt.shape[-1] == 6, f"input's last dimension ({rt.shape[-1]}) must match the map's IN (6)"
        lead = list(rt.shape[:-1])
        r2 = rt.reshape(-1, 6)
        if r2.device != dev or r2.dtype != torch.float32 or not r2.is_contiguous():
            r2 = r2.to(device=dev, dtype=torch.float32).contiguous()
        out = torch.empty(lead + [1], dtype=torch.float32, device=dev)
        st = self._device_state(dev)
        n = len(st["layers"])
        need = int(N.lib().rdvb_transmittance_workspace_bytes(r2.shape[0], n, N.int_array(st["dims"]),
                                                              N.int_array(st["flags"])))
        if st["ws"] is None or st["ws"].numel() < need:
            st["ws"] = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
        with _timed():
            N.check(N.lib().rdvb_transmittance_rm(
                r2.data_ptr(), r2.shape[0], N.float_array(self.transform), self.step_size, self.density_scale,
                _enc_arg(st), n,
                N.int_array(st["dims"]), N.ptr_array([w.data_ptr() for w in st["W"]]),
                N.ptr_array([b.data_ptr() for b in st["b"]]), N.int_array(st["flags"]), st["input_relu"],
                st["ws"].data_ptr(), st["ws"].numel(), out.data_ptr(), stream_handle()), "rdvb_transmittance_rm")
        return RDVObject(out)

    def last_evaluations(self) -> int:
        """Extinction evaluations (march steps) of the last call on this
        device; synchronises with it."""
        st = self._state.get(current_device().index)
        if st is None or st["ws"] is None:
            return 0
        return int(st["ws"][8:16].view(torch.int64).item())


class TensorGrid:
    """Grid[IN, OUT] over a tensor whose last dimension is OUT (the
    reference's TensorGrid, rdv/maths/__init__.py:487-505; IN = ndim - 1,
    addressed row-major, rdv/shaders/grids/tensor_grid.h)."""

    def __init__(self, data):
        t = data._tensor if isinstance(data, RDVObject) else torch.as_tensor(data)
        assert t.dim() >= 2, "a TensorGrid needs at least one index dimension and the OUT dimension"
        self.data = t
        self.IN = t.dim() - 1
        self.OUT = t.shape[-1]
        self.shape = list(t.shape[:-1])


class VoxelMajorantField:
    """Map[6, 2] (rdv/domain/volumes.py:196-212,
    rdv/shaders/volumes/voxel_majorant_field.h): for an object-space
    position and direction, the majorant of the voxel holding the position
    and the distance along the direction to that voxel's exit. ``grid`` is a
    Grid[3, 1] over [-1, 1]^3: a TensorGrid, or its tensor [D, H, W, 1]."""

    def __init__(self, grid):
        if not isinstance(grid, TensorGrid):
            grid = TensorGrid(grid)
        assert grid.IN == 3 and grid.OUT == 1, "the majorant grid must be a Grid[3, 1]"
        self.grid = grid


class SphereMajorantField:
    """Map[6, 2] (rdv/domain/volumes.py:215-224,
    rdv/shaders/volumes/sphere_majorant_field.h): ``grid`` is a Grid[3, 2]
    over [-1, 1]^3 holding per voxel (majorant, radius), the radius a
    half-width in voxels of the box around the voxel's centre that the
    majorant bounds. For an object-space position and direction: the
    majorant of the voxel holding the position and the distance along the
    direction to that box's exit (at least 1e-6), so one free flight may
    cross many voxels. A TensorGrid, or its tensor [D, H, W, 2]."""

    def __init__(self, grid):
        if not isinstance(grid, TensorGrid):
            grid = TensorGrid(grid)
        assert grid.IN == 3 and grid.OUT == 2, "the sphere majorant grid must be a Grid[3, 2]"
        self.grid = grid


def _as_majorant_field(majorant):
    """volumes.py:227-242: a field as given, a Grid[3, 1] wrapped as a voxel field."""
    if isinstance(majorant, (VoxelMajorantField, SphereMajorantField)):
        return majorant
    if isinstance(majorant, (TensorGrid, torch.Tensor, RDVObject)):
        return VoxelMajorantField(majorant)
    raise NotImplementedError("majorant must be a VoxelMajorantField, a SphereMajorantField or a Grid[3, 1]")


def _field_args(field, dev):
    """(device grid, [D, H, W], RDVB_MAJORANT_*) of a majorant field."""
    g = field.grid.data
    if g.device != dev or g.dtype != torch.float32 or not g.is_contiguous():
        g = g.to(device=dev, dtype=torch.float32).contiguous()
    kind = N.RDVB_MAJORANT_SPHERE if isinstance(field, SphereMajorantField) else N.RDVB_MAJORANT_VOXEL
    return g, list(g.shape[:3]), kind


def _draw_seeds():
    """Per-dispatch seeds as the reference draws them: 4 integers in
    [128, 2^30) (core/_common.py:66-75)."""
    return tuple(_random.randint(128, (1 << 30) - 1) for _ in range(4))


class RatiotrackingTransmittance(RaymarchingTransmittance):
    """Map[6, 1]: ray -> ratio-tracking estimate of the transmittance."""

    _draws_random = True

    def __init__(self, extinction: Map, majorant, transform=None, density_scale: float = 1.0):
        super().__init__(extinction, transform=transform, density_scale=density_scale)
        del self.step_size
        self.majorant = _as_majorant_field(majorant)
        self.last_seeds = None

    def __call__(self, rays, seeds=None, draws_before: int = 0):
        dev = current_device()
        rt = rays._tensor if isinstance(rays, RDVObject) else wrap(rays)._tensor
        assert rt.shape[-1] == 6, f"input's last dimension ({rt.shape[-1]}) must match the map's IN (6)"
        lead = list(rt.shape[:-1])
        r2 = rt.reshape(-1, 6)
        if r2.device != dev or r2.dtype != torch.float32 or not r2.is_contiguous():
            r2 = r2.to(device=dev, dtype=torch.float32).contiguous()
        out = torch.empty(lead + [1], dtype=torch.float32, device=dev)
        st = self._device_state(dev)
        g, gdims, kind = _field_args(self.majorant, dev)
        seeds = _draw_seeds() if seeds is None else tuple(int(v) for v in seeds)
        assert len(seeds) == 4, "seeds must be 4 integers"
        self.last_seeds = seeds
        if st["ws"] is None:
            st["ws"] = torch.empty(256, dtype=torch.uint8, device=dev)
        n = len(st["layers"])
        with _timed():
            N.check(N.lib().rdvb_transmittance_rt(
                r2.data_ptr(), r2.shape[0], N.float_array(self.transform), self.density_scale, g.data_ptr(),
                N.int_array(gdims), kind, N.uint32_array(seeds), int(draws_before), _enc_arg(st), n,
                N.int_array(st["dims"]),
                N.ptr_array([w.data_ptr() for w in st["W"]]), N.ptr_array([b.data_ptr() for b in st["b"]]),
                N.int_array(st["flags"]), st["input_relu"], st["ws"].data_ptr(), st["ws"].numel(), out.data_ptr(),
                stream_handle()), "rdvb_transmittance_rt")
        return RDVObject(out)


def _environment_args(env, dev):
    """(RDVB_ENV_*, rgb, image, [H, W], sampler flags) of a PBVR
    environment: a Constant of 3 values, or XRProject() >> TensorSampler of
    a [H, W, 3] image."""
    if isinstance(env, Constant):
        assert env.OUT == 3, "a constant environment holds 3 values (RGB)"
        return N.RDVB_ENV_CONSTANT, [float(v) for v in env.data.tolist()], None, [0, 0], 0
    if isinstance(env, Composite) and isinstance(env.g, XRProject) and isinstance(env.f, TensorSampler):
        smp = env.f
        assert smp.IN == 2 and smp.OUT == 3, "the environment image must be [H, W, 3]"
        img = smp.t._tensor
        if img.device != dev or img.dtype != torch.float32 or not img.is_contiguous():
            img = img.to(device=dev, dtype=torch.float32).contiguous()
        flags = ((N.RDVB_SAMPLER_CLAMP if smp.clamp else 0) | (N.RDVB_SAMPLER_ALIGNED if smp.aligned else 0) |
                 (N.RDVB_SAMPLER_LINEAR if smp.linear else 0))
        return N.RDVB_ENV_EQUIRECT, [0.0, 0.0, 0.0], img, list(img.shape[:2]), flags
    raise NotImplementedError("the environment must be a Constant[3, 3] or XRProject() >> TensorSampler(image)")


class PBVR(RaymarchingTransmittance):
    """Map[6, 3]: ray -> one unbiased delta-tracking sample of the radiance
    along it (rdv/domain/volumes.py:257-326, rdv/shaders/volumes/pbvr.h);
    averaged over dispatches it converges to the volume's rendering.

    ``extinction`` is a Map[3, 1] in the [-1, 1]^3 box (Linear / LinearFast
    / ReLU chain); ``environment`` a Map[3, 3] from a world direction to RGB
    radiance: ``Constant((r, g, b))`` or ``XRProject() >> TensorSampler(image
    [H, W, 3])``; ``majorant`` a VoxelMajorantField, a SphereMajorantField,
    or a bare Grid[3, 1] wrapped as a voxel field; ``transform`` the node's
    mat4x3; ``albedo`` (RGB) and ``g`` (Henyey-Greenstein anisotropy) are
    uniform; ``max_bounces`` bounds the real scattering events of a path.
    The extinction is used unscaled (PBVR has no density scale). Each call
    draws fresh generator seeds, as the reference does per dispatch;
    ``node(rays, seeds=...)`` fixes them (rdvb_pbvr)."""

    OUT = 3
    _draws_random = True

    def __init__(self, extinction: Map, environment: Map, majorant, transform=None, albedo=(1.0, 1.0, 1.0),
                 g: float = 0.0, max_bounces: int = 32) -> None:
        super().__init__(extinction, transform=transform)
        del self.step_size, self.density_scale
        env = environment
        if env.__is_generic__:
            env = env._bind(in_size=3, out_size=3)
        assert env.IN == 3 and env.OUT == 3, "environment must be a Map[3, 3]"
        self.environment = env
        self.majorant = _as_majorant_field(majorant)
        a = torch.as_tensor(albedo, dtype=torch.float32).reshape(-1)
        assert a.numel() == 3, "albedo must hold 3 values"
        self.albedo = tuple(float(v) for v in a)
        self.g = float(g)
        self.max_bounces = int(max_bounces)
        self.last_seeds = None

    def __call__(self, rays, seeds=None, draws_before: int = 0):
        dev = current_device()
        rt = rays._tensor if isinstance(rays, RDVObject) else wrap(rays)._tensor
        assert rt.shape[-1] == 6, f"input's last dimension ({rt.shape[-1]}) must match the map's IN (6)"
        lead = list(rt.shape[:-1])
        r2 = rt.reshape(-1, 6)
        if r2.device != dev or r2.dtype != torch.float32 or not r2.is_contiguous():
            r2 = r2.to(device=dev, dtype=torch.float32).contiguous()
        out = torch.empty(lead + [3], dtype=torch.float32, device=dev)
        st = self._device_state(dev)
        g, gdims, kind = _field_args(self.majorant, dev)
        env_kind, env_rgb, env_img, env_dims, env_flags = _environment_args(self.environment, dev)
        seeds = _draw_seeds() if seeds is None else tuple(int(v) for v in seeds)
        assert len(seeds) == 4, "seeds must be 4 integers"
        self.last_seeds = seeds
        if st["ws"] is None:
            st["ws"] = torch.empty(256, dtype=torch.uint8, device=dev)
        n = len(st["layers"])
        with _timed():
            N.check(N.lib().rdvb_pbvr(
                r2.data_ptr(), r2.shape[0], N.float_array(self.transform), g.data_ptr(), N.int_array(gdims), kind,
                N.float_array(self.albedo), self.g, self.max_bounces, env_kind, N.float_array(env_rgb),
                env_img.data_ptr() if env_img is not None else None, N.int_array(env_dims), env_flags,
                N.uint32_array(seeds), int(draws_before), _enc_arg(st), n, N.int_array(st["dims"]),
                N.ptr_array([w.data_ptr() for w in st["W"]]), N.ptr_array([b.data_ptr() for b in st["b"]]),
                N.int_array(st["flags"]), st["input_relu"], st["ws"].data_ptr(), st["ws"].numel(), out.data_ptr(),
                stream_handle()), "rdvb_pbvr")
        return RDVObject(out)


def _albedo_of(scattering_albedo):
    """The 3 values of a uniform scattering albedo: a Constant[3, 3] map (the
    form this library evaluates), or 3 numbers."""
    if isinstance(scattering_albedo, Constant):
        assert scattering_albedo.OUT == 3, "the scattering albedo must hold 3 values (RGB)"
        return tuple(float(v) for v in scattering_albedo.data.tolist())
    if isinstance(scattering_albedo, Map):
        raise NotImplementedError("the scattering albedo must be a Constant (a spatially uniform albedo)")
    a = torch.as_tensor(scattering_albedo, dtype=torch.float32).reshape(-1)
    assert a.numel() == 3, "the scattering albedo must hold 3 values (RGB)"
    return tuple(float(v) for v in a)


class _PBVRLight(RaymarchingTransmittance):
    """Shared part of PBVRT and PBVR_NEE (rdvb_pbvrt)."""

    _draws_random = True
    _variant = None

    def __init__(self, extinction, majorant, scattering_albedo, transform, light_direction, density_scale, g,
                 max_bounces, environment=None, light_intensity=None):
        super().__init__(extinction, transform=transform, density_scale=density_scale)
        del self.step_size
        self.majorant = _as_majorant_field(majorant)
        self.albedo = _albedo_of(scattering_albedo)
        ld = torch.as_tensor(light_direction, dtype=torch.float32).reshape(-1)
        assert ld.numel() == 3, "light_direction must hold 3 values"
        self.light_direction = tuple(float(v) for v in ld)
        self.light_intensity = (1.0, 1.0, 1.0) if light_intensity is None else \
            tuple(float(v) for v in torch.as_tensor(light_intensity, dtype=torch.float32).reshape(-1))
        assert len(self.light_intensity) == 3, "light_intensity must hold 3 values"
        self.environment = environment
        if environment is not None:
            env = environment._bind(in_size=3, out_size=3) if environment.__is_generic__ else environment
            assert env.IN == 3 and env.OUT == 3, "environment must be a Map[3, 3]"
            self.environment = env
        self.g = float(g)
        self.max_bounces = int(max_bounces)
        self.last_seeds = None

    def __call__(self, rays, seeds=None, draws_before: int = 0):
        dev = current_device()
        rt = rays._tensor if isinstance(rays, RDVObject) else wrap(rays)._tensor
        assert rt.shape[-1] == 6, f"input's last dimension ({rt.shape[-1]}) must match the map's IN (6)"
        lead = list(rt.shape[:-1])
        r2 = rt.reshape(-1, 6)
        if r2.device != dev or r2.dtype != torch.float32 or not r2.is_contiguous():
            r2 = r2.to(device=dev, dtype=torch.float32).contiguous()
        out = torch.empty(lead + [self.OUT], dtype=torch.float32, device=dev)
        st = self._device_state(dev)
        g, gdims, kind = _field_args(self.majorant, dev)
        if self.environment is not None:
            env_kind, env_rgb, env_img, env_dims, env_flags = _environment_args(self.environment, dev)
        else:
            env_kind, env_rgb, env_img, env_dims, env_flags = N.RDVB_ENV_CONSTANT, [0.0, 0.0, 0.0], None, [0, 0], 0
        dens, levels = None, 0
        sampler = getattr(self, "environment_sampler", None)
        if sampler is not None:
            dens, levels = sampler.densities, sampler.levels
            if dens.device != dev:
                dens = dens.to(dev)
        seeds = _draw_seeds() if seeds is None else tuple(int(v) for v in seeds)
        assert len(seeds) == 4, "seeds must be 4 integers"
        self.last_seeds = seeds
        if st["ws"] is None:
            st["ws"] = torch.empty(256, dtype=torch.uint8, device=dev)
        n = len(st["layers"])
        with _timed():
            N.check(N.lib().rdvb_pbvrt(
                r2.data_ptr(), r2.shape[0], N.float_array(self.transform), self.density_scale, g.data_ptr(),
                N.int_array(gdims), kind, N.float_array(self.albedo), self.g, self.max_bounces,
                N.float_array(self.light_direction), N.float_array(self.light_intensity), self._variant, env_kind,
                N.float_array(env_rgb), env_img.data_ptr() if env_img is not None else None, N.int_array(env_dims),
                env_flags, dens.data_ptr() if dens is not None else None, levels, N.uint32_array(seeds),
                int(draws_before), _enc_arg(st), n, N.int_array(st["dims"]),
                N.ptr_array([w.data_ptr() for w in st["W"]]), N.ptr_array([b.data_ptr() for b in st["b"]]),
                N.int_array(st["flags"]), st["input_relu"], st["ws"].data_ptr(), st["ws"].numel(), out.data_ptr(),
                stream_handle()), "rdvb_pbvrt")
        return RDVObject(out)


class PBVRT(_PBVRLight):
    """Map[6, 4]: ray -> one sample of (RGB radiance, alpha) by delta
    tracking with next-event estimation toward a directional light
    (rdv/domain/volumes.py:326-387, rdv/shaders/volumes/pbvrt.h). alpha is 1
    while the ray has not scattered (fully background, for compositing over
    a backdrop rendered elsewhere), 0 once it has; then RGB is the NEE sum
    times ``light_intensity`` plus the throughput times ``environment`` in
    the escape direction. ``extinction`` a Map[3, 1] chain, ``majorant`` a
    voxel or sphere majorant field (or a bare Grid[3, 1]), ``environment``
    a Map[3, 3] (``Constant`` or ``XRProject() >> TensorSampler(image)``),
    ``scattering_albedo`` a ``Constant`` of 3 values (or 3 numbers),
    ``light_direction`` normalized here, ``density_scale`` scales the
    extinction and the majorant, ``g`` the Henyey-Greenstein anisotropy,
    ``max_bounces`` the real scattering events (rdvb_pbvrt)."""

    OUT = 4
    _variant = N.RDVB_PBVRT

    def __init__(self, extinction: Map, majorant, environment: Map, scattering_albedo, transform=None,
                 light_direction=(0.0, 1.0, 0.0), light_intensity=None, density_scale: float = 1.0, g: float = 0.0,
                 max_bounces: int = 32) -> None:
        super().__init__(extinction, majorant, scattering_albedo, transform, light_direction, density_scale, g,
                         max_bounces, environment=environment, light_intensity=light_intensity)


class PBVR_NEE(_PBVRLight):
    """Map[6, 3]: ray -> the next-event-estimation part of delta tracking
    toward a directional light (rdv/domain/volumes.py:390-442,
    rdv/shaders/volumes/pbvr_nee.h): the sum over real collisions of
    throughput * shadow transmittance * phase; no environment, no light
    intensity, no alpha. Arguments as PBVRT (rdvb_pbvrt)."""

    OUT = 3
    _variant = N.RDVB_PBVR_NEE

    def __init__(self, extinction: Map, majorant, scattering_albedo, transform=None,
                 light_direction=(0.0, 1.0, 0.0), density_scale: float = 1.0, g: float = 0.0,
                 max_bounces: int = 32) -> None:
        super().__init__(extinction, majorant, scattering_albedo, transform, light_direction, density_scale, g,
                         max_bounces)


def _xr_quadtree(image: torch.Tensor, levels: int) -> torch.Tensor:
    """The XREnvironmentSampler's quadtree (the layout of
    rdv/domain/rendering.py:175-278): the image resampled to 2^levels x
    2^levels cell centres by the GridSampler (clamp, not aligned, linear,
    rdvb_grid_sampler), its channels summed, each row weighted by the solid
    angle sin(beta1) - sin(beta0) of its band of the equirectangular
    parametrisation, normalised to 1; then per depth d and node (Morton
    order: child c = 2 row bit + column bit, node 4 n + 1 + c) the
    cumulative probabilities of its 4 children (0.25 each under an empty
    parent), the last forced to 1. Returns a flat fp32 tensor of
    4 (4^levels - 1) / 3 values on the image's device."""
    assert 1 <= levels <= 12, "levels must be in [1, 12]"
    dev = image.device
    res = 1 << levels
    idx = torch.arange(res, dtype=torch.float32, device=dev)
    c = (idx + 0.5) / res * 2 - 1                         # RegularGrid cell centres (mode 1)
    yy, xx = torch.meshgrid(c, c, indexing="ij")
    pts = torch.stack([xx, yy], -1).reshape(-1, 2).contiguous()
    img = image.to(torch.float32).contiguous()
    resized = torch.empty(res * res, img.shape[-1], dtype=torch.float32, device=dev)
    GridSampler(img, clamp=True, aligned=False, linear=True)._sample(pts, resized)
    resized = resized.reshape(res, res, -1).cpu()
    dens = resized[..., 0].clone()
    for k in range(1, resized.shape[-1]):
        dens = dens + resized[..., k]
    dens = dens.clamp_min(0)
    v0 = torch.arange(res, dtype=torch.float32) / res
    v1 = (torch.arange(res, dtype=torch.float32) + 1) / res
    half_pi = torch.tensor(3.14159265358979 / 2, dtype=torch.float32)
    w_row = torch.sin((v1 * 2 - 1) * half_pi) - torch.sin((v0 * 2 - 1) * half_pi)
    dens = (dens * w_row[:, None]).clamp_min(0)
    dens = dens / dens.sum().clamp_min(1e-12)
    pyramid = [dens]
    for _ in range(levels):
        g = pyramid[-1]
        pyramid.append(g.reshape(g.shape[0] // 2, 2, g.shape[1] // 2, 2).sum(dim=(1, 3)))
    pyramid.reverse()                                     # pyramid[d]: 2^d x 2^d

    def morton(t, d):
        if d == 0:
            return t.reshape(1)
        bits = t.reshape([2] * (2 * d))                   # row bits, then column bits (MSB first)
        order = [a for i in range(d) for a in (i, d + i)]
        return bits.permute(order).reshape(-1)

    parts = []
    for d in range(levels):
        parent = morton(pyramid[d], d)
        kids = morton(pyramid[d + 1], d + 1).reshape(-1, 4)
        p = torch.where(parent[:, None] > 1e-12, kids / parent.clamp_min(1e-12)[:, None],
                        torch.full_like(kids, 0.25))
        cum = torch.cumsum(p, dim=1)
        cum[:, 3] = 1.0
        parts.append(cum.reshape(-1))
    return torch.cat(parts).to(dev).contiguous()


class XREnvironmentSampler:
    """Map[6, 3 + 3 + 1] (rdv/domain/rendering.py:281-323,
    rdv/shaders/rendering/xr_environment_sampler.h): importance-samples a
    world direction from an equirectangular environment by a quadtree of
    its solid-angle-weighted pixel densities (built once here from
    ``image``); returns the direction, the environment there divided by the
    pdf, and the pdf. ``environment`` is the Map[3, 3] looked up at the
    sampled direction (``XRProject() >> TensorSampler(image)`` or a
    ``Constant``); ``image`` [H, W, C] the data the densities come from.
    Evaluated inside PBVR_ENV's kernel."""

    IN = 6
    OUT = 7

    def __init__(self, environment: Map, image, levels: int = 8) -> None:
        env = environment._bind(in_size=3, out_size=3) if environment.__is_generic__ else environment
        assert env.IN == 3 and env.OUT == 3, "environment must be a Map[3, 3]"
        self.environment = env
        self.levels = int(levels)
        img = image._tensor if isinstance(image, RDVObject) else torch.as_tensor(image)
        if img.device.type != "cuda":
            img = img.to(current_device())
        self.densities = _xr_quadtree(img, self.levels)


class PBVR_ENV(_PBVRLight):
    """Map[6, 3]: ray -> the next-event-estimation sum of delta tracking
    where each real collision's NEE direction is importance-sampled from the
    environment (rdv/domain/volumes.py:445-502,
    rdv/shaders/volumes/pbvr_env.h): throughput * shadow transmittance *
    phase * environment / pdf. ``environment_sampler`` an
    ``XREnvironmentSampler``; other arguments as PBVR_NEE (rdvb_pbvrt)."""

    OUT = 3
    _variant = N.RDVB_PBVR_ENV

    def __init__(self, extinction: Map, majorant, scattering_albedo, environment_sampler, transform=None,
                 density_scale: float = 1.0, g: float = 0.0, max_bounces: int = 32) -> None:
        assert isinstance(environment_sampler, XREnvironmentSampler), \
            "environment_sampler must be an XREnvironmentSampler"
        super().__init__(extinction, majorant, scattering_albedo, transform, (0.0, 1.0, 0.0), density_scale, g,
                         max_bounces, environment=environment_sampler.environment)
        self.environment_sampler = environment_sampler
