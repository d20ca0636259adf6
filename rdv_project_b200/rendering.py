"""Camera rays and the MLP volume ray-march.

* ``Cameras(width, height, poses, aspect_ratio=None, fov=None, jitter=False)``
  mirrors the reference's pinhole ray grid (rdv/domain/rendering.py:10-42,
  rdv/shaders/rendering/cameras.h:1-20): ``poses`` is ``[num_cameras, 9]``
  (origin | target | up); calling it returns ``[num_cameras, height, width,
  6]`` float32 (origin, unit direction) -> rdvb_camera_rays. With
  ``jitter=True`` every pixel's ray passes through a random point of the
  pixel instead of its centre: the first two draws of the pixel's own
  generator (the reference's Taus + LCG, started from the call's seeds
  spawned by the flat pixel index) -> rdvb_camera_rays_jittered. Each call
  draws fresh seeds, as the reference does per dispatch; ``cameras(seeds=...)``
  fixes them.
* ``VolumeRenderer(mlp, n_samples=128)`` renders the BASELINE volume
  workload: rays of a pinhole camera clipped to the reference's implicit
  [-1, 1]^3 box (rdv/shaders/libraries/math_library.h:48-57), 128 midpoint
  samples per ray, the composed ``LinearFast`` MLP (3 -> ... -> 4) evaluated
  per sample, softplus density, sigmoid colour, front-to-back alpha
  compositing -> RGBA ``[rows, width, 4]`` float32 (black background,
  A = 1 - transmittance). One fused tensor-core kernel per call
  (rdvb_raymarch_render); ``row_begin``/``row_end`` render a band of rows, the
  unit the multi-GPU path shards.
"""
from __future__ import annotations

import math

import torch

from . import _native as N
from .core import RDVObject, _timed, current_device, stream_handle, wrap
from .maps import Map, XRProject, _ChainPlan, dir2xr


class Cameras:
    """Pinhole ray generator over [num_cameras, height, width] pixels."""

    def __init__(self, width: int, height: int, poses, aspect_ratio: float | None = None, fov: float | None = None,
                 jitter: bool = False) -> None:
        if aspect_ratio is None:
            aspect_ratio = width / height
        if fov is None:
            fov = math.pi / 4
        if not isinstance(poses, RDVObject):
            poses = wrap(poses)
        assert poses.shape[1] == 9, "poses must be a [num_cameras, 9] tensor (ori | target | up)"
        self.shape = [poses.shape[0], height, width]
        self.width, self.height = width, height
        self.poses = poses
        self.aspect_ratio = aspect_ratio
        self.fov = fov
        self.pixel_jitter = 1 if jitter else 0
        self.last_seeds = None

    def __rshift__(self, m):
        """Camera grid composed with a Map[6, k] (e.g. RaymarchingTransmittance)."""
        return _CameraGrid(self, m)

    def __call__(self, seeds=None) -> RDVObject:
        dev = current_device()
        poses = self.poses._tensor.to(device=dev, dtype=torch.float32).contiguous()
        out = torch.empty(self.shape + [6], dtype=torch.float32, device=dev)
        with _timed():
            if self.pixel_jitter:
                from .volumes import _draw_seeds

                seeds = _draw_seeds() if seeds is None else tuple(int(v) for v in seeds)
                assert len(seeds) == 4, "seeds must be 4 integers"
                self.last_seeds = seeds
                N.check(N.lib().rdvb_camera_rays_jittered(
                    poses.data_ptr(), self.shape[0], self.width, self.height, float(self.aspect_ratio),
                    float(self.fov), N.uint32_array(seeds), out.data_ptr(), stream_handle()),
                    "rdvb_camera_rays_jittered")
            else:
                N.check(N.lib().rdvb_camera_rays(poses.data_ptr(), self.shape[0], self.width, self.height,
                                                 float(self.aspect_ratio), float(self.fov), out.data_ptr(),
                                                 stream_handle()), "rdvb_camera_rays")
        return RDVObject(out)


class _CameraGrid:
    """``cameras >> m``: m evaluated on every ray of the grid ->
    ``[num_cameras, height, width, m.OUT]``."""

    def __init__(self, cameras: Cameras, m) -> None:
        assert m.IN is None or m.IN == 6, "a camera grid produces 6 values per ray (origin, direction)"
        self.cameras = cameras
        self.map = m

    def __call__(self, seeds=None) -> RDVObject:
        """One dispatch of the composition. A node that draws random numbers
        (RatiotrackingTransmittance) continues each pixel's generator after
        the camera's draws, as the reference's single per-thread state does
        (RatiotrackingTransmittance, PBVR):
        the same seeds, 2 draws already taken when the camera jitters."""
        from .volumes import _draw_seeds

        if getattr(self.map, "_draws_random", False):
            seeds = _draw_seeds() if seeds is None else tuple(int(v) for v in seeds)
            rays = self.cameras(seeds=seeds) if self.cameras.pixel_jitter else self.cameras()
            return self.map(rays, seeds=seeds, draws_before=2 if self.cameras.pixel_jitter else 0)
        rays = self.cameras(seeds=seeds) if self.cameras.pixel_jitter else self.cameras()
        return self.map(rays)


class VolumeRenderer:
    """Emission-absorption volume render of an MLP density/colour field over
    the [-1, 1]^3 box (see the module docstring)."""

    def __init__(self, mlp: Map, n_samples: int = 128) -> None:
        assert mlp.IN == 3 and mlp.OUT == 4, "the MLP must map positions (3) to (density, r, g, b) (4)"
        assert n_samples == 128, "n_samples must be 128 (one tensor-core tile per ray)"
        self.mlp = mlp
        self.n_samples = n_samples
        self._plans = {}
        self._ws = {}

    def _plan(self, dev):
        plan = self._plans.get(dev.index)
        if plan is None:
            plan = _ChainPlan(self.mlp, dev)
            if plan.operand is None or plan.input_relu:
                raise NotImplementedError("the ray-march MLP must be a LinearFast (or LinearFastBF16) chain")
            self._plans[dev.index] = plan
        plan.refresh()
        if plan.packed is None:
            raise NotImplementedError("the MLP does not fit the tensor-core kernel (widths <= 128, <= 16 layers)")
        return plan

    def render(self, pose9, width: int, height: int, fov: float | None = None, aspect_ratio: float | None = None,
               row_begin: int = 0, row_end: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        dev = current_device()
        row_end = height if row_end is None else row_end
        plan = self._plan(dev)
        pose = [float(v) for v in torch.as_tensor(pose9, dtype=torch.float32).reshape(-1).tolist()]
        assert len(pose) == 9, "pose9 must hold origin | target | up"
        rows = row_end - row_begin
        if out is None:
            out = torch.empty((rows, width, 4), dtype=torch.float32, device=dev)
        assert out.shape == (rows, width, 4) and out.dtype == torch.float32 and out.is_contiguous()
        lib = N.lib()
        need = int(lib.rdvb_raymarch_workspace_bytes(width, height))
        ws = self._ws.get(dev.index)
        if ws is None or ws.numel() < need:
            ws = torch.empty(need, dtype=torch.uint8, device=dev)
            self._ws[dev.index] = ws
        with _timed():
            N.check(lib.rdvb_raymarch_render(
                N.float_array(pose), width, height, float(fov) if fov else 0.0,
                float(aspect_ratio) if aspect_ratio else 0.0, self.n_samples, len(plan.layers),
                N.int_array(plan.dims), N.int_array(plan.flags), plan.packed.data_ptr(), row_begin, row_end,
                ws.data_ptr(), ws.numel(), out.data_ptr(), stream_handle()), "rdvb_raymarch_render")
        return out
