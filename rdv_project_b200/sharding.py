"""Multi-GPU sharding of the hot path: one process per GPU, the batch (MLP
rows, image row bands) split into contiguous ranges, each rank computing its
range with no cross-rank traffic, and one all-gather of the results (NCCL
over NVLink, the copy engines, or NVLink multicast stores on GPUs; gloo in
the CPU tests).

The reference has no multi-device execution at all; this is the B200
scale-out of its data-parallel operators. Kernels read only local tensors.

``sharded_map_p2p`` does the exchange without NCCL: the output buffers
(``PeerBuffer``) are mapped into every rank's process, and each rank copies
the rows it computed into all of them with the copy engines over NVLink,
slab by slab, while the next slab's kernel runs on every SM; a one-element
all-reduce orders the step. ``sharded_map_nvls`` sends each rank's rows once,
through the NVLink switch: a small copy kernel stores them to the multicast
address of a symmetric buffer (``MulticastBuffer``) and the switch delivers
them to every rank.

``sharded_map_overlapped`` is the pipelined library-collective form: the
rows are cut into slabs, every slab is split evenly over the ranks, and the
NCCL all-gather of slab k runs (on NCCL's stream) while slab k + 1
computes. Given pinned host buffers it also streams its input in and its
rows out on copy streams, overlapping PCIe with the kernels.
"""
from __future__ import annotations

import ctypes

import torch


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of `rank`'s contiguous share of n units: the first
    n % world ranks get one unit more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    if n < 0:
        raise ValueError("n must be >= 0")
    base, extra = divmod(n, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def shard_sizes(n: int, world: int) -> list[int]:
    return [shard_range(n, world, r)[1] - shard_range(n, world, r)[0] for r in range(world)]


def all_gather_rows(local: torch.Tensor, n: int, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Concatenates every rank's `local` block (rank order, leading dimension
    = its shard of n rows) into an [n, ...] tensor on every rank, with one
    all_gather_into_tensor. Unequal shards are padded to the largest and
    trimmed."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sizes = shard_sizes(n, world)
    if local.shape[0] != sizes[rank]:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its shard of {n} is {sizes[rank]}")
    tail = tuple(local.shape[1:])
    m = max(sizes) if sizes else 0
    if all(s == m for s in sizes):
        if out is None:
            out = torch.empty((n,) + tail, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    padded = torch.zeros((m,) + tail, dtype=local.dtype, device=local.device)
    padded[:local.shape[0]] = local
    full = torch.empty((m * world,) + tail, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(full, padded, group=group)
    if out is None:
        out = torch.empty((n,) + tail, dtype=local.dtype, device=local.device)
    for r, s in enumerate(sizes):
        b, _ = shard_range(n, world, r)
        out[b:b + s] = full[r * m:r * m + s]
    return out


def sharded_map(m, x: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Evaluates Map `m` on this rank's rows of x ([n, IN], the full batch or
    any tensor indexable by row) and all-gathers [n, OUT] on every rank."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = x.shape[0]
    b, e = shard_range(n, world, rank)
    local = m(x[b:e])
    local = local.as_tensor("torch") if hasattr(local, "as_tensor") else local
    return all_gather_rows(local, n, group=group, out=out)


def sharded_render(renderer, pose9, width: int, height: int, group=None, **kw) -> torch.Tensor:
    """Renders this rank's band of image rows with a VolumeRenderer and
    all-gathers the [height, width, 4] RGBA image on every rank."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    b, e = shard_range(height, world, rank)
    band = renderer.render(pose9, width, height, row_begin=b, row_end=e, **kw)
    return all_gather_rows(band, height, group=group)


# ------------------------------------------------------------ overlapped form
def slab_bounds(n: int, world: int, chunks: int, align: int = 128) -> list[tuple[int, int]]:
    """[begin, end) global row ranges of the slabs of a pipelined sharded
    map: `chunks` slabs (fewer when n is small) whose size is a multiple of
    world * align, so that every rank's piece of every slab but the last is
    the same whole number of `align`-row tiles."""
    if n < 0 or world < 1 or chunks < 1 or align < 1:
        raise ValueError("n >= 0, world >= 1, chunks >= 1 and align >= 1 are required")
    if n == 0:
        return []
    unit = world * align
    size = -(-n // chunks)
    size = -(-size // unit) * unit
    return [(b, min(n, b + size)) for b in range(0, n, size)]


def piece_bounds(n: int, world: int, rank: int, chunks: int, align: int = 128) -> list[tuple[int, int]]:
    """The global row ranges rank `rank` computes: its shard_range share of
    every slab."""
    out = []
    for b, e in slab_bounds(n, world, chunks, align):
        pb, pe = shard_range(e - b, world, rank)
        out.append((b + pb, b + pe))
    return out


class _Ring:
    """Device staging buffers (two, reused call after call) for pieces of a
    host input, cached per (device, dtype, columns, rows)."""

    _cache: dict = {}

    @classmethod
    def get(cls, dev, dtype, cols, rows):
        key = (str(dev), dtype, cols, rows)
        bufs = cls._cache.get(key)
        if bufs is None:
            bufs = [torch.empty(rows, cols, dtype=dtype, device=dev) for _ in range(2)]
            cls._cache[key] = bufs
        return bufs


def _rank_world(group):
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def sharded_map_overlapped(m, x: torch.Tensor | None = None, *, group=None, out: torch.Tensor | None = None,
                           chunks: int = 8, x_host: torch.Tensor | None = None,
                           y_host: torch.Tensor | None = None, evaluate=None, reserve_ctas: int = 0,
                           align: int = 128, shard: bool = True) -> torch.Tensor:
    """Map `m` over n rows, split over the ranks of `group` (or this process
    alone when no process group is initialised), every rank ending with the
    full [n, OUT] result in `out`.

    The rows are cut into `chunks` slabs (``slab_bounds``); each rank
    evaluates its piece of slab k straight into `out` at the piece's global
    rows, then starts an in-place all-gather of slab k (async, NCCL stream),
    so the exchange of slab k overlaps the kernel of slab k + 1.

    Input: `x`, the full [n, IN] batch on the device (a rank reads only its
    pieces), or `x_host`, the full batch in (pinned) host memory: each rank
    then copies its pieces in on a copy stream, one piece ahead of the
    kernels, through two device staging buffers. `y_host` (pinned host
    [n, OUT]), if given, receives the rows this rank computed, copied back on
    a second copy stream as each piece finishes -- the union over ranks is
    the whole result.

    `reserve_ctas` leaves that many SMs free of the persistent MLP kernel
    while the call runs (``rdvb_set_max_ctas``), so the all-gather's NCCL
    kernels, which cannot share an SM with it, start at once.

    `evaluate(x_piece, y_piece)` replaces the map evaluation (it must write
    y_piece from x_piece); by default it is ``maps.evaluate_into(m, ...)``.
    With ``shard=False`` the whole batch is this process's own (no split, no
    exchange): the host-streaming pipeline alone.
    """
    import torch.distributed as dist

    rank, world = _rank_world(group) if shard else (0, 1)
    src = x if x is not None else x_host
    if src is None:
        raise ValueError("give x (device) or x_host (host) input rows")
    n = src.shape[0]
    if out is None:
        raise ValueError("out ([n, OUT] on this rank's device) is required")
    if out.shape[0] != n:
        raise ValueError(f"out has {out.shape[0]} rows, the input {n}")
    if y_host is not None and y_host.shape[0] != n:
        raise ValueError(f"y_host has {y_host.shape[0]} rows, the input {n}")
    if evaluate is None:
        from .maps import evaluate_into

        def evaluate(xs, ys):
            evaluate_into(m, xs, ys)

    cuda = out.device.type == "cuda"
    slabs = slab_bounds(n, world, chunks, align)
    pieces = piece_bounds(n, world, rank, chunks, align)
    comp = torch.cuda.current_stream(out.device) if cuda else None
    h2d = d2h = None
    ring = None
    free_ev = [None, None]
    if x_host is not None and x is None:
        rows_max = max((e - b for b, e in pieces), default=0)
        if cuda:
            h2d = torch.cuda.Stream(out.device)
            ring = _Ring.get(out.device, x_host.dtype, x_host.shape[1], max(rows_max, 1))
    if y_host is not None and cuda:
        d2h = torch.cuda.Stream(out.device)
    prev_cap = None
    if cuda and reserve_ctas > 0 and world > 1:
        from . import _native as N

        sms = torch.cuda.get_device_properties(out.device).multi_processor_count
        prev_cap = N.set_max_ctas(max(1, sms - reserve_ctas))
    works = []
    try:
        for k, ((sb, se), (pb, pe)) in enumerate(zip(slabs, pieces)):
            rows = pe - pb
            # ---- input piece
            if x is not None:
                xs = x[pb:pe]
            elif cuda:
                buf = ring[k % 2][:rows]
                with torch.cuda.stream(h2d):
                    if free_ev[k % 2] is not None:
                        h2d.wait_event(free_ev[k % 2])
                    buf.copy_(x_host[pb:pe], non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(h2d)
                comp.wait_event(ready)
                xs = buf
            else:
                xs = x_host[pb:pe]
            # ---- kernel: the piece's rows straight into `out`
            if rows:
                evaluate(xs, out[pb:pe])
            if cuda:
                done = torch.cuda.Event()
                done.record(comp)
                if ring is not None:
                    free_ev[k % 2] = done
                if d2h is not None and rows:
                    d2h.wait_event(done)
                    with torch.cuda.stream(d2h):
                        y_host[pb:pe].copy_(out[pb:pe], non_blocking=True)
            elif y_host is not None and rows:
                y_host[pb:pe].copy_(out[pb:pe])
            # ---- exchange of the slab, in place
            if world > 1:
                if (se - sb) % world == 0:
                    works.append(dist.all_gather_into_tensor(out[sb:se], out[pb:pe], group=group, async_op=True))
                else:
                    # ragged last slab: padded all-gather (pieces differ by a row)
                    local = out[pb:pe].clone()
                    all_gather_rows(local, se - sb, group=group, out=out[sb:se])
    finally:
        if prev_cap is not None:
            from . import _native as N

            N.set_max_ctas(prev_cap)
    for w in works:
        w.wait()
    if cuda:
        if d2h is not None:
            comp.wait_stream(d2h)
        if h2d is not None:
            comp.wait_stream(h2d)
    return out


class _DeviceArray:
    """A raw device allocation seen as an array (__cuda_array_interface__),
    so torch.as_tensor wraps it without a copy."""

    def __init__(self, ptr: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


class PeerBuffer:
    """An [n, cols] fp32 buffer on every rank of `group`, each rank's buffer
    mapped into every other rank's process (CUDA IPC over NVLink), so a
    rank can copy rows straight into all of them: the output of
    ``sharded_map_p2p``. Collective to create (every rank of the group
    calls it with the same n and cols); ``close()`` (also collective) unmaps
    and frees.

    ``tensor``: this rank's buffer as a torch tensor; ``peer_ptrs``: the
    device addresses of the other ranks' buffers in this process, in rank
    order without this rank."""

    def __init__(self, n: int, cols: int, group=None):
        import torch.distributed as dist

        from . import _native as N

        self.group = group
        self.rank, self.world = _rank_world(group)
        if self.world - 1 > N.RDVB_MAX_PEERS:
            raise ValueError(f"at most {N.RDVB_MAX_PEERS + 1} ranks share a PeerBuffer, got {self.world}")
        self.n, self.cols = int(n), int(cols)
        lib = N.lib()
        nbytes = max(1, self.n * self.cols) * 4
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * N.RDVB_IPC_HANDLE_BYTES)()
        N.check(lib.rdvb_ipc_alloc(nbytes, ctypes.byref(ptr), handle), "rdvb_ipc_alloc")
        self._ptr = int(ptr.value)
        self._opened = []
        self.tensor = torch.as_tensor(_DeviceArray(self._ptr, (self.n, self.cols)), device="cuda")
        mine = bytes(handle)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, mine, group=group)
        else:
            handles = [mine]
        self.peer_ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                continue
            hb = (ctypes.c_ubyte * N.RDVB_IPC_HANDLE_BYTES).from_buffer_copy(h)
            pp = ctypes.c_void_p()
            N.check(lib.rdvb_ipc_open(hb, ctypes.byref(pp)), "rdvb_ipc_open")
            self._opened.append(int(pp.value))
            self.peer_ptrs.append(int(pp.value))

    def rows_of_peers(self, begin: int) -> list[int]:
        """The peers' addresses of row `begin` (same offset as in this rank's buffer)."""
        off = int(begin) * self.cols * 4
        return [p + off for p in self.peer_ptrs]

    def close(self) -> None:
        """Collective: every rank unmaps the others' buffers, waits for the
        group, then frees its own."""
        import torch.distributed as dist

        from . import _native as N

        if self._ptr is None:
            return
        torch.cuda.synchronize()
        for p in self._opened:
            N.check(N.lib().rdvb_ipc_close(p), "rdvb_ipc_close")
        self._opened = []
        self.peer_ptrs = []
        if self.world > 1:
            dist.barrier(group=self.group)
        self.tensor = None
        N.check(N.lib().rdvb_ipc_free(self._ptr), "rdvb_ipc_free")
        self._ptr = None


def sharded_map_p2p(m, x: torch.Tensor, buf: PeerBuffer, group=None, chunks: int = 8, align: int = 128,
                    evaluate=None, copy_streams: int = 7) -> torch.Tensor:
    """Map `m` over the n rows of `x` (the full batch on this rank's device;
    a rank reads only its rows), split over the ranks of `group`, every rank
    ending with the full [n, OUT] result in ``buf.tensor``.

    The rows are cut into `chunks` slabs (``slab_bounds``). Each rank
    evaluates its piece of slab k into its own buffer with every SM, then
    copies those rows into every peer's buffer on a copy stream
    (``rdvb_peer_copy``: one cudaMemcpyAsync per peer, the copy engines over
    NVLink into memory the peers mapped to this process) while slab k + 1
    computes. A one-element all-reduce on the compute stream, after the last
    copy, orders the step: no rank reads another rank's rows before they
    landed. Unlike an NCCL all-gather this takes no SM from the kernels.
    `evaluate(x_piece, y_piece)` replaces the map evaluation (default
    ``maps.evaluate_into``). The peers are split over `copy_streams` side
    streams (at most one per peer)."""
    import torch.distributed as dist

    from . import _native as N

    if evaluate is None:
        from .maps import evaluate_into

        def evaluate(xs, ys):
            evaluate_into(m, xs, ys)

    rank, world = _rank_world(group)
    n = x.shape[0]
    if buf.n != n:
        raise ValueError(f"the buffer holds {buf.n} rows, the input {n}")
    out = buf.tensor
    comp = torch.cuda.current_stream(out.device)
    # the peers split over several copy streams, so several copy engines
    # send at once (one stream would queue the copies to 7 peers)
    n_cs = max(1, min(len(buf.peer_ptrs), copy_streams)) if buf.peer_ptrs else 0
    streams = _copy_streams(out.device, n_cs)
    row_bytes = buf.cols * 4
    for pb, pe in piece_bounds(n, world, rank, chunks, align):
        if pe <= pb:
            continue
        evaluate(x[pb:pe], out[pb:pe])
        if streams:
            done = torch.cuda.Event()
            done.record(comp)
            peers = buf.rows_of_peers(pb)
            for j, cs in enumerate(streams):
                mine = peers[j::n_cs]
                cs.wait_event(done)
                N.check(N.lib().rdvb_peer_copy(out[pb:pe].data_ptr(), N.ptr_array(mine), len(mine),
                                               (pe - pb) * row_bytes, cs.cuda_stream), "rdvb_peer_copy")
    for cs in streams:
        comp.wait_stream(cs)
    if world > 1:
        dist.all_reduce(_barrier_flag(out.device), group=group)
    return out


_streams: dict = {}


def _copy_streams(dev, k: int) -> list:
    """k side streams of `dev` (created once, reused)."""
    have = _streams.setdefault(str(dev), [])
    while len(have) < k:
        have.append(torch.cuda.Stream(dev))
    return have[:k]


_flags: dict = {}


def _barrier_flag(dev) -> torch.Tensor:
    t = _flags.get(str(dev))
    if t is None:
        t = torch.zeros(1, dtype=torch.float32, device=dev)
        _flags[str(dev)] = t
    return t


class MulticastBuffer:
    """An [n, cols] fp32 buffer on every rank of `group`, allocated as torch
    symmetric memory and bound to an NVLink multicast (NVLS) object: a store
    to ``mc_ptr`` + offset reaches every rank's buffer through the switch.
    Collective to create and to ``close()``, in an initialised process group
    (NCCL). Raises RuntimeError where the GPUs offer no multicast."""

    def __init__(self, n: int, cols: int, group=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.group = group if group is not None else dist.group.WORLD
        self.rank, self.world = _rank_world(group)
        self.n, self.cols = int(n), int(cols)
        if self.cols % 4:
            raise ValueError("the multicast exchange moves 16-byte chunks: cols must be a multiple of 4")
        full = symm.empty(max(1, self.n), self.cols, dtype=torch.float32, device="cuda")
        self.handle = symm.rendezvous(full, self.group)
        self.tensor = full[: self.n]
        mc = int(self.handle.multicast_ptr or 0)
        if not mc:
            self.close()
            raise RuntimeError("these GPUs offer no NVLink multicast (NVLS) for symmetric memory")
        # the tensor's place in the symmetric allocation, in the multicast mapping
        self.mc_ptr = mc + (self.tensor.data_ptr() - int(self.handle.buffer_ptrs[self.rank]))

    def close(self) -> None:
        """Collective: every rank waits for the group, then drops the buffer."""
        import torch.distributed as dist

        if self.tensor is None:
            return
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        self.handle = None
        self.tensor = None


def sharded_map_nvls(m, x: torch.Tensor, buf: MulticastBuffer, group=None, chunks: int = 8, align: int = 128,
                     reserve_ctas: int = 32, evaluate=None) -> torch.Tensor:
    """``sharded_map_p2p`` with the exchange through the NVLink switch: after
    each piece's kernel, a copy kernel of `reserve_ctas` CTAs (the MLP kernel
    leaves that many SMs free, ``rdvb_set_max_ctas``) writes the piece's rows
    once to the buffer's multicast address (``rdvb_multicast_copy``,
    multimem.st) and the switch delivers them to every rank, while the next
    piece computes. A one-element all-reduce then orders the step."""
    import torch.distributed as dist

    from . import _native as N

    if evaluate is None:
        from .maps import evaluate_into

        def evaluate(xs, ys):
            evaluate_into(m, xs, ys)

    rank, world = _rank_world(group)
    n = x.shape[0]
    if buf.n != n:
        raise ValueError(f"the buffer holds {buf.n} rows, the input {n}")
    out = buf.tensor
    comp = torch.cuda.current_stream(out.device)
    cs = _copy_streams(out.device, 1)[0] if world > 1 else None
    row_bytes = buf.cols * 4
    prev_cap = None
    if cs is not None and reserve_ctas > 0:
        sms = torch.cuda.get_device_properties(out.device).multi_processor_count
        prev_cap = N.set_max_ctas(max(1, sms - reserve_ctas))
    try:
        for pb, pe in piece_bounds(n, world, rank, chunks, align):
            if pe <= pb:
                continue
            evaluate(x[pb:pe], out[pb:pe])
            if cs is not None:
                done = torch.cuda.Event()
                done.record(comp)
                cs.wait_event(done)
                N.check(N.lib().rdvb_multicast_copy(out[pb:pe].data_ptr(), buf.mc_ptr + pb * row_bytes,
                                                    (pe - pb) * row_bytes, max(1, reserve_ctas), cs.cuda_stream),
                        "rdvb_multicast_copy")
    finally:
        if prev_cap is not None:
            N.set_max_ctas(prev_cap)
    if cs is not None:
        comp.wait_stream(cs)
        dist.all_reduce(_barrier_flag(out.device), group=group)
    return out
