"""Host-side multi-rank logic (CPU, gloo, world size 2): shard ranges and the
final all-gather of row blocks. The per-rank compute here is a CPU stand-in
(an affine map on torch CPU tensors); the GPU path runs the same functions
with NCCL and the CUDA kernels (bench.py --gpus N)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from rdv_project_b200.sharding import all_gather_rows, shard_range, shard_sizes, sharded_map


def test_shard_ranges_partition():
    for n in [0, 1, 7, 64, 1000, 1080, 67_108_864]:
        for world in [1, 2, 3, 4, 8]:
            ranges = [shard_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (b0, e0), (b1, e1) in zip(ranges, ranges[1:]):
                assert e0 == b1
            sizes = shard_sizes(n, world)
            assert max(sizes) - min(sizes) <= 1 and sum(sizes) == n
    assert shard_range(1080, 8, 3) == (405, 540)
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _AffineStandIn:
    """CPU stand-in for a Map: [rows, 3] -> [rows, 4]."""

    IN, OUT = 3, 4

    def __init__(self):
        g = torch.Generator().manual_seed(5)
        self.W = torch.randn(4, 3, generator=g)
        self.b = torch.randn(4, generator=g)

    def __call__(self, x):
        return x @ self.W.T + self.b


def _worker(rank, world, port, n):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        x = torch.arange(n * 3, dtype=torch.float32).reshape(n, 3) / 7.0
        m = _AffineStandIn()
        full = sharded_map(m, x)
        torch.testing.assert_close(full, m(x))
        # the gather of bare blocks, e.g. image row bands [rows, width, 4]
        b, e = shard_range(n, world, rank)
        band = torch.full((e - b, 2, 4), float(rank))
        img = all_gather_rows(band, n)
        for r in range(world):
            rb, re = shard_range(n, world, r)
            assert torch.all(img[rb:re] == r)
        with pytest.raises(ValueError):
            all_gather_rows(torch.zeros(e - b + 1, 4), n)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [8, 7, 1])
def test_sharded_map_and_gather_gloo_world2(n):
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    mp.spawn(_worker, args=(2, _free_port(), n), nprocs=2, join=True)


def test_slab_and_piece_bounds():
    from rdv_project_b200.sharding import piece_bounds, slab_bounds

    for n in [1, 127, 128, 1000, 4096, 67_108_864]:
        for world in [1, 2, 4, 8]:
            for chunks in [1, 3, 8]:
                slabs = slab_bounds(n, world, chunks)
                assert slabs[0][0] == 0 and slabs[-1][1] == n
                assert all(e0 == b1 for (_, e0), (b1, _) in zip(slabs, slabs[1:]))
                assert len(slabs) <= chunks
                # every slab but the last is a whole number of 128-row tiles per rank
                assert all((e - b) % (world * 128) == 0 for b, e in slabs[:-1])
                covered = sorted(p for r in range(world) for p in piece_bounds(n, world, r, chunks))
                rows = [i for b, e in covered for i in (b, e)]
                assert sum(e - b for b, e in covered) == n
                assert all(e0 == b1 for (_, e0), (b1, _) in zip(covered, covered[1:]))
    assert slab_bounds(0, 2, 4) == []
    assert slab_bounds(67_108_864, 8, 8) == [(k * 8_388_608, (k + 1) * 8_388_608) for k in range(8)]


def _overlapped_worker(rank, world, port, n, chunks):
    import torch.distributed as dist

    from rdv_project_b200.sharding import piece_bounds, sharded_map_overlapped

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        x = torch.arange(n * 3, dtype=torch.float32).reshape(n, 3) / 7.0
        m = _AffineStandIn()
        calls = []

        def evaluate(xs, ys):
            calls.append(xs.shape[0])
            ys.copy_(m(xs))

        want = m(x)
        out = torch.full((n, 4), float("nan"))
        sharded_map_overlapped(m, x, out=out, chunks=chunks, evaluate=evaluate, align=4)
        torch.testing.assert_close(out, want)
        mine = piece_bounds(n, world, rank, chunks, align=4)
        assert sum(calls) == sum(e - b for b, e in mine)  # a rank evaluates only its pieces
        # host-streamed input and this rank's rows copied back
        out2 = torch.full((n, 4), float("nan"))
        y_host = torch.full((n, 4), float("nan"))
        sharded_map_overlapped(m, x_host=x, y_host=y_host, out=out2, chunks=chunks, evaluate=evaluate, align=4)
        torch.testing.assert_close(out2, want)
        for b, e in mine:
            torch.testing.assert_close(y_host[b:e], want[b:e])
        # shard=False: the whole batch is this process's, no exchange
        out3 = torch.full((n, 4), float("nan"))
        calls.clear()
        sharded_map_overlapped(m, x, out=out3, chunks=chunks, evaluate=evaluate, align=4, shard=False)
        torch.testing.assert_close(out3, want)
        assert sum(calls) == n
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n,chunks", [(64, 4), (61, 3), (9, 8), (1, 2)])
def test_sharded_map_overlapped_gloo_world2(n, chunks):
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    mp.spawn(_overlapped_worker, args=(2, _free_port(), n, chunks), nprocs=2, join=True)


def test_sharded_map_overlapped_single_process():
    from rdv_project_b200.sharding import sharded_map_overlapped

    m = _AffineStandIn()
    x = torch.randn(50, 3)
    out = torch.empty(50, 4)
    sharded_map_overlapped(m, x, out=out, chunks=3, evaluate=lambda xs, ys: ys.copy_(m(xs)), align=8)
    torch.testing.assert_close(out, m(x))
    with pytest.raises(ValueError):
        sharded_map_overlapped(m, x, out=torch.empty(49, 4), evaluate=lambda xs, ys: None)
    with pytest.raises(ValueError):
        sharded_map_overlapped(m, None, out=out)
