"""Multi-GPU checks that need two or more GPUs on one node (skipped
otherwise): the NCCL-free exchange (each rank's rows copied by the copy
engines into every rank's IPC-mapped buffer, sharding.sharded_map_p2p)
against the same slab pieces gathered by NCCL, bit for bit, and against the
oracle."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_copy_gather_matches_nccl_gather():
    world = min(torch.cuda.device_count(), 8)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "mp_gather_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=420, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    line = [l for l in res.stdout.splitlines() if l.startswith("{")][-1]
    rep = json.loads(line)
    assert rep["world"] == world
    for c in rep["cases"]:
        assert c["equal_nccl"] and c["equal_again"] and c["finite"], c
        assert c.get("nvls_equal_nccl", True), c
        assert c["status"] == 0, c
        tol = 1e-5 if c["math"] == "f32" else 1e-2
        assert c["normwise"] <= tol and c["elementwise"] <= tol, c


def test_single_rank_peer_buffer_and_peer_copy(cuda_device):
    """One process: PeerBuffer allocates through rdvb_ipc_alloc (no peers to
    map), sharded_map_p2p over one rank equals the map itself bit for bit,
    and rdvb_peer_copy sends a buffer to two destinations."""
    import rdv_project_b200 as rdv
    import rdv_project_b200._native as N
    from rdv_project_b200.sharding import PeerBuffer, sharded_map_p2p

    g = torch.Generator().manual_seed(4)
    dims = [3, 64, 64, 4]
    m = None
    for i in range(3):
        f = rdv.LinearFast((torch.randn(dims[i + 1], dims[i], generator=g) * 0.5).to(cuda_device),
                           (torch.randn(dims[i + 1], generator=g) * 0.1).to(cuda_device))
        m = f if m is None else m >> f
        if i < 2:
            m = m >> rdv.relu
    n = 100_003
    x = (torch.rand(n, 3, generator=g) * 2 - 1).to(cuda_device)
    buf = PeerBuffer(n, 4)
    assert buf.peer_ptrs == [] and tuple(buf.tensor.shape) == (n, 4)
    sharded_map_p2p(m, x, buf, chunks=3)
    want = m(rdv.wrap(x)).as_tensor("torch")
    assert torch.equal(buf.tensor, want)
    a, b = torch.empty_like(want), torch.empty_like(want)
    N.check(N.lib().rdvb_peer_copy(buf.tensor.data_ptr(), N.ptr_array([a.data_ptr(), b.data_ptr()]), 2,
                                   want.numel() * 4, torch.cuda.current_stream().cuda_stream), "rdvb_peer_copy")
    torch.cuda.synchronize()
    assert torch.equal(a, want) and torch.equal(b, want)
    buf.close()
    assert rdv.device_status() == 0
