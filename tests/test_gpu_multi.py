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
        assert c["status"] == 0, c
        tol = 1e-5 if c["math"] == "f32" else 1e-2
        assert c["normwise"] <= tol and c["elementwise"] <= tol, c
