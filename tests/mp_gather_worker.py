"""One rank of the peer-copy gather check (launched by tests/test_gpu_multi.py
under torchrun, one process per GPU). Every rank maps every other rank's
output buffer (PeerBuffer) and evaluates its pieces of the slabs, copying
each piece into every peer's buffer with the copy engines
(sharding.sharded_map_p2p); the gathered result must equal, bit for bit, the
same pieces evaluated and gathered by NCCL (sharding.sharded_map_overlapped),
and agree with the oracle on sampled rows. Where the GPUs offer NVLink
multicast, the exchange through the switch (sharding.sharded_map_nvls) must
equal it too. Rank 0 prints one JSON line."""
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

CASES = [
    # dims, math, rows: the config-5 architecture with a ragged last slab and
    # a partial 32-row group; a bfloat16 chain; an fp32 chain (CUDA cores)
    ([3, 64, 64, 64, 64, 4], "f16", 1_000_003),
    ([4, 32, 16], "bf16", 4099),
    ([3, 16, 5], "f32", 777),
]


def build(rdv, dims, math, dev, seed):
    g = torch.Generator().manual_seed(seed)
    cls = {"f32": rdv.Linear, "f16": rdv.LinearFast, "bf16": rdv.LinearFastBF16}[math]
    m, layers = None, []
    for i in range(len(dims) - 1):
        W = torch.randn(dims[i + 1], dims[i], generator=g) * (2.0 / dims[i]) ** 0.5
        b = torch.randn(dims[i + 1], generator=g) * 0.1
        relu = i < len(dims) - 2
        layers.append({"W": W.numpy(), "b": b.numpy(), "math": math, "relu": relu})
        f = cls(W.to(dev), b.to(dev))
        m = f if m is None else m >> f
        if relu:
            m = m >> rdv.relu
    return m, layers


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    import rdv_project_b200 as rdv
    from oracle import mlp as omlp
    from rdv_project_b200.sharding import MulticastBuffer, PeerBuffer, sharded_map_nvls, sharded_map_overlapped, \
        sharded_map_p2p

    out = []
    for ci, (dims, math, n) in enumerate(CASES):
        m, layers = build(rdv, dims, math, dev, seed=11 + ci)
        x = (torch.rand(n, dims[0], generator=torch.Generator().manual_seed(ci)) * 2 - 1).to(dev)
        buf = PeerBuffer(n, dims[-1])
        got = []
        for _ in range(2):  # the buffer reused
            buf.tensor.fill_(float("nan"))
            dist.barrier()
            sharded_map_p2p(m, x, buf, chunks=4)
            torch.cuda.synchronize()
            got.append(buf.tensor.clone())
        ref = torch.empty(n, dims[-1], device=dev)
        sharded_map_overlapped(m, x, out=ref, chunks=4)
        torch.cuda.synchronize()
        sel = np.arange(0, n, max(1, n // 2000))
        nw, el = omlp.rel_errors(got[0][torch.from_numpy(sel).to(dev)].cpu().numpy(),
                                 omlp.mlp_forward(x.cpu().numpy()[sel], layers, tail_exact=True))
        rec = {"dims": dims, "math": math, "rows": n, "equal_nccl": bool(torch.equal(got[0], ref)),
               "equal_again": bool(torch.equal(got[0], got[1])), "finite": bool(torch.isfinite(got[0]).all()),
               "normwise": float(nw), "elementwise": float(el), "status": int(rdv.device_status())}
        buf.close()
        if dims[-1] % 4 == 0:
            # the same through the NVLink switch (multimem.st), where the GPUs offer multicast
            try:
                mb = MulticastBuffer(n, dims[-1])
            except RuntimeError:
                mb = None
            if mb is not None:
                mb.tensor.fill_(float("nan"))
                dist.barrier()
                sharded_map_nvls(m, x, mb, chunks=4, reserve_ctas=16)
                torch.cuda.synchronize()
                rec["nvls_equal_nccl"] = bool(torch.equal(mb.tensor, ref))
                rec["status"] = max(rec["status"], int(rdv.device_status()))
                mb.close()
        out.append(rec)
    if rank == 0:
        print(json.dumps({"world": world, "cases": out}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
