"""evaluate_chain() over LinearTensorOp* / ReLUTensorOp pipelines
(rdv/maths/__init__.py:1369-1379): runs of ops that feed only one another
run as one fused kernel launch, and must give bit for bit the results of
dispatching the ops one by one (the eager dispatch every op does at
construction). Ops inside a fused run materialise on first use."""
import numpy as np
import pytest
import torch

from oracle import mlp as omlp

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rdv():
    import rdv_project_b200 as rdv
    return rdv


def _w(out_f, in_f, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(out_f, in_f, generator=g) * (2.0 / in_f) ** 0.5, torch.randn(out_f, generator=g) * 0.1


def _pipeline(rdv, x, dev, kinds):
    """x -> kinds[0] -> ReLU -> kinds[1] -> ReLU -> kinds[2]; widths 32 -> 64 -> 64 -> 16."""
    dims = [32, 64, 64, 16]
    ops = []
    cur = x
    for i, cls in enumerate(kinds):
        W, b = _w(dims[i + 1], dims[i], 100 + i)
        cur = getattr(rdv, cls)(cur, W.to(dev), b.to(dev))
        ops.append(cur)
        if i < len(kinds) - 1:
            cur = rdv.ReLUTensorOp(cur)
            ops.append(cur)
    return ops


@pytest.mark.parametrize("kinds", [("LinearTensorOpFast", "LinearTensorOpSmall", "LinearTensorOpMine"),
                                   ("LinearTensorOp", "LinearTensorOp", "LinearTensorOp"),
                                   ("LinearTensorOpSimple", "LinearTensorOpFast", "LinearTensorOpSmall")])
def test_fused_chain_equals_per_op_dispatch(rdv, cuda_device, kinds):
    g = torch.Generator().manual_seed(0)
    x = (torch.randn(4096, 32, generator=g)).to(cuda_device)
    ops = _pipeline(rdv, x, cuda_device, kinds)
    final = ops[-1]
    # in-place edit of the leaf, then the fused re-evaluation
    x.mul_(0.5).add_(0.25)
    final.evaluate_chain()
    assert all(op._stale for op in ops[:-1]) and not final._stale
    got = final.as_type("torch").clone()
    # reference: a fresh pipeline on the edited input, dispatched op by op
    ref_ops = _pipeline(rdv, x.clone(), cuda_device, kinds)
    torch.cuda.synchronize()
    assert torch.equal(got, ref_ops[-1].as_type("torch"))
    # the stale intermediates materialise on use, with the per-op values
    for op, ref in zip(ops[:-1], ref_ops[:-1]):
        assert torch.equal(op.as_type("torch"), ref.as_type("torch"))
        assert not op._stale
    # and the fused result meets the oracle (each op's own arithmetic:
    # float16 staging for the coopmat ops, with the bias first for Small and
    # Simple; exact fp32 for LinearTensorOp)
    dims = [32, 64, 64, 16]
    layers = []
    for i, cls in enumerate(kinds):
        W, b = _w(dims[i + 1], dims[i], 100 + i)
        layers.append({"W": W.numpy(), "b": b.numpy(), "math": "f32" if cls == "LinearTensorOp" else "f16",
                       "relu": i < len(kinds) - 1, "bias_first": cls in ("LinearTensorOpSmall", "LinearTensorOpSimple")})
    ref = omlp.mlp_forward(x.cpu().numpy(), layers)
    tol = 1e-5 if all(k == "LinearTensorOp" for k in kinds) else 2e-3
    nw, el = omlp.rel_errors(got.cpu().numpy(), ref)
    assert nw <= tol and el <= tol, (nw, el)


def test_mixed_precision_pipeline_is_not_fused_across_arithmetics(rdv, cuda_device):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2048, 32, generator=g).to(cuda_device)
    kinds = ("LinearTensorOp", "LinearTensorOpFast", "LinearTensorOp")
    ops = _pipeline(rdv, x, cuda_device, kinds)
    x.mul_(-1.0)
    ops[-1].evaluate_chain()
    ref_ops = _pipeline(rdv, x.clone(), cuda_device, kinds)
    torch.cuda.synchronize()
    assert torch.equal(ops[-1].as_type("torch"), ref_ops[-1].as_type("torch"))
    for op, ref in zip(ops, ref_ops):
        assert torch.equal(op.result.as_tensor("torch"), ref.result.as_tensor("torch"))


def test_branch_point_is_materialised_and_downstream_evaluate_sees_fresh_inputs(rdv, cuda_device):
    g = torch.Generator().manual_seed(2)
    x = torch.randn(1024, 32, generator=g).to(cuda_device)
    W1, b1 = _w(64, 32, 7)
    W2, b2 = _w(16, 64, 8)
    W3, b3 = _w(32, 64, 9)
    a = rdv.LinearTensorOpFast(x, W1.to(cuda_device), b1.to(cuda_device))
    r = rdv.ReLUTensorOp(a)
    left = rdv.LinearTensorOpSmall(r, W2.to(cuda_device), b2.to(cuda_device))
    right = rdv.LinearTensorOpSmall(r, W3.to(cuda_device), b3.to(cuda_device))  # second consumer of r
    x.add_(1.0)
    # `right` is not part of left's chain: a, r, left run fused, r is left stale
    left.evaluate_chain()
    assert r._stale and not left._stale
    right.evaluate()       # materialises r first, then reads its fresh result
    assert not r._stale
    ref_a = rdv.LinearTensorOpFast(x.clone(), W1.to(cuda_device), b1.to(cuda_device))
    ref_r = rdv.ReLUTensorOp(ref_a)
    ref_left = rdv.LinearTensorOpSmall(ref_r, W2.to(cuda_device), b2.to(cuda_device))
    ref_right = rdv.LinearTensorOpSmall(ref_r, W3.to(cuda_device), b3.to(cuda_device))
    torch.cuda.synchronize()
    assert torch.equal(left.as_type("torch"), ref_left.as_type("torch"))
    assert torch.equal(right.as_type("torch"), ref_right.as_type("torch"))
    # a stale op read through a downstream evaluate(): materialised first
    a2 = rdv.LinearTensorOpFast(x, W1.to(cuda_device), b1.to(cuda_device))
    r2 = rdv.ReLUTensorOp(a2)
    l2 = rdv.LinearTensorOpSmall(r2, W2.to(cuda_device), b2.to(cuda_device))
    x.mul_(2.0)
    l2.evaluate_chain()
    assert a2._stale and r2._stale
    extra = rdv.LinearTensorOpSmall(r2, W3.to(cuda_device), b3.to(cuda_device))  # uses r2.result -> materialised
    assert not r2._stale
    ref2 = rdv.LinearTensorOpSmall(rdv.ReLUTensorOp(rdv.LinearTensorOpFast(x.clone(), W1.to(cuda_device),
                                                                             b1.to(cuda_device))),
                                   W3.to(cuda_device), b3.to(cuda_device))
    torch.cuda.synchronize()
    assert torch.equal(extra.as_type("torch"), ref2.as_type("torch"))
