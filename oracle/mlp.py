"""MLP-chain oracle (test infrastructure only).

Restates the reference's fused Map chain ``linear(W, b, f16) >> relu >> ...``
(rdv/domain/nn.py:99-104 builds Linear or LinearFast; rdv/maths/__init__.py
Map.__rshift__ :1489-1498 composes them; each layer's arithmetic is in
rdv/shaders/maps/linear.h:28-31 (exact fp32) and
rdv/shaders/maps/linear_fast.h:61-98 (float16 operands, fp32 accumulate,
bias added after)). A trailing partial 32-row workgroup runs exact fp32
(linear_fast.h:44,102-108 via cooperative_library.h:20-33).

Layer description used throughout: a list of dicts
``{"W": [out, in] float32, "b": [out] float32, "math": "f32"|"f16"|"bf16",
"relu": bool}``, optionally ``"bias_first": True`` for the float16 layers of
LinearTensorOpSmall / LinearTensorOpSimple, whose accumulators start from
the bias (rdv/shaders/tensors/linear_tensor_op_small.h:99).
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from ._clib import oracle_lib, ptr, ptr_array

MATH_CODES = {"f32": 0, "f16": 1, "bf16": 2}
FLAG_RELU = 4
FLAG_BIAS_FIRST = 8


def layer_flags(layers) -> np.ndarray:
    return np.array([MATH_CODES[l["math"]] | (FLAG_RELU if l["relu"] else 0)
                     | (FLAG_BIAS_FIRST if l.get("bias_first") else 0) for l in layers], dtype=np.int32)


def mlp_forward(x: np.ndarray, layers, input_relu: bool = False, tail_exact: bool = False,
                threads: int | None = None) -> np.ndarray:
    """Row-by-row C restatement (oracle/c/oracle.c): sequential fp32
    accumulation, float16/bfloat16 staging per layer. Rows are split across
    threads; each thread runs the single-threaded C routine on its slice."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[0]
    dims = np.array([layers[0]["W"].shape[1]] + [l["W"].shape[0] for l in layers], dtype=np.int32)
    assert x.shape[1] == dims[0]
    Ws = [np.ascontiguousarray(l["W"], dtype=np.float32) for l in layers]
    bs = [np.ascontiguousarray(l["b"], dtype=np.float32) for l in layers]
    flags = layer_flags(layers)
    y = np.empty((n, int(dims[-1])), dtype=np.float32)
    lib = oracle_lib()
    wp, bp = ptr_array(Ws), ptr_array(bs)
    threads = threads or max(1, min(os.cpu_count() or 1, 32))
    # The 32-row workgroup fallback depends on the global row index, so
    # every slice boundary is a multiple of 32 and the tail rule is applied
    # only in the slice that holds the trailing partial workgroup.
    n_full = (n // 32) * 32 if tail_exact else n
    bounds = []
    step = max(32, ((n // threads) + 31) // 32 * 32)
    for s in range(0, n, step):
        bounds.append((s, min(n, s + step)))

    def run(b):
        s, e = b
        if e <= s:
            return
        tail = 1 if (tail_exact and e > n_full) else 0
        lib.oracle_mlp_forward(ptr(x[s:e]), e - s, len(layers), ptr(dims), wp, bp, ptr(flags),
                               int(input_relu), tail, ptr(y[s:e]))

    if len(bounds) == 1:
        run(bounds[0])
    else:
        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(run, bounds))
    return y


def stage(a: np.ndarray, math: str) -> np.ndarray:
    """float16 / bfloat16 staging (round to nearest even) as float32 values."""
    a = np.asarray(a, dtype=np.float32)
    if math == "f16":
        return a.astype(np.float16).astype(np.float32)
    if math == "bf16":
        u = a.view(np.uint32).astype(np.uint64)
        lsb = (u >> 16) & 1
        r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
        nan = np.isnan(a)
        out = r.view(np.float32).copy()
        out[nan] = np.nan
        return out
    return a


def mlp_forward_f64(x: np.ndarray, layers, input_relu: bool = False) -> np.ndarray:
    """Vectorised float64 evaluation of the same staged operands (the
    products are exact in fp32 for float16 operands, so this is the
    rounding-free value the fp32 accumulation approximates). Used at sizes
    where the row-by-row routine is too slow and as the accuracy yardstick."""
    a = np.asarray(x, dtype=np.float32)
    if input_relu:
        a = np.maximum(a, 0)
    a = a.astype(np.float64)
    for l in layers:
        W = l["W"].astype(np.float32)
        if l["math"] == "f32":
            out = a @ W.astype(np.float64).T + l["b"].astype(np.float64)
        else:
            xs = stage(a.astype(np.float32), l["math"]).astype(np.float64)
            ws = stage(W, l["math"]).astype(np.float64)
            out = xs @ ws.T + l["b"].astype(np.float64)
        if l["relu"]:
            out = np.maximum(out, 0.0)
        # next layer consumes the fp32 value (stored as float in the shader)
        a = out.astype(np.float32).astype(np.float64)
    return a


def mlp_forward_blas(x: np.ndarray, layers, input_relu: bool = False) -> np.ndarray:
    """CPU baseline: fp32 BLAS GEMMs on staged operands (the torch/CPU-style
    restatement of the reference path that the benchmark times)."""
    a = np.asarray(x, dtype=np.float32)
    if input_relu:
        a = np.maximum(a, 0)
    for l in layers:
        W = l["_Wstaged"] if "_Wstaged" in l else stage(l["W"], l["math"])
        xs = a if l["math"] == "f32" else stage(a, l["math"])
        a = xs @ W.T
        a += l["b"]
        if l["relu"]:
            np.maximum(a, 0, out=a)
    return a


def mlp_forward_torch_cpu(x, layers, input_relu: bool = False, threads: int | None = None):
    """CPU baseline on torch's CPU kernels (the torch/CPU restatement of the
    reference path): float16/bfloat16 staging by dtype round trip, fp32 GEMM,
    fp32 bias, ReLU. `layers` entries may carry a pre-staged "_Wt" torch
    tensor (see prestage_torch). Uses all host threads unless told otherwise."""
    import torch

    if threads:
        torch.set_num_threads(threads)
    a = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    if input_relu:
        a = torch.relu(a)
    for l in layers:
        Wt = l["_Wt"] if "_Wt" in l else _torch_stage(torch.as_tensor(l["W"]), l["math"]).t().contiguous()
        xs = a if l["math"] == "f32" else _torch_stage(a, l["math"])
        a = torch.addmm(torch.as_tensor(l["b"]), xs, Wt)
        if l["relu"]:
            a.relu_()
    return a


def _torch_stage(t, math):
    import torch

    if math == "f16":
        return t.to(torch.float16).to(torch.float32)
    if math == "bf16":
        return t.to(torch.bfloat16).to(torch.float32)
    return t


def prestage_torch(layers):
    import torch

    out = []
    for l in layers:
        d = dict(l)
        d["_Wt"] = _torch_stage(torch.as_tensor(l["W"]), l["math"]).t().contiguous()
        d["b"] = torch.as_tensor(l["b"])
        out.append(d)
    return out


def prestage(layers):
    """Caches each layer's staged weight for repeated mlp_forward_blas calls."""
    out = []
    for l in layers:
        d = dict(l)
        d["_Wstaged"] = np.ascontiguousarray(stage(l["W"], l["math"]))
        out.append(d)
    return out


def rel_errors(y: np.ndarray, ref: np.ndarray):
    """The comparison metric used by every parity test:
    normwise  max|y - ref| / max|ref|
    elementwise max(|y - ref| / (|ref| + rms(ref)))."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    diff = np.abs(y - ref)
    scale = np.max(np.abs(ref)) if ref.size else 0.0
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    normwise = float(diff.max() / scale) if ref.size and scale > 0 else float(diff.max() if ref.size else 0.0)
    elem = float(np.max(diff / (np.abs(ref) + rms))) if ref.size and rms > 0 else normwise
    return normwise, elem


def within_tolerance(y, ref, tol: float) -> bool:
    """BASELINE tolerance: normwise <= tol and elementwise <= tol (elementwise
    measured against |ref| + rms(ref), which keeps near-zero outputs from
    dominating)."""
    nw, el = rel_errors(y, ref)
    return nw <= tol and el <= tol
