"""Builds the CUDA extension in-tree: rdv_project_b200/_lib/librdvb.so.

    python -m rdv_project_b200.csrc.build [--verbose]

nvcc cross-compiles for sm_100a (no GPU needed). The library links the CUDA
runtime statically so it has no run-time dependency beyond the driver.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIB_DIR = os.path.join(PKG, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "librdvb.so")
SOURCES = ["rdvb.cu"]
HEADERS = ["ptx.cuh", "rng.cuh", "mlp_tc.cuh", "mlp_simt.cuh", "winograd.cuh", "winograd_f43.cuh", "raymarch.cuh", "transmittance.cuh",
           "resample.cuh", "conv_tc.cuh", "sampler.cuh", "pbvr.cuh",
           "exchange.cuh"]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def nvcc_cmd(out: str, extra=()):
    return [
        nvcc_path(),
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-lineinfo", "-O3", "-std=c++17",
        "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC", "-shared",
        "-I", os.path.join(ROOT, "include"),
        "-I", HERE,
        "-o", out,
        *[os.path.join(HERE, s) for s in SOURCES],
        *extra,
    ]


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(HERE, f) for f in SOURCES + HEADERS] + [os.path.join(ROOT, "include", "rdvb.h")]
    return any(os.path.exists(d) and os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> str:
    if not force and not _stale():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    cmd = nvcc_cmd(tmp, extra)
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building librdvb.so")
    if verbose or ptxas_info:
        sys.stdout.write(res.stdout + res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB_PATH)
