"""Builds liblfm3attn.so in this directory from csrc/ for sm_100a (nvcc cross-compiles without a GPU), and the
kernels alone as cubin/lfm3attn_sm100a.cubin: the image a caller loads through the CUDA driver API with
lfm3a_load_cubin (the engine embeds it, as it embeds its own code objects)."""
from __future__ import annotations

import os
import pathlib
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
SRC = HERE / "csrc" / "lfm3attn.cu"
OUT = HERE / "liblfm3attn.so"
CUBIN = HERE / "cubin" / "lfm3attn_sm100a.cubin"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = pathlib.Path(home) / "bin" / "nvcc"
    return str(path) if path.exists() else "nvcc"


CUBIN_FLAGS = ["-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17"]


def needs_build(target: pathlib.Path = OUT) -> bool:
    if not target.exists():
        return True
    newest = max(p.stat().st_mtime for p in (HERE / "csrc").iterdir())
    header = HERE.parent / "include" / "lfm3attn.h"
    newest = max(newest, header.stat().st_mtime)
    return newest > target.stat().st_mtime


def _run(cmd, verbose: bool) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode})")
    if verbose:
        sys.stderr.write(res.stderr)


def build_cubin(out: pathlib.Path = CUBIN, verbose: bool = False) -> pathlib.Path:
    """The kernels of csrc/lfm3attn.cu as one sm_100a cubin (device code only)."""
    out.parent.mkdir(parents=True, exist_ok=True)
    _run([nvcc(), *CUBIN_FLAGS, "-o", str(out), str(SRC)], verbose)
    return out


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    if force or needs_build():
        cmd = [nvcc(), *NVCC_FLAGS, "-o", str(OUT), str(SRC)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd, verbose)
    if force or needs_build(CUBIN):
        build_cubin(verbose=verbose)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
