"""Builds libapex_attn.so in-tree (next to the apex_attn package) with nvcc for sm_100a.

Usage: python apex-tune-results_b200/build.py [--verbose]
The library links the CUDA runtime statically and resolves cuTensorMapEncodeTiled through
cudaGetDriverEntryPoint, so it needs no -lcuda and loads on a machine without a GPU.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "apex_attn", "libapex_attn.so")
SOURCES = [os.path.join(CSRC, "attn_fwd.cu")]
HEADERS = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))] + [
    os.path.join(ROOT, "include", "apex_attn.h")]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def command(out: str = OUT) -> list[str]:
    return [nvcc_path(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
            "-lineinfo", "-Xptxas", "-v", "-Xcompiler", "-fPIC", "-shared",
            "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-o", out, *SOURCES]


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(f) <= t for f in SOURCES + HEADERS + [__file__])


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    tmp = OUT + ".tmp"
    proc = subprocess.run(command(tmp), capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("nvcc failed building libapex_attn.so")
    log = proc.stdout + proc.stderr
    if verbose:
        sys.stdout.write(log)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
