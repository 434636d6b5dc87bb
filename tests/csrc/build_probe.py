"""Builds the test-only probe library tests/_build/libumma_probe.so (nvcc, sm_100a)."""
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE.parent / "_build" / "libumma_probe.so"


def build(force=False):
    src = HERE / "umma_probe.cu"
    deps = [src, HERE.parents[1] / "sorernn_b200" / "csrc" / "sm100.cuh", HERE.parents[1] / "sorernn_b200" / "csrc" / "tmap.h"]
    if not force and OUT.exists() and all(OUT.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    cmd = ["/usr/local/cuda/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-lineinfo",
           "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-o", str(OUT), str(src)]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
