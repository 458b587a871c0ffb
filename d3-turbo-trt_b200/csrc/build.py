"""Build libd3b200.so (the C-ABI CUDA library) in-tree for sm_100a.

    python d3-turbo-trt_b200/csrc/build.py [--verbose] [--ptxas-info]

Each .cu file is compiled separately with nvcc (in parallel), then linked into
``d3-turbo-trt_b200/libd3b200.so`` with the CUDA runtime linked statically, so
the library needs nothing at run time but the NVIDIA driver. Objects go to
``d3-turbo-trt_b200/_build/``. A file is recompiled when it or any header in
``csrc/`` or ``include/`` is newer than its object.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
ROOT = PKG.parent
BUILD = PKG / "_build"
LIB = PKG / "libd3b200.so"
SOURCES = ["capi.cu", "act_quant.cu", "norm_quant.cu", "readout.cu", "w8a8_gemm.cu", "prefix_bidir.cu", "snapshot.cu", "gated_delta.cu", "causal_conv.cu", "glue_quant.cu", "qk_norm_rope.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I",
    str(ROOT / "include"),
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libd3b200")
    return path


def _headers_mtime() -> float:
    files = list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((f.stat().st_mtime for f in files), default=0.0)


def _compile(src: str, ptxas_info: bool) -> tuple[str, str]:
    obj = BUILD / (Path(src).stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
    return src, res.stderr


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    todo = []
    for src in SOURCES:
        obj = BUILD / (Path(src).stem + ".o")
        if force or ptxas_info or not obj.exists() or obj.stat().st_mtime < max(hdr, (CSRC / src).stat().st_mtime):
            todo.append(src)
    with cf.ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 4)) as ex:
        for src, log in ex.map(lambda s: _compile(s, ptxas_info), todo):
            if verbose or ptxas_info:
                print(f"[nvcc] {src}\n{log}", file=sys.stderr)
    objs = [str(BUILD / (Path(s).stem + ".o")) for s in SOURCES]
    if todo or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, ptxas_info=a.ptxas_info, force=a.force))
