"""Build the native library `ratchet_b200/_fgg.so` for sm_100a with nvcc.

    python -m ratchet_b200.build            # build if sources are newer
    python -m ratchet_b200.build --force    # always rebuild

The library is a plain C-ABI shared object (include/fgg_api.h); it links the
CUDA runtime statically and fetches the driver's tensor-map encoder at run
time, so it needs no libcuda at link time and cross-compiles on a machine
without a GPU.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "_fgg.so"
SOURCES = ["fgg_common.cu", "fgg_nvfp4.cu", "fgg_mx.cu", "fgg_quant.cu", "fgg_scratch.cu",
           "fgg_moe.cu", "fgg_peer.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def _sources() -> list[Path]:
    return [CSRC / s for s in SOURCES if (CSRC / s).exists()]


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = _sources() + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "fgg_api.h"]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    out_dir = PKG / "_build"
    out_dir.mkdir(exist_ok=True)
    objs = []
    # Only the C ABI is exported: template statics stay private to this library
    # even when another copy of it is loaded into the same process.
    common = [nvcc(), "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-Xcompiler", "-fno-gnu-unique",
              "-I", str(ROOT / "include"), "--expt-relaxed-constexpr"]
    if ptxas_verbose:
        common += ["-Xptxas", "-v"]
    jobs = []
    for src in _sources():
        obj = out_dir / (src.stem + ".o")
        cmd = common + ["-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        jobs.append(cmd)
        objs.append(str(obj))
    # one nvcc per translation unit, in parallel
    with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 1)) as pool:
        for r in pool.map(lambda c: subprocess.run(c, check=True), jobs):
            pass
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs, "-cudart", "static"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args(argv)
    path = build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
