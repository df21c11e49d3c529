"""Build the in-tree native libraries.

* ``_lib/libprana_cuda.so`` -- the sm_100a decode path behind include/prana_cuda.h
  (nvcc, ``-gencode arch=compute_100a,code=sm_100a``, IEEE divide/sqrt: never fast-math).
* ``_lib/libprana_synth.so`` -- the host-only seeded GGUF generator.

Run ``python -m prana_b200.build`` (or ``__graft_entry__.build()``).  Builds are
incremental on source modification times.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "_lib"
ROOT = PKG.parent

CUDA_SOURCES = ["kernels.cu", "attention.cu", "decode.cu", "ctx.cu", "model.cu", "noalloc.cu", "comm.cu", "qgemm.cu", "tokenizer.cpp", "sampler.cpp", "pool.cu", "loader.cu", "sample.cu"]
CUDA_HEADERS = ["common.cuh", "gemv.cuh", "finish.cuh", "mbar.cuh", "comm.h", "internal.h", "host.h", "unicode_alpha.h", "sampler.h", "tc.cuh"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC,-ffp-contract=off",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or Path(cand).exists()):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:4])} ...")


def build_cuda(force: bool = False, verbose: bool = False) -> Path:
    LIB.mkdir(exist_ok=True)
    out = LIB / "libprana_cuda.so"
    deps = [CSRC / s for s in CUDA_SOURCES + CUDA_HEADERS] + [ROOT / "include" / "prana_cuda.h"]
    if not force and not _stale(out, deps):
        return out
    objs = []
    obj_dir = LIB / "obj"
    obj_dir.mkdir(exist_ok=True)
    hdr_deps = [CSRC / h for h in CUDA_HEADERS] + [ROOT / "include" / "prana_cuda.h"]
    cmds = []
    for src in CUDA_SOURCES:
        obj = obj_dir / (Path(src).stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [CSRC / src] + hdr_deps):
            cmd = [_nvcc(), *NVCC_FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
            if verbose:
                cmd += ["-Xptxas", "-v"]
                print(" ".join(cmd))
            cmds.append(cmd)
    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=len(CUDA_SOURCES)) as ex:
        list(ex.map(_run, cmds))
    _run([_nvcc(), "-shared", "-cudart", "static", "-o", str(out), *map(str, objs), "-ldl"])
    return out


def build_synth(force: bool = False) -> Path:
    LIB.mkdir(exist_ok=True)
    out = LIB / "libprana_synth.so"
    deps = [CSRC / "synth.c", CSRC / "synth.h"]
    if force or _stale(out, deps):
        cc = os.environ.get("CC", "gcc")
        _run([cc, "-O2", "-fPIC", "-shared", "-pthread", "-std=gnu11", "-ffp-contract=off",
              "-o", str(out), str(CSRC / "synth.c"), "-lm"])
    return out


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_synth(force)
    build_cuda(force, verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print("built", LIB)
