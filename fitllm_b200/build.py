"""Build libfitq.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m fitllm_b200.build [--verbose]

The library is written to ``fitllm_b200/_lib/libfitq.so``.  The CUDA runtime
is linked statically and the driver is reached through
cudaGetDriverEntryPoint, so the library loads on a machine without a GPU
driver (its calls then report FITQ_ERR_NO_DEVICE).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libfitq.so"
INCLUDE = PKG.parent / "include"

SOURCES = ["nf4.cu", "gemm_sm100.cu", "lora.cu", "gemv.cu", "optim.cu", "abi.cu",
           "gemv_noalloc.cu", "layer_ops.cu", "gemm_sm100_2cta.cu", "gemv_tc.cu", "attn.cu", "ce.cu",
           "selftest.cu", "gemm_nf4.cu", "gemm_nf4_2cta.cu", "merge.cu", "train_attn.cu"]
HEADERS = ["common.cuh", "kernels.cuh", "pair.cuh", "nf4_decode.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-cudart", "static",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libfitq")
    return cand


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [INCLUDE / "fitq.h", Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu into one shared object (parallel per-file objects, one link)."""
    if not force and not _stale():
        return LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    obj_dir = OUT_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    cc = nvcc()
    procs = []
    for s in SOURCES:
        obj = obj_dir / (Path(s).stem + ".o")
        cmd = [cc, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / s), "-o", str(obj)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        procs.append((s, cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for s, cmd, p in procs:
        out, _ = p.communicate()
        text = out.decode(errors="replace")
        if p.returncode != 0:
            failed.append((s, text))
        elif verbose and text.strip():
            print(f"--- {s}\n{text}")
    if failed:
        msg = "\n".join(f"--- {s}\n{t}" for s, t in failed)
        raise RuntimeError(f"nvcc failed:\n{msg}")
    objs = [str(obj_dir / (Path(s).stem + ".o")) for s in SOURCES]
    tmp = LIB.with_suffix(".so.tmp")
    link = [cc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static",
            "-o", str(tmp), *objs]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force or a.verbose, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
