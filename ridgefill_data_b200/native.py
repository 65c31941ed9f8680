"""Standalone native programs (no Python or torch inside): built in-tree with nvcc for sm_100a.

  identity_check   csrc/native/identity_check.cu + csrc/gemm.cu + csrc/gemm2sm.cu + csrc/gemv.cu: the fill GEMM
                   (one-SM and two-SM kernels) with an identity map must copy
                   its input bit for bit (both N-tile widths, with and without the bias epilogue)

build_native() compiles every program into ridgefill_data_b200/bin/ (the driver's build step calls it);
run(name, *args) runs one and returns (exit code, stdout).
"""
from __future__ import annotations

import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BIN = PKG / "bin"
NVCC = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
        "--expt-relaxed-constexpr", f"-I{CSRC}"]
PROGRAMS = {"identity_check": ([CSRC / "native" / "identity_check.cu", CSRC / "gemm.cu", CSRC / "gemm2sm.cu",
                                 CSRC / "gemv.cu"],
                               ["-lcuda"])}


def build_native(names=None):
    BIN.mkdir(exist_ok=True)
    out = {}
    for name, (srcs, libs) in PROGRAMS.items():
        if names is not None and name not in names:
            continue
        target = BIN / name
        newest = max(p.stat().st_mtime for p in srcs + [CSRC / "gemm.h", CSRC / "ptx.cuh", CSRC / "kernels.h"])
        if not target.exists() or target.stat().st_mtime < newest:
            subprocess.run(NVCC + [str(s) for s in srcs] + libs + ["-o", str(target)], check=True)
        out[name] = target
    return out


def run(name, *args, timeout=300):
    path = BIN / name
    if not path.exists():
        build_native([name])
    p = subprocess.run([str(path), *map(str, args)], capture_output=True, text=True, timeout=timeout)
    return p.returncode, p.stdout + p.stderr
