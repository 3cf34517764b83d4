"""Build recipe for libmetalattn.so (sm_100a) and the CPU oracle library.

The CUDA library is compiled in-tree with nvcc for sm_100a only; the oracle
(test infrastructure) is compiled with g++.  Both builds are incremental on
source timestamps.  Run ``python -m metalllm_b200.build`` or call
:func:`build_all`.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libmetalattn.so"
ORACLE_DIR = ROOT / "oracle"
ORACLE_LIB = ORACLE_DIR / "libattn_oracle.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmetalattn")
    return cand


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build command failed ({res.returncode}): {' '.join(cmd)}")


def build_cuda(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every .cu under csrc/ into libmetalattn.so (sm_100a)."""
    cu = sorted(CSRC.glob("*.cu"))
    deps = cu + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))
    if not force and not _stale(LIB, deps):
        return LIB
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    objs = []
    nvcc = _nvcc()
    for src in cu:
        obj = build_dir / (src.stem + ".o")
        if force or _stale(obj, [src] + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))):
            cmd = [nvcc, *NVCC_FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd += ["-Xptxas", "-v"]
                print(" ".join(cmd))
            _run(cmd)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp), *objs,
          "-Xcompiler", "-fPIC"])
    os.replace(tmp, LIB)
    return LIB


def build_oracle(force: bool = False) -> Path:
    """Compiles the CPU oracle (test infrastructure) into oracle/libattn_oracle.so."""
    src = ORACLE_DIR / "attn_oracle.cpp"
    if not force and not _stale(ORACLE_LIB, [src]):
        return ORACLE_LIB
    tmp = ORACLE_LIB.with_suffix(".so.tmp")
    _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-pthread", "-fno-fast-math",
          "-ffp-contract=off", str(src), "-o", str(tmp)])
    os.replace(tmp, ORACLE_LIB)
    return ORACLE_LIB


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_cuda(force=force, verbose=verbose)
    build_oracle(force=force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
    print(ORACLE_LIB)
