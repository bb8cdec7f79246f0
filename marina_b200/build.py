"""Build recipes for the package's native libraries, compiled in-tree so the built `.so`
files travel with the source tree:

* ``libmarina_b200.so`` -- the CUDA evaluator (sm_100a only) and its C ABI
  (``include/marina_b200.h``);
* ``libmarina_b200_test.so`` -- the GPU test-suite's kernel-level entry points
  (``include/marina_b200_test.h``) over the same kernel sources compiled with ``MRN_TEST_HOOKS``;
  the evaluator library exports none of them;
* ``libmarina_chess.so`` -- the host-side position library (move generation, the
  reference's board/action encoding, seeded random playouts; ``include/marina_chess.h``) and
  the batched PUCT search that drives the evaluator for the nodes/s measurement
  (``include/marina_search.h``).

``python -m marina_b200.build`` builds both. Rebuilds are skipped when the output is newer
than every source.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"

CUDA_LIB = PKG / "libmarina_b200.so"
TEST_LIB = PKG / "libmarina_b200_test.so"
CHESS_LIB = PKG / "libmarina_chess.so"

CUDA_SOURCES = ["gemm.cu", "kernels.cu", "attention.cu", "runtime.cu", "static_forward.cu", "group.cpp"]
TEST_SOURCES = ["gemm.cu", "kernels.cu", "attention.cu", "api_test.cu"]
CUDA_HEADERS = ["ptx.cuh", "rows.cuh", "e4m3x2.cuh", "gemm.cuh", "gemm.h", "tmap.h", "kernels.cuh", "launch.h", "runtime.h"]
CHESS_SOURCES = ["chess.cpp", "puct.cpp"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-DMRN_BUILD_LIBRARY",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (Path(cand).exists() or cand == "nvcc"):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build failed ({' '.join(cmd[:3])} ...):\n{proc.stdout}")


def _build_shared(out: Path, sources: list[str], objdir: Path, extra: list[str], headers: list[Path], force: bool,
                  verbose: bool) -> Path:
    srcs = [CSRC / s for s in sources]
    deps = srcs + headers + [Path(__file__)]
    if not force and not _stale(out, deps):
        return out
    objdir.mkdir(parents=True, exist_ok=True)
    nvcc = _nvcc()
    objs = []
    for s in srcs:
        o = objdir / (s.stem + ".o")
        flags = list(NVCC_FLAGS) + extra + (["-Xptxas", "-v"] if verbose else [])
        if force or _stale(o, [s] + headers + [Path(__file__)]):
            _run([nvcc, *flags, f"-I{INCLUDE}", "-c", str(s), "-o", str(o)])
        objs.append(str(o))
    tmp = out.with_suffix(".so.tmp")
    _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp), *objs,
          "-cudart", "static", "-Xcompiler", "-fPIC", "-lpthread", "-ldl", "-lrt"])
    tmp.replace(out)
    return out


def build_cuda(force: bool = False, verbose: bool = False) -> Path:
    headers = [CSRC / h for h in CUDA_HEADERS] + [INCLUDE / "marina_b200.h"]
    return _build_shared(CUDA_LIB, CUDA_SOURCES, PKG / "_build", [], headers, force, verbose)


def build_test(force: bool = False, verbose: bool = False) -> Path:
    headers = [CSRC / h for h in CUDA_HEADERS] + [INCLUDE / "marina_b200.h", INCLUDE / "marina_b200_test.h"]
    return _build_shared(TEST_LIB, TEST_SOURCES, PKG / "_build" / "test", ["-DMRN_TEST_HOOKS"], headers, force,
                         verbose)


def build_chess(force: bool = False) -> Path:
    srcs = [CSRC / s for s in CHESS_SOURCES]
    deps = srcs + [INCLUDE / "marina_chess.h", INCLUDE / "marina_search.h", Path(__file__)]
    if not force and not _stale(CHESS_LIB, deps):
        return CHESS_LIB
    tmp = CHESS_LIB.with_suffix(".so.tmp")
    _run(["g++", "-O3", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", "-pthread", f"-I{INCLUDE}",
          *map(str, srcs), "-o", str(tmp)])
    tmp.replace(CHESS_LIB)
    return CHESS_LIB


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_chess(force)
    build_cuda(force, verbose)
    build_test(force, verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(CUDA_LIB)
    print(TEST_LIB)
    print(CHESS_LIB)
