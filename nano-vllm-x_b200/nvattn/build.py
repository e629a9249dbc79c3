"""Build recipe for libnvattn.so (sm_100a only).

Compiles every ``csrc/*.cu`` with nvcc for ``arch=compute_100a,code=sm_100a``
into objects under ``<project>/_build/`` and links them into
``nvattn/libnvattn.so`` next to the Python loader, so the library travels
with the source tree. Rebuilds only what changed (mtime of the .cu and of
every header it can include).

    python -m nvattn.build            # build
    python -m nvattn.build --verbose  # also print ptxas register/smem usage
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
PROJECT_DIR = PKG_DIR.parent
REPO_DIR = PROJECT_DIR.parent
CSRC_DIR = PROJECT_DIR / "csrc"
INCLUDE_DIR = REPO_DIR / "include"
BUILD_DIR = PROJECT_DIR / "_build"
LIB_PATH = PKG_DIR / "libnvattn.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    *ARCH_FLAGS,
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = Path(home) / "bin" / "nvcc"
    if p.exists():
        return str(p)
    raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")


def _headers() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, verbose: bool) -> str:
    cmd = [nvcc_path(), *NVCC_FLAGS, f"-I{INCLUDE_DIR}", "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return r.stderr if verbose else ""


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile csrc/*.cu for sm_100a and link libnvattn.so; returns its path."""
    BUILD_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC_DIR.glob("*.cu"))
    if not sources:
        raise RuntimeError(f"no CUDA sources under {CSRC_DIR}")
    headers = _headers()
    jobs = []
    objs = []
    for src in sources:
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or verbose or _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for src, log in zip([j[0] for j in jobs],
                            ex.map(lambda j: _compile(j[0], j[1], verbose), jobs)):
            if verbose and log:
                print(f"--- {src.name}\n{log}", file=sys.stderr)
    if force or jobs or _stale(LIB_PATH, objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(verbose=args.verbose, force=args.force))


if __name__ == "__main__":
    main()
