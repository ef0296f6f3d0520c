"""Build recipe for the two libraries over the sm_100a kernels.

* ``libako_b200.so`` — the product: the C ABI of ``include/ako_b200.h``.
* ``libako_b200_measure.so`` — the same kernels compiled with
  ``AKO_B200_MEASUREMENT``, which also exports the launch overrides of
  ``include/ako_b200_measure.h`` for sweeps, benchmarks and tests.

Each ``csrc/*.cu`` file is compiled to an object with nvcc (in parallel).
Sources that never mention the measurement switch compile once and link
into both libraries; the rest compile once per library. The libraries are
linked next to this file, so they travel with the source tree. Objects are
rebuilt when their source, a shared header or the flags change.

Run as ``python -m ako_b200.build [--ptxas-verbose]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PACKAGE_DIR / "_build"
LIB_PATH = PACKAGE_DIR / "libako_b200.so"
MEASURE_LIB_PATH = PACKAGE_DIR / "libako_b200_measure.so"
MEASURE_DEFINE = "-DAKO_B200_MEASUREMENT"
#: Text that marks a source whose code differs in the measurement build.
_SWITCHES = ("AKO_B200_MEASUREMENT", "AKO_B200_OVERRIDE")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O2",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _headers_digest() -> str:
    h = hashlib.sha256()
    for p in sorted([*CSRC.glob("*.cuh"), *CSRC.glob("*.hpp"), *INCLUDE.glob("*.h")]):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()[:16]


def _varies(src: Path) -> bool:
    text = src.read_text()
    return any(s in text for s in _SWITCHES)


def _object_for(src: Path, flags: list[str], digest: str, tag: str) -> Path:
    key = hashlib.sha256((src.read_text() + " ".join(flags) + digest).encode()).hexdigest()[:16]
    return BUILD_DIR / f"{src.stem}{tag}.{key}.o"


def _compile(nvcc: str, src: Path, obj: Path, flags: list[str]) -> tuple[Path, str]:
    cmd = [nvcc, *flags, "-c", str(src), "-o", str(obj) + ".tmp"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    os.replace(str(obj) + ".tmp", obj)
    return obj, proc.stdout + proc.stderr


def _link(nvcc: str, objects: list[Path], lib: Path) -> None:
    stale = [o for o in objects if not lib.exists() or o.stat().st_mtime > lib.stat().st_mtime]
    if not stale and lib.exists():
        return
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, lib)


def build(*, ptxas_verbose: bool = False, jobs: int | None = None, quiet: bool = True) -> Path:
    """Compile every kernel source and link both libraries; returns the product library's path."""
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    flags = list(NVCC_FLAGS)
    if ptxas_verbose:
        flags += ["-Xptxas", "-v"]
    mflags = [*flags, MEASURE_DEFINE]
    digest = _headers_digest()
    product: list[Path] = []
    measure: list[Path] = []
    todo: dict[Path, tuple[Path, list[str]]] = {}
    for src in sorted(CSRC.glob("*.cu")):
        obj = _object_for(src, flags, digest, "")
        product.append(obj)
        todo[obj] = (src, flags)
        if _varies(src):
            mobj = _object_for(src, mflags, digest, ".measure")
            measure.append(mobj)
            todo[mobj] = (src, mflags)
        else:
            measure.append(obj)
    work = [(s, o, f) for o, (s, f) in todo.items() if ptxas_verbose or not o.exists()]
    if work:
        workers = jobs or min(len(work), os.cpu_count() or 4)
        with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
            futures = [pool.submit(_compile, nvcc, s, o, f) for s, o, f in work]
            for fut in futures:
                _, log = fut.result()
                if log.strip() and (ptxas_verbose or not quiet):
                    print(log, file=sys.stderr)
    _link(nvcc, product, LIB_PATH)
    _link(nvcc, measure, MEASURE_LIB_PATH)
    # Drop objects of earlier source revisions.
    keep = {o.name for o in todo}
    for old in BUILD_DIR.glob("*.o"):
        if old.name not in keep:
            old.unlink()
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills per kernel")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    args = ap.parse_args()
    path = build(ptxas_verbose=args.ptxas_verbose, jobs=args.jobs, quiet=False)
    print(path)
    print(MEASURE_LIB_PATH)


if __name__ == "__main__":
    main()
