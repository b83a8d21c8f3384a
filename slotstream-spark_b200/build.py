"""Build libslotstream_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python slotstream-spark_b200/build.py [--force] [--jobs N]

Each csrc/*.cu is compiled to an object under _build/ (rebuilt only when the source or a header is newer),
then linked into slotstream_b200/_lib/libslotstream_b200.so. The CUDA runtime is linked statically, so
the library only needs the driver at run time.
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
LIBDIR = HERE / "slotstream_b200" / "_lib"
LIB = LIBDIR / "libslotstream_b200.so"

NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
         "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC)]


def _headers():
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, newest_header: float) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or newest_header > t


def _compile(src: Path, obj: Path, extra):
    cmd = [NVCC, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src.name, r.returncode, r.stdout + r.stderr


def build(force: bool = False, jobs: int = 8, extra=None, verbose: bool = False) -> Path:
    extra = list(extra or [])
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    newest = max((h.stat().st_mtime for h in _headers()), default=0.0)
    todo = [(s, BUILD / (s.stem + ".o")) for s in srcs]
    work = [(s, o) for s, o in todo if force or _stale(o, s, newest)]
    if work:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            for name, rc, out in ex.map(lambda so: _compile(*so, extra), work):
                if verbose or rc:
                    sys.stderr.write(f"--- {name}\n{out}")
                if rc:
                    raise RuntimeError(f"nvcc failed on {name}")
    objs = [o for _, o in todo]
    if force or work or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(tmp), *map(str, objs),
               "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/shared-memory use per kernel")
    a = ap.parse_args()
    ex = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, jobs=a.jobs, extra=ex, verbose=a.verbose or a.ptxas_v))
