"""Build libb2e.so in-tree with nvcc for sm_100a.

    python -m hackathon_b200.build [--force] [--jobs N]

Each csrc/*.cu compiles to an object under hackathon_b200/_build/ (in parallel),
then they link into hackathon_b200/lib/libb2e.so. An object is rebuilt when its
source or any header is newer. The library links the CUDA runtime statically, so
it loads without a toolkit on the library path.

A second library, hackathon_b200/lib/libb2e_trace.so, is the same objects with
latency.cu compiled under B2E_LAT_TRACE: the one-kernel latency path stamps
each stage with %globaltimer (python -m hackathon_b200.profiling latency-trace).
The product loads libb2e.so; only that profiling command loads the trace build.

csrc/rows.c, a CPython extension of the drop-in client (Python lists of features
to float32 rows), compiles with the host C compiler to
hackathon_b200/lib/_b2e_rows<EXT_SUFFIX>.
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
REPO = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libb2e.so"
TRACE_LIB = PKG / "lib" / "libb2e_trace.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", str(REPO / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


def _headers():
    return list(CSRC.glob("*.cuh")) + list((REPO / "include").glob("*.h"))


def _stale(src: Path, obj: Path, newest_header: float) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or newest_header > t


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    newest = max((h.stat().st_mtime for h in _headers()), default=0.0)
    cc = nvcc()

    def compile_one(src: Path):
        obj = BUILD / (src.stem + ".o")
        if force or _stale(src, obj, newest):
            cmd = [cc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
            if verbose and r.stderr.strip():
                print(r.stderr, file=sys.stderr)
        return obj

    def compile_trace():
        src, obj = CSRC / "latency.cu", BUILD / "latency_trace.o"
        if force or _stale(src, obj, newest):
            cmd = [cc, *ARCH, *NVCC_FLAGS, "-DB2E_LAT_TRACE", "-c", str(src), "-o", str(obj)]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name} (trace):\n{r.stdout}\n{r.stderr}")
        return obj

    with ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        trace_obj = ex.submit(compile_trace)
        objs = list(ex.map(compile_one, srcs))
        trace_obj = trace_obj.result()
    _link(cc, LIB, objs, force)
    _link(cc, TRACE_LIB, [o for o in objs if o.stem != "latency"] + [trace_obj], force)
    build_rows(force)
    return LIB


def build_rows(force: bool = False) -> Path:
    """csrc/rows.c against the running interpreter's headers."""
    import sysconfig

    src = CSRC / "rows.c"
    out = LIB.parent / ("_b2e_rows" + sysconfig.get_config_var("EXT_SUFFIX"))
    if force or not out.exists() or src.stat().st_mtime > out.stat().st_mtime:
        cc = os.environ.get("CC") or shutil.which("gcc") or shutil.which("cc")
        if cc is None:
            raise RuntimeError("no C compiler for csrc/rows.c (set CC)")
        cmd = [cc, "-O3", "-shared", "-fPIC", "-I", sysconfig.get_paths()["include"], str(src), "-o", str(out)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"cc failed on rows.c:\n{r.stdout}\n{r.stderr}")
    return out


def _link(cc: str, lib: Path, objs, force: bool) -> None:
    if force or not lib.exists() or any(o.stat().st_mtime > lib.stat().st_mtime for o in objs):
        tmp = lib.with_suffix(".so.tmp")
        cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, lib)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))


if __name__ == "__main__":
    main()
