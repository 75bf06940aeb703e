"""Build the sm_100a shared library ``libpulsar_b200.so`` in-tree with nvcc.

    python -m pulsar_b200.build            # from the pulsar-300m_b200 directory
    python pulsar-300m_b200/pulsar_b200/build.py

Every ``csrc/*.cu`` is compiled for ``-gencode arch=compute_100a,code=sm_100a`` with
``-lineinfo`` (objects in ``_build/``, compiled in parallel) and linked into
``pulsar_b200/libpulsar_b200.so``. The library has no torch dependency: it exports the
C ABI declared in ``include/pulsar_b200.h``.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)               # pulsar-300m_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG_DIR, "libpulsar_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-cudart", "static", "--expt-relaxed-constexpr",
              "-I" + os.path.join(REPO, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _needs_build(objs) -> bool:
    if not os.path.exists(LIB):
        return True
    lib_t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(REPO, "include", "pulsar_b200.h")]
    return any(os.path.getmtime(d) > lib_t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if not force and not _needs_build(objs):
        return LIB
    cc = nvcc()

    def compile_one(src, obj):
        cmd = [cc, *ARCH, *NVCC_FLAGS, *extra_flags, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        for err in ex.map(compile_one, srcs, objs):
            if verbose and err:
                print(err)
    tmp = LIB + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    v = "-v" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas" in sys.argv else []
    print(build(force="--force" in sys.argv, verbose=v or bool(extra), extra_flags=extra))
