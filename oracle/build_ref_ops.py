"""Build recipe for the reference's own CUDA ops (test and bench infrastructure only).

Compiles the reference extension's two source files, ``csrc/kernels.cu`` and
``csrc/pulsar_cuda.cpp`` of the reference tree, exactly as they are, with this image's nvcc for
sm_100a. The flags are those of the reference's ``setup.py`` (-O3, C++20, relaxed constexpr,
fast math). The output is a torch extension module named ``pulsar_cuda_ref`` under
``oracle/_ref/pulsar_cuda_ref/``. That folder is git-ignored, but it travels with the
repository snapshot, so GPU tests and ``bench.py --ops`` can load the built module where the
reference sources are absent.

The module is a checker and a timing baseline: tests compare the ``pulsar_cuda`` shim ops with
it, and the bench's op leg times both on the same device. Nothing in the product loads it.

Usage: ``python oracle/build_ref_ops.py [reference_root]`` (default: ``$PULSAR_REFERENCE`` or
``/root/reference``); ``load()`` imports an already built module, or returns None.
"""

from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "pulsar_cuda_ref")
NAME = "pulsar_cuda_ref"


def _so_path():
    hits = sorted(glob.glob(os.path.join(OUT, NAME + "*.so")))
    return hits[0] if hits else None


def build(ref_root: str | None = None, force: bool = False) -> str | None:
    """Compile the reference ops when the reference tree is present; returns the .so path (the
    existing one when already built and not forced), or None without a reference tree."""
    ref_root = ref_root or os.environ.get("PULSAR_REFERENCE", "/root/reference")
    srcs = [os.path.join(ref_root, "csrc", "kernels.cu"), os.path.join(ref_root, "csrc", "pulsar_cuda.cpp")]
    if not all(os.path.exists(s) for s in srcs):
        return _so_path()
    if _so_path() and not force:
        return _so_path()
    os.makedirs(OUT, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils import cpp_extension

    cpp_extension.load(
        name=NAME,
        sources=srcs,
        extra_cflags=["-O3", "-std=c++20"],
        extra_cuda_cflags=["-O3", "-std=c++20", "--expt-relaxed-constexpr", "-use_fast_math", "-Xptxas=-O3"],
        build_directory=OUT,
        verbose=False,
        is_python_module=True,
    )
    return _so_path()


def load():
    """The built reference ops module, or None when it has not been built."""
    so = _so_path()
    if so is None:
        return None
    if NAME in sys.modules:
        return sys.modules[NAME]
    import torch  # noqa: F401  (the extension links against torch's libraries)

    loader = importlib.machinery.ExtensionFileLoader(NAME, so)
    spec = importlib.util.spec_from_file_location(NAME, so, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[NAME] = mod
    return mod


if __name__ == "__main__":
    path = build(sys.argv[1] if len(sys.argv) > 1 else None, force="--force" in sys.argv)
    print(path or "reference sources not found; nothing built")
