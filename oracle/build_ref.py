"""Builds the REFERENCE's own CUDA extension (kernel/w4a4.cu, unmodified, compiled from where it lies
in the reference checkout) into oracle/_ref/ -- test infrastructure only, like the rest of oracle/.

The reference file is a PyTorch extension (pybind11 + ATen) exporting ``quantize`` and ``matmul``.
It is compiled here with nvcc for sm_100a against the PyTorch headers and libraries of this image,
through torch.utils.cpp_extension (ninja), into oracle/_ref/dscq_ref_w4a4.so. Only its
``quantize`` entry (quantize_cuda, kernel/w4a4.cu:164-187, no capability guard) is used, by
tests/test_reference_kernel_gpu.py, as a GPU-side check that the asymmetric codes, scales and zero
points of this library equal the reference kernel's own on a B200. Its ``matmul`` refuses compute
capability >= 9.0 (kernel/w4a4.cu:206) and is never called.

    python oracle/build_ref.py [path/to/reference]

The reference checkout defaults to $DSCQ_REFERENCE, else a directory named ``reference`` beside the
repository. Without a checkout the script does nothing (the GPU box only uses the prebuilt .so).
"""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "_ref")
NAME = "dscq_ref_w4a4"
SO = os.path.join(OUT, NAME + ".so")


def reference_dir(arg: str | None = None) -> str:
    return arg or os.environ.get("DSCQ_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")


def build(ref: str | None = None, verbose: bool = False) -> str | None:
    src = os.path.join(reference_dir(ref), "kernel", "w4a4.cu")
    if not os.path.exists(src):
        return SO if os.path.exists(SO) else None
    if os.path.exists(SO) and os.path.getmtime(SO) >= os.path.getmtime(src):
        return SO
    os.makedirs(OUT, exist_ok=True)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"  # -gencode arch=compute_100a,code=sm_100a only
    from torch.utils import cpp_extension

    cpp_extension.load(name=NAME, sources=[src], build_directory=OUT, extra_cuda_cflags=["-O3"], verbose=verbose)
    return SO


def load():
    """Imports the prebuilt extension (after torch). Raises FileNotFoundError if it was not built."""
    import importlib.util

    import torch  # noqa: F401  (the extension links against libtorch / libc10)

    if not os.path.exists(SO):
        raise FileNotFoundError(f"{SO} not built (python oracle/build_ref.py with the reference checkout present)")
    spec = importlib.util.spec_from_file_location(NAME, SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
