"""Build the reference's own kernel into ``oracle/_ref/`` — TEST INFRASTRUCTURE.

Recipe: ``oracle/ref_binding.cu`` includes the reference's
``nvfp4_dual_gemm.cu`` (and through it ``tcgen05-interface.cuh`` and
``tma-interface.cuh``) from the reference checkout, and is compiled with the
flags the reference's own JIT build uses (submission.py:1136-1150:
``-O3 --use_fast_math -gencode=arch=compute_100a,code=sm_100a
--expt-relaxed-constexpr --relocatable-device-code=false``, linked with
``-lcuda``) into the Python module ``oracle/_ref/nvfp4_ref*.so``.  Only the
output lands under ``oracle/_ref/`` (git-ignored); the built module travels
to GPU machines with the checkout, the reference sources do not.

The reference directory defaults to ``reference`` beside this repository and can be overridden with ``NVFP4DG_REFERENCE_DIR``.

The module exposes ``cuda_nvfp4_dual_gemm(A, B1, B2, SFA, SFB1, SFB2, C)``
(the reference's own dispatch entry) and ``cuda_nvfp4_dual_gemm_generic``
(the same arguments; the reference's launcher template instantiated for
``GENERIC_SHAPES``).
Safe shapes: only those in the reference's dispatch table
(nvfp4_dual_gemm.cu:403-442) with K / 256 >= 4; for K / 256 < 4 the
reference's producer prologue issues scale copies past the end of the scale
buffers (nvfp4_dual_gemm.cu:246-248), so those shapes are never run.
"""
from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
OUT_DIR = os.path.join(HERE, "_ref")
MODULE = "nvfp4_ref"

# Shapes of the reference's dispatch table that are safe to run.
SAFE_SHAPES = {
    (256, 4096, 7168), (512, 4096, 7168), (256, 3072, 4096),
    (512, 3072, 7168), (1536, 512, 7168), (3072, 1024, 1536),
    (7168, 2304, 2048), (4608, 384, 7168), (7168, 384, 2304),
    (512, 768, 7168),
}
# The reference returns C as a transposed view for this shape
# (nvfp4_dual_gemm.cu:413-415): column-major storage.
TRANSPOSED_SHAPES = {(512, 3072, 7168)}
# Shapes outside the dispatch table run through the harness-side
# instantiation of the reference's launcher template
# (``cuda_nvfp4_dual_gemm_generic`` in ref_binding.cu): the benchmark's
# prefill shape and its N-sharded rank slices for 1, 2, 4 and 8 GPUs.
GENERIC_SHAPES = {(4096, 14336, 4096)} | {
    (8192, 28672 // w, 8192) for w in (1, 2, 4, 8)}


def entry(mod, shape):
    """The reference module's function that runs `shape`, or None."""
    if mod is None:
        return None
    if tuple(shape) in SAFE_SHAPES:
        return mod.cuda_nvfp4_dual_gemm
    if tuple(shape) in GENERIC_SHAPES and hasattr(
            mod, "cuda_nvfp4_dual_gemm_generic"):
        return mod.cuda_nvfp4_dual_gemm_generic
    return None


def reference_dir() -> str:
    return os.environ.get("NVFP4DG_REFERENCE_DIR",
                          os.path.join(os.path.dirname(REPO), "reference"))


def built_path() -> str | None:
    hits = sorted(glob.glob(os.path.join(OUT_DIR, MODULE + "*.so")))
    return hits[0] if hits else None


def build(verbose: bool = False) -> str:
    """Compile the reference kernel module; returns the .so path."""
    src_dir = reference_dir()
    if not os.path.exists(os.path.join(src_dir, "nvfp4_dual_gemm.cu")):
        raise FileNotFoundError(f"reference sources not found in {src_dir}")
    os.makedirs(OUT_DIR, exist_ok=True)
    from torch.utils import cpp_extension

    stubs = "/usr/local/cuda/lib64/stubs"
    try:
        _compile_and_import(cpp_extension, src_dir, stubs, verbose)
    except (ImportError, OSError) as exc:
        # cpp_extension.load imports the module after linking it; on a
        # machine without a GPU driver that import fails (libcuda.so.1 is
        # absent) although the module was built.
        if built_path() is None:
            raise
        if verbose:
            print(f"built, not imported here: {exc}")
    path = built_path()
    if path is None:
        raise RuntimeError("reference build produced no module")
    return path


def _compile_and_import(cpp_extension, src_dir: str, stubs: str,
                        verbose: bool) -> None:
    cpp_extension.load(
        name=MODULE,
        sources=[os.path.join(HERE, "ref_binding.cu")],
        extra_include_paths=[src_dir],
        extra_cuda_cflags=[
            "-O3",
            "--use_fast_math",
            "-gencode=arch=compute_100a,code=sm_100a",
            "--expt-relaxed-constexpr",
            "--relocatable-device-code=false",
        ],
        extra_ldflags=[f"-L{stubs}", "-lcuda"],
        build_directory=OUT_DIR,
        verbose=verbose,
        is_python_module=True,
    )


def load():
    """Import the prebuilt reference module (no compilation); None if absent."""
    path = built_path()
    if path is None:
        return None
    import torch  # noqa: F401  (libtorch must be loaded first)

    if MODULE in sys.modules:
        return sys.modules[MODULE]
    loader = importlib.machinery.ExtensionFileLoader(MODULE, path)
    spec = importlib.util.spec_from_file_location(MODULE, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[MODULE] = mod
    return mod


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
