"""Build the reference CUDA rasterizer extension as a GPU-side parity oracle.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this file or
its output; only `tests/` (GPU parity tests) and `__graft_entry__.build()`
touch it.

The reference's native path is two source files, `src/cuda/rasterizer.cpp`
(pybind11 + libtorch) and `src/cuda/kernel.cu` (CUDA + CUB). This recipe
compiles them where they lie, with `torch.utils.cpp_extension.load`, for
sm_100 (the reference's own `setup.py` passes no arch flags, so its arch comes
from TORCH_CUDA_ARCH_LIST; 10.0 is the B200). The reference's own build
system (`setup.py`) is not run, no source is copied, and every output goes to
`oracle/_ref/` (git-ignored; it travels to the GPU box with the tree).

The built module is named `gs_reference_rasterizer` and exposes the reference's
seven functions (`project_points`, `project_points_backward`,
`evaluate_spherical_harmonics`, `evaluate_spherical_harmonics_backward`,
`compute_tile_intersection`, `rasterize`, `rasterize_backward`).
"""
from __future__ import annotations

import glob
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_OUT = os.path.join(HERE, "_ref")
MODULE_NAME = "gs_reference_rasterizer"
REFERENCE_ROOT = os.environ.get("GS_REFERENCE_ROOT", "/root/reference")


def built_path() -> str | None:
    """Path of the built reference extension, or None when it is not built."""
    hits = sorted(glob.glob(os.path.join(REF_OUT, "build", MODULE_NAME + "*.so")))
    return hits[0] if hits else None


def build(verbose: bool = False) -> str | None:
    """Compile the reference extension into oracle/_ref/build (skipped if fresh).

    Returns the .so path, or None when the reference sources are absent (the
    GPU box has only the prebuilt file).
    """
    src_dir = os.path.join(REFERENCE_ROOT, "src", "cuda")
    sources = [os.path.join(src_dir, "rasterizer.cpp"), os.path.join(src_dir, "kernel.cu")]
    existing = built_path()
    if not all(os.path.exists(s) for s in sources):
        return existing
    if existing is not None:
        newest_src = max(os.path.getmtime(s) for s in sources)
        if os.path.getmtime(existing) >= newest_src:
            return existing
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    from torch.utils.cpp_extension import load

    build_dir = os.path.join(REF_OUT, "build")
    os.makedirs(build_dir, exist_ok=True)
    load(
        name=MODULE_NAME,
        sources=sources,
        build_directory=build_dir,
        extra_cflags=["-O2"],
        extra_cuda_cflags=["-O3"],
        verbose=verbose,
    )
    return built_path()


def load_module():
    """Import the prebuilt reference extension (needs torch already imported)."""
    path = built_path()
    if path is None:
        return None
    import torch  # noqa: F401  (the extension links against libtorch)

    spec = importlib.util.spec_from_file_location(MODULE_NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    out = build(verbose="-v" in sys.argv)
    print(out)
