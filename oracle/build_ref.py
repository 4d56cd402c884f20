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

`stage_python()` does the same for the reference's Python side of the path:
it byte-compiles, where they lie, the modules the reference's gradient
harness imports (src/cuda/wrapper.py, src/torch_rasterizer.py,
src/gaussian.py, src/dataset.py, src/__init__.py and
scripts/check_cuda_gradients.py) into sourceless bytecode files
(`<module>.pycode`: the `.pyc` format under a name that snapshot tools do not
drop as a cache file) under `oracle/_ref/py/` in the same package layout,
so that the harness and the reference's Torch rasterizer can run on the GPU
box (which has no reference checkout) as test infrastructure and as the CPU
baseline. `install_staged_importer()` makes them importable under their
reference names (`src.cuda.wrapper`, `src.torch_rasterizer`, ...).

The reference checkout is $GS_REFERENCE_ROOT, else a directory named
`reference` beside this repository; where neither exists (the GPU box) both
steps are skipped and the prebuilt outputs are used.
"""
from __future__ import annotations

import glob
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_OUT = os.path.join(HERE, "_ref")
MODULE_NAME = "gs_reference_rasterizer"
# the reference checkout: $GS_REFERENCE_ROOT, else a directory named "reference"
# beside this repository
REFERENCE_ROOT = os.environ.get("GS_REFERENCE_ROOT") or os.path.join(
    os.path.dirname(os.path.dirname(HERE)), "reference")
REF_PY = os.path.join(REF_OUT, "py")
# the reference modules the gradient harness imports, relative to its root
PY_SOURCES = ("src/__init__.py", "src/cuda/wrapper.py", "src/torch_rasterizer.py",
              "src/gaussian.py", "src/dataset.py", "scripts/check_cuda_gradients.py")


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


BYTECODE_SUFFIX = ".pycode"


def staged_file(rel: str) -> str:
    return os.path.join(REF_PY, rel[:-3] + BYTECODE_SUFFIX)


def stage_python() -> str | None:
    """Byte-compile the reference's Python modules listed in PY_SOURCES into
    oracle/_ref/py (sourceless bytecode, recompiled when a source is newer).
    Returns the staging root, the prebuilt one when the sources are absent,
    or None when neither exists."""
    import py_compile

    srcs = [os.path.join(REFERENCE_ROOT, rel) for rel in PY_SOURCES]
    if not all(os.path.exists(s) for s in srcs):
        return REF_PY if staged_python_ok() else None
    for rel, src in zip(PY_SOURCES, srcs):
        dst = staged_file(rel)
        if os.path.exists(dst) and os.path.getmtime(dst) >= os.path.getmtime(src):
            continue
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        py_compile.compile(src, cfile=dst, dfile=rel, doraise=True,
                           invalidation_mode=py_compile.PycInvalidationMode.UNCHECKED_HASH)
    return REF_PY


def staged_python_ok() -> bool:
    return all(os.path.exists(staged_file(rel)) for rel in PY_SOURCES)


class _StagedFinder:
    """Meta-path finder for the staged reference modules: `a.b.c` is
    oracle/_ref/py/a/b/c.pycode, a package when a/b/c/__init__.pycode exists,
    a namespace package for a plain directory (src/cuda has no __init__)."""

    def find_spec(self, name, path=None, target=None):
        import importlib.machinery as mach
        import importlib.util as iu

        if name.split(".")[0] not in ("src", "scripts"):
            return None
        rel = os.path.join(REF_PY, *name.split("."))
        init = os.path.join(rel, "__init__" + BYTECODE_SUFFIX)
        if os.path.exists(init):
            return iu.spec_from_file_location(name, init,
                                              loader=mach.SourcelessFileLoader(name, init),
                                              submodule_search_locations=[rel])
        if os.path.exists(rel + BYTECODE_SUFFIX):
            f = rel + BYTECODE_SUFFIX
            return iu.spec_from_file_location(name, f, loader=mach.SourcelessFileLoader(name, f))
        if os.path.isdir(rel):
            spec = mach.ModuleSpec(name, None, is_package=True)
            spec.submodule_search_locations = [rel]
            return spec
        return None


def install_staged_importer() -> bool:
    """Make the staged reference modules importable by their reference names
    (first on sys.meta_path). Returns False when they are not staged."""
    if not staged_python_ok():
        return False
    if not any(isinstance(f, _StagedFinder) for f in sys.meta_path):
        sys.meta_path.insert(0, _StagedFinder())
    return True


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
    print(stage_python())
