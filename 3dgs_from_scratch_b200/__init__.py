"""B200-native differentiable Gaussian-splatting rasterizer.

Drop-in for the rasterizer of ruguangyou/3dgs_from_scratch: `render` and the
three autograd Functions mirror src/cuda/wrapper.py, `cuda_rasterizer`
mirrors the reference's native module, and every computation runs in the
hand-written sm_100a kernels of lib3dgs_b200.so (C ABI: include/gs_b200.h).

The package directory name starts with a digit, so import it with
importlib.import_module("3dgs_from_scratch_b200").
"""
from . import _native
from . import cuda_rasterizer
from . import scenes
from .wrapper import ProjectPointsFunction, RasterizeFunction, SphericalHarmonicsFunction, render

__all__ = ["render", "ProjectPointsFunction", "SphericalHarmonicsFunction", "RasterizeFunction",
           "cuda_rasterizer", "scenes", "load_native", "native_path"]


def load_native():
    """Load lib3dgs_b200.so now (raises if it is missing or cannot load)."""
    return _native.lib()


def native_path() -> str:
    return _native.LIB_PATH
