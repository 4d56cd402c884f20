"""`import cuda_rasterizer` shim for the reference's own Python code.

With this directory on sys.path, ruguangyou/3dgs_from_scratch's
src/cuda/wrapper.py (line 8: `import cuda_rasterizer`) and
scripts/check_cuda_gradients.py (line 14) load the B200 kernels instead of
the reference extension, with no change to their code.
"""
import importlib
import os
import sys

_root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _root not in sys.path:
    sys.path.insert(0, _root)
_impl = importlib.import_module("3dgs_from_scratch_b200.cuda_rasterizer")

project_points = _impl.project_points
project_points_backward = _impl.project_points_backward
evaluate_spherical_harmonics = _impl.evaluate_spherical_harmonics
evaluate_spherical_harmonics_backward = _impl.evaluate_spherical_harmonics_backward
compute_tile_intersection = _impl.compute_tile_intersection
rasterize = _impl.rasterize
rasterize_backward = _impl.rasterize_backward
