"""`from fused_ssim import fused_ssim` shim for the reference's scripts.

With this directory on sys.path, scripts/train.py (line 6) and
scripts/evaluate.py (line 4) take SSIM from this library's kernels.
"""
import importlib
import os
import sys

_root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _root not in sys.path:
    sys.path.insert(0, _root)
fused_ssim = importlib.import_module("3dgs_from_scratch_b200.ssim").fused_ssim
