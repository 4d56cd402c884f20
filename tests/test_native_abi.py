"""The C-ABI library: it loads, exports every entry point declared in
include/gs_b200.h, the ctypes signatures match the header, and host-only
queries behave. No kernel is launched here."""
import ctypes
import importlib
import os
import re

import pytest
import torch

from conftest import REPO

HEADER = os.path.join(REPO, "include", "gs_b200.h")


def declared():
    src = open(HEADER).read()
    out = {}
    for m in re.finditer(r"GS_API\s+(\w+)\s+(gs_\w+)\(([^;]*)\);", src, re.S):
        params = m.group(3).strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        out[m.group(2)] = (m.group(1), n)
    return out


def test_header_declares_entry_points():
    d = declared()
    assert len(d) >= 20
    for name in ("gs_project_points", "gs_project_points_backward", "gs_evaluate_sh",
                 "gs_evaluate_sh_backward", "gs_tile_layout", "gs_rasterize",
                 "gs_rasterize_backward", "gs_sort_pairs", "gs_preprocess_forward",
                 "gs_preprocess_backward", "gs_blend_forward", "gs_blend_backward"):
        assert name in d


def test_library_exports_every_declared_symbol(gs):
    lib = ctypes.CDLL(gs.native_path())
    for name in declared():
        assert hasattr(lib, name), name


def test_ctypes_signatures_match_header(gs):
    from importlib import import_module

    nat = import_module("3dgs_from_scratch_b200._native")
    d = declared()
    assert set(nat.SIGNATURES) == set(d)
    for name, (_, nparams) in d.items():
        assert len(nat.SIGNATURES[name][1]) == nparams, name


def test_host_queries(gs):
    lib = gs.load_native()
    assert lib.gs_version() >= 1
    assert lib.gs_launch_count() >= 0
    a = lib.gs_sort_scratch_bytes(10_000)
    b = lib.gs_sort_scratch_bytes(10_000_000)
    assert 0 < a < b
    assert lib.gs_tile_layout_scratch_bytes(100, 1000, 64, 64) > 1000 * 6
    assert lib.gs_scan_scratch_bytes(100_000) >= 8


def test_product_path_has_no_cpu_fallback(gs):
    n = 8
    z = torch.zeros
    with pytest.raises(RuntimeError):
        gs.render(torch.eye(4), torch.eye(3), 16, 16, z(n, 3), z(n, 3), z(n, 4), z(n), z(n, 3),
                  z(n, 15, 3))


def test_entry_points_reject_bad_arguments_before_touching_a_device(gs):
    """Size and pointer checks come first: these calls return
    GS_ERR_INVALID_ARGUMENT (1) without a GPU."""
    lib = gs.load_native()
    nat = importlib.import_module("3dgs_from_scratch_b200._native")
    bad = nat.GS_ERR_INVALID_ARGUMENT
    P = None
    assert lib.gs_preprocess_forward_views(10, 0, *[P] * 9, 0.01, 100.0, 0.0, 0.5, 128.0, 16, 16,
                                           0, 1, *[P] * 8) == bad          # no views
    assert lib.gs_preprocess_backward_views(10, 2, *[P] * 9, 0, 16, 0, 1, 0, P, P, 2, P, 8,
                                            *[P] * 6, P) == bad            # width 0
    assert lib.gs_ssim_forward(0, 16, 16, P, P, 1, P, 0, P, P) == bad      # no planes
    assert lib.gs_ssim_forward(1, 8, 64, P, P, 1, P, 0, P, P) == bad       # valid needs > 10 rows
    assert lib.gs_l1_ssim_loss_grad(8, 64, P, P, 0, 0.2, P, P, P, 0, P) == bad
    assert lib.gs_dp_adam_step(0, 0, P, P, P, P, P, 16, P, P, 6, P, P, P, 0.9, 0.999, 1, 1, 1,
                               P, P) == bad                                # world 0
    assert lib.gs_densify_accumulate(-1, P, P, 16, 16, P, P, P) == bad
    assert lib.gs_reset_opacities(-1, P, P, P, 0.0, P) == bad
    assert lib.gs_l1_loss_grad(-1, P, P, 0, P, P, P) == bad
