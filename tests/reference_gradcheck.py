"""Run the reference's own gradient regression harness
(scripts/check_cuda_gradients.py of ruguangyou/3dgs_from_scratch, lines
1016-1048) against this library, through the `cuda_rasterizer` and
`fused_ssim` drop-in modules (3dgs_from_scratch_b200/dropin).

Test infrastructure: tests/test_gpu_reference_gradcheck.py starts this file
in a fresh interpreter. The harness and the reference modules it imports are
the byte-compiled copies oracle/build_ref.py stages under oracle/_ref/py
(imported by their reference names through build_ref's staged-module
finder); the harness runs unchanged, with its own argument parser
(e.g. `--seeds 7 --skip-real-train-loss`).

Two packages that the reference's src/dataset.py imports at module level,
pycolmap and imageio, are absent here; they are only used by the real-data
check (`check_end_to_end_real_train_loss`, which needs COLMAP data that does
not exist here and is skipped with --skip-real-train-loss), so empty stand-in
modules satisfy the import.
"""
from __future__ import annotations

import os
import runpy
import sys
import types

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DROPIN = os.path.join(REPO, "3dgs_from_scratch_b200", "dropin")
sys.path.insert(0, REPO)
from oracle import build_ref  # noqa: E402

HARNESS = build_ref.staged_file("scripts/check_cuda_gradients.py")


def _stub_absent(name: str, **attrs) -> None:
    try:
        __import__(name)
    except ImportError:
        mod = types.ModuleType(name)
        for k, v in attrs.items():
            setattr(mod, k, v)
        sys.modules[name] = mod


def main(argv) -> None:
    if not os.path.exists(HARNESS):
        raise SystemExit(f"reference harness not staged: {HARNESS} (oracle/build_ref.py)")
    sys.path.insert(0, DROPIN)
    build_ref.install_staged_importer()
    _stub_absent("pycolmap", SceneManager=object)
    _stub_absent("imageio")
    if "imageio.v2" not in sys.modules:
        try:
            __import__("imageio.v2")
        except ImportError:
            v2 = types.ModuleType("imageio.v2")
            sys.modules["imageio.v2"] = v2
            sys.modules["imageio"].v2 = v2
    import cuda_rasterizer  # noqa: E402  (the drop-in, first on the path)
    import fused_ssim  # noqa: E402,F401

    print(f"cuda_rasterizer from {cuda_rasterizer.__file__}", flush=True)
    sys.argv = ["check_cuda_gradients.py"] + list(argv)
    runpy.run_path(HARNESS, run_name="__main__")
    nat = sys.modules.get("3dgs_from_scratch_b200._native")
    if nat is not None:
        print(f"native library {nat.LIB_PATH}, launches {nat.launch_count()}", flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])
