"""gs_exclusive_scan_noalloc: the scan entry point for callers that may not
allocate device memory themselves (a host application that owns all GPU
memory, a frame loop that must not call cudaMalloc/cudaFree). It keeps its
look-back state in a fixed device array inside the library instead of
caller-provided scratch; these tests check, through the C ABI, that it
returns exactly what the allocating gs_exclusive_scan returns, on two calls
in a row (the array keeps the previous call's contents, which the entry
point must clear), and that it rejects sizes beyond its limit.

This file is collected last on purpose (tests/test_zz_*)."""
import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
MAX_N = 1 << 24


def scan_with_scratch(nat, counts):
    n = counts.numel()
    out = torch.empty(n, dtype=torch.int32, device=DEV)
    total = torch.zeros(1, dtype=torch.int64, device=DEV)
    nb = int(nat.query("gs_scan_scratch_bytes", n))
    scratch = torch.empty(max(nb, 8), dtype=torch.uint8, device=DEV)
    nat.call("gs_exclusive_scan", n, counts.data_ptr(), out.data_ptr(), total.data_ptr(),
             scratch.data_ptr(), nb, nat.stream_ptr())
    return out, total


def scan_noalloc(nat, counts):
    n = counts.numel()
    out = torch.empty(n, dtype=torch.int32, device=DEV)
    total = torch.zeros(1, dtype=torch.int64, device=DEV)
    rc = nat.query("gs_exclusive_scan_noalloc", n, counts.data_ptr(), out.data_ptr(),
                   total.data_ptr(), nat.stream_ptr())
    assert rc == 0, rc
    return out, total


def test_noalloc_scan_matches_allocating_scan_twice():
    nat = importlib.import_module("3dgs_from_scratch_b200._native")
    rng = np.random.default_rng(11)
    for n in (3_000_001, 4_097):  # a large call, then a smaller one over the stale array
        counts = torch.from_numpy(rng.integers(0, 40, n).astype(np.int32)).to(DEV)
        ref_out, ref_total = scan_with_scratch(nat, counts)
        out, total = scan_noalloc(nat, counts)
        torch.cuda.synchronize()
        assert nat.query("gs_check_status", nat.stream_ptr()) == 0
        assert torch.equal(out, ref_out)
        assert int(total.item()) == int(ref_total.item()) == int(counts.long().sum().item())
        expect = torch.cumsum(counts.long(), 0) - counts.long()
        assert torch.equal(out.long(), expect)


def test_noalloc_scan_allocates_nothing_and_launches_once():
    """The property the entry point exists for: after a warm-up call, a call
    leaves the device's free memory unchanged and adds exactly one kernel
    launch (the scan; the clearing of the array is a memset)."""
    nat = importlib.import_module("3dgs_from_scratch_b200._native")
    n = 2_000_003
    counts = torch.ones(n, dtype=torch.int32, device=DEV)
    out = torch.empty(n, dtype=torch.int32, device=DEV)
    total = torch.zeros(1, dtype=torch.int64, device=DEV)
    args = (n, counts.data_ptr(), out.data_ptr(), total.data_ptr(), nat.stream_ptr())
    assert nat.query("gs_exclusive_scan_noalloc", *args) == 0  # warm-up (symbol lookup)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    launches0 = nat.launch_count()
    assert nat.query("gs_exclusive_scan_noalloc", *args) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert nat.launch_count() - launches0 == 1
    assert free1 == free0
    assert int(total.item()) == n
    assert int(out[-1].item()) == n - 1


def test_noalloc_scan_limits():
    nat = importlib.import_module("3dgs_from_scratch_b200._native")
    total = torch.full((1,), 7, dtype=torch.int64, device=DEV)
    assert nat.query("gs_exclusive_scan_noalloc", 0, None, None, total.data_ptr(),
                     nat.stream_ptr()) == 0
    assert int(total.item()) == 0
    # beyond the fixed array: rejected before any launch, no pointer is touched
    assert nat.query("gs_exclusive_scan_noalloc", MAX_N + 1, None, None, total.data_ptr(),
                     nat.stream_ptr()) == nat.GS_ERR_CAPACITY
