"""mt_diff_reduce_noalloc — the comparison entry point that allocates nothing.

It serves callers that must not allocate device memory: a host binding of
the C ABI that only holds buffers lent to it, or a verification check that
runs while the memory pool is deliberately filled with NaNs, where scratch
allocation would disturb the pool under test. Its scratch is a static device
array inside libmt.so, shared by every call on a device.

Checked here through the C ABI (ctypes, no Python wrapper) against the
workspace entry point mt_diff_reduce on two calls in a row, with the same
tolerance the other diff-reduction tests use: the statistics must be equal
field for field (same kernel, same block partition). Kept in a file pytest
collects last so a failure here never hides another test's result.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from metal_autotune_b200 import lib

pytestmark = pytest.mark.gpu

FIELDS = [name for name, _ in lib.DiffStats._fields_]


def _noalloc(a, b, rtol, atol):
    mt = lib.load()
    stats = torch.zeros(C.sizeof(lib.DiffStats), dtype=torch.uint8, device=a.device)
    rc = mt.mt_diff_reduce_noalloc(a.data_ptr(), b.data_ptr(), a.numel(), lib.dtype_code(a.dtype), rtol, atol, 0.0,
                                   stats.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, mt.mt_last_error_string()
    return lib.read_diff_stats(stats)


def _with_workspace(a, b, rtol, atol):
    return lib.read_diff_stats(lib.diff_reduce(a, b, rtol=rtol, atol=atol))


def test_noalloc_matches_workspace_entry_on_two_calls(cuda):
    rng = np.random.default_rng(77)
    cases = [(300_001, torch.float32, 1e-3, 1e-3), (1 << 20, torch.bfloat16, 2e-2, 4e-2)]
    for n, dt, rtol, atol in cases:  # two calls in a row, the second reuses the scratch of the first
        ref = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(dt).cuda()
        cand = (ref.float() + torch.from_numpy(rng.standard_normal(n).astype(np.float32) * 0.01).cuda()).to(dt)
        cand[n // 2] = ref[n // 2].float() + 1.0
        got = _noalloc(cand, ref, rtol, atol)
        want = _with_workspace(cand, ref, rtol, atol)
        for f in FIELDS:
            assert getattr(got, f) == getattr(want, f), f
        assert got.over_count > 0 and got.excess_index >= 0


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    mt = lib.load()
    n = 1048576 + 1
    a = torch.zeros(n, device="cuda")
    stats = torch.zeros(C.sizeof(lib.DiffStats), dtype=torch.uint8, device="cuda")
    rc = mt.mt_diff_reduce_noalloc(a.data_ptr(), a.data_ptr(), n, lib.MT_F32, 0.0, 0.0, 0.0, stats.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream)
    assert rc == -1
    assert b"static scratch maximum" in mt.mt_last_error_string()
