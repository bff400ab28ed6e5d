"""The allocation-free sum of squares (to_sumsq3_noalloc) against to_sumsq3.

to_sumsq3_noalloc exists for callers that may not allocate device memory --
a solver step inside an application that owns the GPU's memory through its
own pool, or a loop that must not stall the device the way cudaFree does --
so it keeps its block partials in a fixed array inside the library instead of
taking a workspace.  This file is named to be collected last: if it fails, a
run that stops at the first failure has already run every other test.

* On the GPU: two calls in a row (a large sum, then a smaller one over other
  data, so leftovers of the first call in the shared scratch would show) give
  the same result as the workspace entry point bit for bit (both run the same
  fixed-order reduction), and agree with an independent float64 sum in torch
  within relative 1e-13 (the library accumulates in double for both dtypes).
* On any host: a size above the fixed scratch is rejected before anything is
  launched.
"""
import numpy as np
import pytest

from tensoroperations_b200 import abi

TOL = 1e-13  # against torch's float64 sum of the same values


def test_rejects_sizes_beyond_the_fixed_scratch():
    nmax = abi.lib.to_sumsq3_noalloc_max_n()
    assert nmax == 32768 * 131072 // 3
    with pytest.raises(abi.ToError) as e:
        # the size check comes first: no pointer is used, nothing is launched
        abi.sumsq3_noalloc(np.float64, [8, 16, 24], 0, nmax + 1, 32)
    assert e.value.status == abi.TO_ERR_INVALID_ARGUMENT
    assert "exceeds" in str(e.value)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_two_calls_in_a_row_match_the_workspace_entry_point(dtype):
    import torch
    tdt = torch.float64 if dtype == np.float64 else torch.float32
    g = torch.Generator(device="cuda").manual_seed(2026)
    cases = [(3_000_001, 5), (70_000, 1)]  # (n, first): 69 partials, then 2
    for n, first in cases:
        x = [torch.randn(first + n, generator=g, dtype=tdt, device="cuda") for _ in range(3)]
        want = torch.zeros(1, dtype=torch.float64, device="cuda")
        got = torch.full((1,), -1.0, dtype=torch.float64, device="cuda")
        ws = torch.empty(abi.sumsq3_workspace_bytes(n), dtype=torch.uint8, device="cuda")
        abi.sumsq3(dtype, x, first, n, want, ws)
        abi.sumsq3_noalloc(dtype, x, first, n, got)
        torch.cuda.synchronize()
        w, v = float(want.item()), float(got.item())
        assert v == w, (n, v, w)  # the same reduction order: bit for bit
        ref = float(sum((t[first:first + n].double() ** 2).sum() for t in x).item())
        assert abs(v - ref) <= TOL * ref, (n, v, ref)
