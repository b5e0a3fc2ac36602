"""The allocation-free greedy pick (b200_argmax_f32_noalloc), through the C ABI.

Some callers cannot allocate device memory -- code running while a CUDA graph
is captured, callers whose device memory all comes from their own allocator,
processes that forbid allocation after start-up -- and opening an engine
allocates. This entry point keeps its scratch in a fixed array inside the
library instead. The test checks it against the engine's b200_argmax_f32 on
the same inputs, bit for bit (the tolerance every parity test here uses), on
two calls in a row, and that sizes beyond its limit are refused. The file
name sorts last so a run that stops at the first failure has run every other
test before this one.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LIMIT = 1 << 25


def _pick_engine(torch, pkg, eng, y, base):
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    eng.argmax(y, y.numel(), out, index_base=base)
    eng.sync()
    return out.cpu().numpy().copy()


def _pick_noalloc(torch, pkg, y, base, stream):
    out = torch.full((2,), -1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    rc = pkg.lib().b200_argmax_f32_noalloc(int(y.data_ptr()), y.numel(), base, int(out.data_ptr()),
                                           ctypes.c_void_p(stream))
    assert rc == 0, pkg.lib().b200_last_error()
    torch.cuda.synchronize()
    return out.cpu().numpy().copy()


def test_no_alloc_pick_matches_the_engine_pick_on_two_calls(cuda_lib, pkg):
    import torch
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    eng = pkg.Engine(0)
    rng = np.random.default_rng(5)
    cases = []
    for n, base in [(128256, 7), (16032, 3 * 16032)]:
        ynp = rng.standard_normal(n).astype(np.float32)
        ynp[n // 5] = ynp[n // 2] = ynp.max() + 0.5        # a tie: the lower index wins
        y = torch.from_numpy(ynp).cuda()
        cases.append((ynp, y, base, _pick_engine(torch, pkg, eng, y, base)))
    # two calls of the new entry point in a row (the second reuses the scratch the first left)
    got = [_pick_noalloc(torch, pkg, y, base, stream.cuda_stream) for _, y, base, _ in cases]
    for (ynp, _, base, want), g in zip(cases, got):
        n = ynp.size
        assert np.array_equal(g, want)
        assert int(g[0]) - base == n // 5
        assert g[1:2].view(np.float32)[0] == ynp[n // 5]
    eng.close()


def test_no_alloc_pick_refuses_sizes_beyond_its_limit(cuda_lib, pkg):
    import torch
    y = torch.zeros(16, device="cuda")
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    rc = pkg.lib().b200_argmax_f32_noalloc(int(y.data_ptr()), LIMIT + 1, 0, int(out.data_ptr()), None)
    assert rc == -22
    assert b"limit" in pkg.lib().b200_last_error()


def _scan(y: np.ndarray) -> int:
    """The reference's pick (tp_llama.cpp:879-882): best = 0, then i wins only if y[i] > y[best]."""
    best = 0
    for i in range(1, y.size):
        if y[i] > y[best]:
            best = i
    return best


@pytest.mark.parametrize("case", ["nan_at_0", "nan_inside", "small_one_cta", "single"])
def test_no_alloc_pick_edge_inputs(cuda_lib, pkg, case):
    """NaN at index 0 (the scan never leaves it), NaN elsewhere (never picked),
    a vector small enough for one CTA, and n = 1: the engine's pick and the
    reference's scan, restated."""
    import torch
    rng = np.random.default_rng(11)
    n = {"nan_at_0": 5000, "nan_inside": 70000, "small_one_cta": 1000, "single": 1}[case]
    ynp = rng.standard_normal(n).astype(np.float32)
    if case == "nan_at_0":
        ynp[0] = np.nan
    if case == "nan_inside":
        ynp[123] = np.nan
        ynp[60000] = np.nan
    y = torch.from_numpy(ynp).cuda()
    eng = pkg.Engine(0)
    want = _pick_engine(torch, pkg, eng, y, 0)
    got = _pick_noalloc(torch, pkg, y, 0, 0)
    eng.close()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert int(got[0]) == _scan(ynp)
