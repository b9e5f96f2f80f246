"""The allocation-free select entry point, called through the C ABI.

mn_dtem_select_noalloc serves callers that cannot allocate device memory:
it keeps its scratch in a fixed array inside the library instead of a
caller-provided workspace.  Its results must equal those of mn_dtem_select
(the entry point that takes a workspace) call after call, including when the
shared scratch still holds the previous call's contents.  This file is
collected last so that a failure here leaves every other test already run.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(seed, batch, donors, slots, dev):
    g = torch.Generator().manual_seed(seed)
    scores = torch.randn(batch, donors, slots, generator=g)
    allowed = torch.rand(batch, donors, slots, generator=g) > 0.35
    allowed[:, :, 0] = True  # every row has a legal receiver: the budget is feasible
    return scores.to(dev), allowed.to(dev)


def _with_workspace(lib, scores, allowed, k):
    b, na, kk = scores.shape
    out = torch.empty_like(scores)
    nbytes = lib.mn_dtem_select_workspace_bytes(b, na)
    ws = torch.empty(int(nbytes), dtype=torch.uint8, device=scores.device)
    status = torch.zeros(1, dtype=torch.int32, device=scores.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(scores.device).cuda_stream)
    rc = lib.mn_dtem_select(b, na, kk, ctypes.c_void_p(scores.data_ptr()),
                            ctypes.c_void_p(allowed.view(torch.uint8).data_ptr()), k, 1.0, 30.0,
                            ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()), nbytes,
                            ctypes.c_void_p(status.data_ptr()), stream)
    assert rc == 0
    return out, status


def _without_allocation(lib, scores, allowed, k):
    b, na, kk = scores.shape
    out = torch.empty_like(scores)
    status = torch.zeros(1, dtype=torch.int32, device=scores.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(scores.device).cuda_stream)
    rc = lib.mn_dtem_select_noalloc(b, na, kk, ctypes.c_void_p(scores.data_ptr()),
                                    ctypes.c_void_p(allowed.view(torch.uint8).data_ptr()), k, 1.0, 30.0,
                                    ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(status.data_ptr()), stream)
    assert rc == 0
    return out, status


def test_noalloc_select_matches_workspace_select_twice():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from mergenet_b200 import _lib
    lib = _lib.lib()
    dev = torch.device("cuda", 0)
    # two calls in a row, different shapes and data: the second finds the
    # first call's leftovers in the shared scratch
    for seed, (batch, donors, slots, k) in [(11, (64, 392, 29, 65)), (12, (3, 50, 9, 7))]:
        scores, allowed = _inputs(seed, batch, donors, slots, dev)
        want, st_want = _with_workspace(lib, scores, allowed, k)
        got, st_got = _without_allocation(lib, scores, allowed, k)
        torch.cuda.synchronize()
        assert int(st_want.item()) == 0 and int(st_got.item()) == 0
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=0, atol=2e-6)


def test_noalloc_select_rejects_oversize():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from mergenet_b200 import _lib
    lib = _lib.lib()
    dev = torch.device("cuda", 0)
    x = torch.zeros(1, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    rows_over = 262144 // 392 + 1  # one batch row beyond the scratch
    rc = lib.mn_dtem_select_noalloc(rows_over, 392, 29, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                    65, 1.0, 30.0, ctypes.c_void_p(x.data_ptr()), None, stream)
    assert rc == _lib.MN_ERR_UNSUPPORTED
