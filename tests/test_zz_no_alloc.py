"""dflash_qmm_noalloc: the matmul for callers that cannot allocate device memory.

Such callers (code recorded inside a CUDA graph someone else captures, plugin hosts
that forbid touching the allocator, latency-critical loops) get the same result as
dflash_qmm with a caller-owned workspace; the scratch is the library's static device
array instead.  This file is collected after every other test, so a run stopping at its
first failure has already run them; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-2  # the same north-star bound the other qmm tests use


def _dev(a, d):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(d).view(torch.bfloat16)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).to(d)
    return torch.from_numpy(a).to(d)


@pytest.mark.parametrize("M,N,K,group,bits", [(8, 17408, 5120, 64, 4), (12, 5120, 17408, 32, 8)])
def test_noalloc_matches_workspace_entry_point_twice(dc, O, cuda, M, N, K, group, bits):
    import torch
    x, wq, s, b = O.make_qmm_case(M, N, K, group, bits, seed_x=31, seed_w=32)
    xd, wd, sd, bd = _dev(x, cuda), _dev(wq, cuda), _dev(s, cuda), _dev(b, cuda)
    ref = dc.qmm(xd, wd, sd, bd, group, bits)
    torch.cuda.synchronize()
    for _ in range(2):  # the static scratch keeps the previous call's contents
        y = dc.qmm_noalloc(xd, wd, sd, bd, group, bits)
        torch.cuda.synchronize()
        assert O.closeness(y.float().cpu().numpy(), ref.float().cpu().numpy()) <= TOL
        assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
    rows = np.arange(0, N, 113)
    want = O.qmm_f64(x, wq[rows], s[rows], b[rows], group, bits)
    assert O.closeness(y.float().cpu().numpy()[:, rows], want) <= TOL
    assert dc.device_error() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch(dc, cuda):
    import torch
    K = 1 << 20  # x in fragment order alone would need 32 MiB
    x = torch.zeros((16, K), dtype=torch.bfloat16, device=cuda)
    w = torch.zeros((1, K // 8), dtype=torch.int32, device=cuda)
    s = torch.zeros((1, K // 64), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(dc.DFlashError) as e:
        dc.qmm_noalloc(x, w, s, s, 64, 4)
    assert e.value.status == dc.DFLASH_ERR_UNSUPPORTED
    assert "static" in dc.last_error()
