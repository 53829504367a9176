"""dflash_qmm_host: x and y in host memory, one call per matmul (copy in, matmul, copy
out on the stream).  Its result must be the bits dflash_qmm gives on device buffers."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import verify_stack as vs



@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,group,bits", [(8, 4096, 1024, 64, 4), (1, 4096, 1024, 64, 4),
                                              (16, 5120, 2048, 32, 8), (5, 1000, 640, 128, 4)])
@pytest.mark.parametrize("pinned", [True, False])
def test_qmm_host_equals_device_qmm(dc, cuda, M, N, K, group, bits, pinned):
    gen = torch.Generator(device=cuda).manual_seed(M + N)
    q = vs.random_quant(gen, N, K, group, bits, cuda)
    x = torch.randn(M, K, generator=gen, device=cuda).to(torch.bfloat16)
    want = dc.qmm(x, q.w, q.scales, q.biases, group, bits)
    x_host = x.cpu()
    y_host = torch.empty(M, N, dtype=torch.bfloat16)
    if pinned:
        x_host, y_host = x_host.pin_memory(), y_host.pin_memory()
    side = torch.cuda.Stream(cuda)
    ws = dc.Workspace(dc.qmm_host_workspace_bytes(M, N, K, group, bits), cuda)
    with torch.cuda.stream(side):
        dc.qmm_host(x_host, q.w, q.scales, q.biases, group, bits, out_host=y_host, workspace=ws)
    side.synchronize()
    torch.cuda.synchronize()
    assert torch.equal(y_host, want.cpu())
    assert dc.device_error() == 0


@pytest.mark.gpu
def test_qmm_host_consecutive_calls_on_two_streams(dc, cuda):
    """Pipelined use as the end-to-end benchmark does: calls alternate between two
    streams, each with its own workspace and host output."""
    M, N, K = 8, 4096, 2048
    gen = torch.Generator(device=cuda).manual_seed(9)
    qs = [vs.random_quant(gen, N, K, 64, 4, cuda) for _ in range(3)]
    xs = [torch.randn(M, K, generator=gen, device=cuda).to(torch.bfloat16) for _ in range(6)]
    wants = [dc.qmm(xs[i], qs[i % 3].w, qs[i % 3].scales, qs[i % 3].biases, 64, 4).cpu() for i in range(6)]
    streams = [torch.cuda.Stream(cuda), torch.cuda.Stream(cuda)]
    wss = [dc.Workspace(dc.qmm_host_workspace_bytes(M, N, K, 64, 4), cuda) for _ in range(2)]
    x_hosts = [x.cpu().pin_memory() for x in xs]
    y_hosts = [torch.empty(M, N, dtype=torch.bfloat16).pin_memory() for _ in range(6)]
    torch.cuda.synchronize()
    for i in range(6):
        with torch.cuda.stream(streams[i & 1]):
            q = qs[i % 3]
            dc.qmm_host(x_hosts[i], q.w, q.scales, q.biases, 64, 4, out_host=y_hosts[i], workspace=wss[i & 1])
    torch.cuda.synchronize()
    for i in range(6):
        assert torch.equal(y_hosts[i], wants[i]), i
    assert np.isfinite(y_hosts[0].float().numpy()).all()
