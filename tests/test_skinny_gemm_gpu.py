"""GPU numerics of the tcgen05 skinny GEMM (y = x w^T) against a PyTorch fp32 matmul."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from kvbm_b200.ops import llama_ops


def _check(M, N, K, ctas, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g)
    w = (torch.randn(N, K, device="cuda", dtype=torch.bfloat16, generator=g) / K ** 0.5).to(torch.bfloat16)
    ref = x.float() @ w.float().t()
    y = llama_ops.skinny_gemm(x, w, ctas=ctas)
    torch.cuda.synchronize()
    assert llama_ops.skinny_gemm_status() == 0
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)
    return x, w, ref


@pytest.mark.parametrize("M,N,K,ctas", [
    (1, 128, 64, 0),        # one tile, one K chunk, BN = 16
    (16, 256, 1024, 1),     # one CTA walks both tiles whole
    (16, 256, 1024, 3),     # 32 chunks over 3 CTAs: tiles shared through the workspace
    (7, 384, 4096, 0),      # rows of x past M read as zeros
    (32, 512, 4096, 5),     # BN = 32
    (33, 1000, 520, 1),     # N and K not multiples of the tile (BN = 64)
    (33, 1000, 520, 7),
    (128, 256, 2048, 0),    # BN = 128 (6-stage ring), 2-chunk ranges
    (128, 1024, 4096, 11),
])
def test_skinny_gemm_matches_fp32(M, N, K, ctas):
    _check(M, N, K, ctas)


@pytest.mark.parametrize("M,N,K", [
    (1, 128, 64),        # one tile, one chunk: a cluster of one
    (16, 256, 1024),
    (7, 384, 4096),
    (32, 512, 4096),
    (33, 1000, 520),     # ragged N and K, BN = 64
    (128, 1024, 4096),   # BN = 128 (4-stage ring)
    (32, 6144, 4096),    # Llama-3-8B qkv
    (32, 4096, 14336),   # Llama-3-8B down
])
def test_skinny_gemm_cluster_matches_fp32(M, N, K):
    prev = llama_ops.set_skinny_gemm_mode("cluster")
    try:
        for _ in range(2):  # the second launch reuses nothing from the first
            _check(M, N, K, 0, seed=M + N)
    finally:
        llama_ops.set_skinny_gemm_mode(prev)


def test_skinny_gemm_default_ctas_and_rearm():
    # repeated launches with shared tiles: the kernel leaves workspace and tickets zeroed
    M, N, K = 32, 4096, 14336
    x, w, ref = _check(M, N, K, 0, seed=1)
    for _ in range(3):
        y = llama_ops.skinny_gemm(x, w)
    torch.cuda.synchronize()
    assert llama_ops.skinny_gemm_status() == 0
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)
    ws = llama_ops._workspaces[torch.cuda.current_device()]
    assert int(ws.tickets.abs().sum()) == 0
    assert float(ws.ws.abs().sum()) == 0.0


def test_skinny_gemm_strided_operands():
    # x rows taken from a wider buffer, output into a column slice of a wider buffer
    M, N, K = 8, 640, 768
    buf = torch.randn(M, K + 64, device="cuda", dtype=torch.bfloat16)
    x = buf[:, 32:32 + K]
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    out = torch.zeros(M, N + 128, device="cuda", dtype=torch.bfloat16)
    llama_ops.skinny_gemm(x, w.to(torch.bfloat16), out=out[:, 64:64 + N])
    torch.cuda.synchronize()
    ref = x.float() @ w.to(torch.bfloat16).float().t()
    torch.testing.assert_close(out[:, 64:64 + N].float(), ref, rtol=2e-2, atol=2e-2)
    assert float(out[:, :64].abs().sum()) == 0.0 and float(out[:, 64 + N:].abs().sum()) == 0.0


@pytest.mark.parametrize("pdl", [True, False])
def test_skinny_gemm_after_rmsnorm_in_graph(pdl):
    # the GEMM reads the norm's output: with programmatic dependent launch it may start
    # early but must still see that output, eagerly and inside a captured graph
    prev = llama_ops.set_skinny_gemm_pdl(pdl)
    try:
        M, K, N = 32, 4096, 6144
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        g = torch.rand(K, device="cuda", dtype=torch.bfloat16) + 0.5
        w = (torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5).to(torch.bfloat16)
        h = torch.empty_like(x)
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)

        def step():
            llama_ops.rmsnorm(x, g, 1e-5, out=h)
            llama_ops.skinny_gemm(h, w, out=y)

        step()
        torch.cuda.synchronize()
        torch.testing.assert_close(y.float(), h.float() @ w.float().t(), rtol=2e-2, atol=2e-2)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(3):
            x.copy_(torch.randn_like(x))
            graph.replay()
            torch.cuda.synchronize()
            ref_h = llama_ops.rmsnorm(x, g, 1e-5)
            torch.testing.assert_close(h, ref_h)
            torch.testing.assert_close(y.float(), ref_h.float() @ w.float().t(), rtol=2e-2, atol=2e-2)
        assert llama_ops.skinny_gemm_status() == 0
    finally:
        llama_ops.set_skinny_gemm_pdl(prev)
