"""The tcgen05 GEMM (TMA + TMEM, kind::f16 and kind::f8f6f4) against an fp32 PyTorch reference (GPU only)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def C():
    from glm53.ops import _ext
    return _ext.require()


@pytest.mark.parametrize("M,N,K", [(128, 256, 512), (200, 300, 1024), (1000, 4096, 4096), (64, 128, 128)])
def test_gemm_bf16(C, M, N, K):
    torch.manual_seed(M + N)
    a = torch.randn(M, K, device=DEV).to(torch.bfloat16)
    b = (torch.randn(N, K, device=DEV) / math.sqrt(K)).to(torch.bfloat16)
    ref = a.float() @ b.float().t()
    y = torch.zeros(M, N, device=DEV)
    C.gemm_bf16(a, b, None, y, 1, 0.0)
    torch.cuda.synchronize()
    assert C.gemm_error(y) == 0
    torch.testing.assert_close(y, ref, atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("M,N,K", [(128, 256, 512), (300, 1000, 2048), (2048, 4096, 4096)])
def test_gemm_w8a8(C, M, N, K):
    from glm53.models.weights import quantize_fp8_rows
    torch.manual_seed(K)
    w = quantize_fp8_rows(torch.randn(N, K) / math.sqrt(K))
    x = torch.randn(M, K).to(torch.bfloat16)
    amax = x.float().abs().amax(1, keepdim=True).clamp_min(1e-8)
    xs = amax / 448.0
    xq = (x.float() / xs).to(torch.float8_e4m3fn).float() * xs
    ref = xq @ w.dequant().t()
    y = torch.zeros(M, N, device=DEV)
    C.gemm_w8(x.to(DEV), w.w.to(DEV), w.s.to(DEV), y, 1, 0.0)
    torch.cuda.synchronize()
    assert C.gemm_error(y) == 0
    torch.testing.assert_close(y.cpu(), ref, atol=3e-3, rtol=3e-3)
    yb = torch.zeros(M, N, device=DEV, dtype=torch.bfloat16)
    C.gemm_w8(x.to(DEV), w.w.to(DEV), w.s.to(DEV), yb, 0, 0.0)
    torch.testing.assert_close(yb.float().cpu(), ref, atol=3e-2, rtol=3e-2)


def test_gemm_swiglu(C):
    from glm53.models.runtime import interleave_gate_up
    from glm53.models.weights import quantize_fp8_rows
    from glm53.models.reference import swiglu
    torch.manual_seed(0)
    M, W, K = 256, 512, 1024
    gu = quantize_fp8_rows(torch.randn(2 * W, K) / math.sqrt(K))
    x = torch.randn(M, K).to(torch.bfloat16)
    amax = x.float().abs().amax(1, keepdim=True).clamp_min(1e-8)
    xq = (x.float() / (amax / 448)).to(torch.float8_e4m3fn).float() * (amax / 448)
    full = xq @ gu.dequant().t()
    ref = swiglu(full[:, :W].to(torch.bfloat16).float(), full[:, W:].to(torch.bfloat16).float(), 10.0)
    il = interleave_gate_up(gu)
    y = torch.zeros(M, W, device=DEV, dtype=torch.bfloat16)
    C.gemm_w8(x.to(DEV), il.w.to(DEV), il.s.to(DEV), y, 3, 10.0)
    torch.testing.assert_close(y.float().cpu(), ref, atol=5e-2, rtol=5e-2)


@pytest.mark.parametrize("M,N,K", [(64, 128, 256), (300, 1000, 2048)])
def test_gemm_w8a16(C, M, N, K):
    """Exact-weight path: fp8 widened to bf16, bf16 activations, per-row scale epilogue."""
    from glm53.models.weights import quantize_fp8_rows
    torch.manual_seed(K + 1)
    w = quantize_fp8_rows(torch.randn(N, K) / math.sqrt(K))
    x = torch.randn(M, K).to(torch.bfloat16)
    ref = x.float() @ w.dequant().t()
    y = torch.zeros(M, N, device=DEV)
    scratch = torch.empty(N * K, dtype=torch.bfloat16, device=DEV)
    C.gemm_w8a16(x.to(DEV), w.w.to(DEV), w.s.to(DEV), y, 1, 0.0, scratch)
    torch.cuda.synchronize()
    assert C.gemm_error(y) == 0
    torch.testing.assert_close(y.cpu(), ref, atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("M,N,K", [(2500, 3000, 512), (130, 8200, 256)])
def test_gemm_persistent_accumulate_and_bf16_out(C, M, N, K):
    """Many tiles per CTA (persistent schedule, both TMEM accumulators reused), fp32 accumulate into an existing
    output and bf16 output with ragged M/N edges (scalar tail stores next to 16-byte stores)."""
    torch.manual_seed(7)
    a = torch.randn(M, K, device=DEV).to(torch.bfloat16)
    b = (torch.randn(N, K, device=DEV) / math.sqrt(K)).to(torch.bfloat16)
    ref = a.float() @ b.float().t()
    base = torch.randn(M, N, device=DEV)
    y = base.clone()
    C.gemm_bf16(a, b, None, y, 2, 0.0)                       # GEMV_F32_ACC
    yb = torch.zeros(M, N, device=DEV, dtype=torch.bfloat16)
    C.gemm_bf16(a, b, None, yb, 0, 0.0)                      # GEMV_BF16
    torch.cuda.synchronize()
    assert C.gemm_error(y) == 0
    torch.testing.assert_close(y, base + ref, atol=2e-3, rtol=2e-3)
    torch.testing.assert_close(yb.float(), ref, atol=2e-2, rtol=2e-2)


def test_gemm_w8a16_batched_per_head_views(C):
    """Batched (per-head) GEMM on strided views, the layout of the absorbed MLA projections at prefill:
    x = q[:, :, :nope].transpose(0, 1) ([H, R, nope] with row stride H*qk), y = q_lat.transpose(0, 1)."""
    from glm53.models.weights import quantize_fp8_rows
    torch.manual_seed(11)
    R, H, nope, rope, L = 300, 6, 64, 32, 128
    q = torch.randn(R, H, nope + rope, device=DEV).to(torch.bfloat16)
    w = quantize_fp8_rows(torch.randn(H, L, nope) / math.sqrt(nope))
    ref = torch.einsum("rhk,hnk->rhn", q[:, :, :nope].float().cpu(), w.dequant())
    y = torch.zeros(R, H, L, device=DEV, dtype=torch.bfloat16)
    scratch = torch.empty(w.w.numel(), dtype=torch.bfloat16, device=DEV)
    C.gemm_w8a16(q[:, :, :nope].transpose(0, 1), w.w.to(DEV), w.s.to(DEV), y.transpose(0, 1), 0, 0.0, scratch)
    torch.cuda.synchronize()
    assert C.gemm_error(y) == 0
    torch.testing.assert_close(y.float().cpu(), ref, atol=2e-2, rtol=2e-2)
