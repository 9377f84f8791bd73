"""Thin Python wrappers over the CUDA extension (glm53_C).  Every wrapper launches on the current CUDA stream and
works on preallocated outputs, so a sequence of calls can be captured in a CUDA graph."""

from __future__ import annotations

import os

import torch

from . import _ext

# the tcgen05 GEMM serves M >= GEMM_MIN_M rows (set GLM53_TCGEN05_GEMM=0 to route large M through the small-M kernel)
GEMM_ENABLED = os.environ.get("GLM53_TCGEN05_GEMM", "1") == "1"
# large-M fp8 projections: exact W8A16 (weights widened to bf16, bf16 activations: the numerics of the decode
# kernel), except the projections listed in GLM53_PREFILL_W8A8, which quantise their activations per row to e4m3
# (kind::f8f6f4, 2x tensor throughput, different numerics).  The default is the reference's production choice:
# the KDA input projection and the MLA output projection (its GLM53_DENSE_W8A8_ONLY=kda.in_proj_qkvbfg_a,
# mla.o_proj); "all" = every large-M fp8 projection, "none" = exact W8A16 everywhere.
_W8A8 = os.environ.get("GLM53_PREFILL_W8A8", "kda_in_proj,mla_o_proj").strip().lower()
PREFILL_W8A8 = _W8A8 in ("1", "all")
W8A8_PROJ = set() if _W8A8 in ("0", "none", "") else {p.strip() for p in _W8A8.split(",")}
_scratch: dict = {}


def _w_scratch(numel: int, device) -> torch.Tensor:
    t = _scratch.get(device)
    if t is None or t.numel() < numel:
        t = torch.empty(numel, dtype=torch.bfloat16, device=device)
        _scratch[device] = t
    return t


def reserve_gemm_scratch(numel: int, device) -> None:
    """Allocate the W8A16 widening scratch up front (before CUDA-graph capture or large allocations)."""
    _w_scratch(numel, torch.device(device))

GEMV_BF16, GEMV_F32, GEMV_F32_ACC, GEMV_SWIGLU = 0, 1, 2, 3
DSA_RING = 32            # tail-ring positions per sequence of the DSA index keys (kDsaRing in csrc/launchers.h)
GEMV_MAX_M = 16
GEMM_MIN_M = 64          # rows from which the tcgen05 GEMM replaces the small-M kernel


def C():
    return _ext.require()


def linear8(x: torch.Tensor, w: torch.Tensor, s: torch.Tensor, y: torch.Tensor, mode: int = GEMV_BF16,
            limit: float = 0.0, proj: str | None = None) -> torch.Tensor:
    """y[M, N] (mode) = x[M, K] @ (w8[N, K] * s)^T for any M (chunks of 16 rows through the small-M kernel, or
    the large-M GEMM when it is available).  Batched form: x [B, M, K], w [B, N, K], s [B, N], y [B, M, N] (per
    attention head; any batch and row strides with contiguous rows).  `proj` names the projection for the W8A8
    policy of large-M calls (GLM53_PREFILL_W8A8)."""
    M = x.shape[-2]
    g = C().gemv
    if M <= GEMV_MAX_M:
        g(x, w, s, y, mode, limit)
        return y
    if GEMM_ENABLED and M >= GEMM_MIN_M:
        if (PREFILL_W8A8 or proj in W8A8_PROJ) and x.dim() == 2:
            C().gemm_w8(x, w, s, y, mode, limit)
        else:
            C().gemm_w8a16(x, w, s, y, mode, limit, _w_scratch(w.numel(), x.device))
        return y
    for m0 in range(0, M, GEMV_MAX_M):
        m1 = min(M, m0 + GEMV_MAX_M)
        g(x[..., m0:m1, :], w, s, y[..., m0:m1, :], mode, limit)
    return y


def w8a8_large_m(proj: str) -> bool:
    """True when a large-M call of projection `proj` runs W8A8 (activations quantised per row to e4m3)."""
    return GEMM_ENABLED and (PREFILL_W8A8 or proj in W8A8_PROJ)


def linear_bf16(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """y fp32 [M, N] = x bf16 [M, K] @ w bf16 [N, K]^T."""
    M = x.shape[0]
    if GEMM_ENABLED and M >= GEMM_MIN_M and x.stride(-1) == 1:
        C().gemm_bf16(x, w, None, y, GEMV_F32, 0.0)
        return y
    for m0 in range(0, M, GEMV_MAX_M):
        m1 = min(M, m0 + GEMV_MAX_M)
        C().gemv(x[m0:m1], w, None, y[m0:m1], GEMV_F32, 0.0)
    return y
