"""Numerics of each CUDA kernel against a plain fp32 PyTorch reference of the same op (GPU only)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def C():
    from glm53.ops import _ext
    return _ext.require()


def test_exl3_unpack_bitexact(C):
    from glm53.ops import exl3
    g = torch.Generator().manual_seed(1)
    tr, _, _ = exl3.random_linear(256, 384, generator=g)
    ref = exl3.unpack(tr)
    out = C.exl3_unpack(tr.to(DEV), 256, 384).cpu()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("M", [1, 3, 8, 11, 16])
@pytest.mark.parametrize("N,K", [(64, 128), (900, 512), (2048, 4096)])
def test_gemv_fp8(C, M, N, K):
    from glm53.models.weights import quantize_fp8_rows
    from glm53.ops import kernels as Kk
    torch.manual_seed(M * 7 + N)
    w = quantize_fp8_rows(torch.randn(N, K) / math.sqrt(K))
    x = torch.randn(M, K).to(torch.bfloat16)
    ref = x.float() @ w.dequant().t()
    wd, sd, xd = w.w.to(DEV), w.s.to(DEV), x.to(DEV)
    y = torch.empty(M, N, dtype=torch.float32, device=DEV)
    Kk.C().gemv(xd, wd, sd, y, Kk.GEMV_F32, 0.0)
    torch.testing.assert_close(y.cpu(), ref, atol=2e-3, rtol=2e-3)
    yb = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    Kk.C().gemv(xd, wd, sd, yb, Kk.GEMV_BF16, 0.0)
    torch.testing.assert_close(yb.float().cpu(), ref, atol=2e-2, rtol=2e-2)
    acc = torch.ones(M, N, dtype=torch.float32, device=DEV)
    Kk.C().gemv(xd, wd, sd, acc, Kk.GEMV_F32_ACC, 0.0)
    torch.testing.assert_close(acc.cpu(), ref + 1, atol=2e-3, rtol=2e-3)


def test_gemv_swiglu_and_batched(C):
    from glm53.models.runtime import interleave_gate_up
    from glm53.models.weights import quantize_fp8_rows
    from glm53.models.reference import swiglu
    from glm53.ops import kernels as Kk
    torch.manual_seed(0)
    W, Kd, M = 256, 512, 8
    gu = quantize_fp8_rows(torch.randn(2 * W, Kd) / math.sqrt(Kd))
    x = torch.randn(M, Kd).to(torch.bfloat16)
    full = x.float() @ gu.dequant().t()
    g, u = full[:, :W].to(torch.bfloat16).float(), full[:, W:].to(torch.bfloat16).float()
    ref = swiglu(g, u, 10.0)
    il = interleave_gate_up(gu)
    y = torch.empty(M, W, dtype=torch.bfloat16, device=DEV)
    Kk.C().gemv(x.to(DEV), il.w.to(DEV), il.s.to(DEV), y, Kk.GEMV_SWIGLU, 10.0)
    torch.testing.assert_close(y.float().cpu(), ref, atol=3e-2, rtol=3e-2)
    # batched: [B, N, K] weights, per-batch strided inputs / outputs
    Bn, N2, K2 = 4, 128, 64
    wb = quantize_fp8_rows(torch.randn(Bn, N2, K2) / 8)
    xb = torch.randn(M, Bn, 96).to(torch.bfloat16)            # use [:, :, :64] as a strided view
    ref = torch.einsum("mbk,bnk->mbn", xb[:, :, :K2].float(), wb.dequant())
    yb = torch.empty(M, Bn, N2, dtype=torch.float32, device=DEV)
    xd = xb.to(DEV)
    Kk.C().gemv(xd[:, :, :K2].transpose(0, 1), wb.w.to(DEV), wb.s.to(DEV), yb.transpose(0, 1), Kk.GEMV_F32, 0.0)
    torch.testing.assert_close(yb.cpu(), ref, atol=2e-3, rtol=2e-3)


def test_gemv_bf16(C):
    from glm53.ops import kernels as Kk
    torch.manual_seed(3)
    x = torch.randn(5, 512).to(torch.bfloat16)
    w = (torch.randn(288, 512) / 20).to(torch.bfloat16)
    ref = x.float() @ w.float().t()
    y = torch.empty(5, 288, device=DEV)
    Kk.linear_bf16(x.to(DEV), w.to(DEV), y)
    torch.testing.assert_close(y.cpu(), ref, atol=1e-3, rtol=1e-3)


def _moe_ref(moe, cfg, x):
    from glm53.models import reference as R
    out = torch.zeros(x.shape[0], cfg.hidden)
    ids, w = R.route(x, moe, cfg)
    for r in range(x.shape[0]):
        for k in range(cfg.top_k):
            out[r] += w[r, k] * R.expert_forward(moe, int(ids[r, k]), x[r:r + 1], cfg)[0]
    return out, ids


@pytest.mark.parametrize("rows", [1, 8, 37])
def test_moe_routed_exl3(C, tiny_cfg, tiny_weights, rows):
    from glm53.models.runtime import Runtime, RuntimeConfig
    cfg = tiny_cfg
    lw = next(l for l in tiny_weights.layers if l.moe is not None)
    w = tiny_weights
    torch.manual_seed(rows)
    x = torch.randn(rows, cfg.hidden).to(torch.bfloat16)
    ref, ids = _moe_ref(lw.moe, cfg, x.float())
    wd = _to_dev(w)
    rt = Runtime(wd, RuntimeConfig(max_rows=64, kv_slots=256, max_blocks=4))
    m = wd.layers[lw.index].moe
    from glm53.ops import kernels as Kk
    Kc = Kk.C()
    xd = x.to(DEV)
    P = rows * cfg.top_k
    G = min(P, cfg.experts)
    Kk.linear_bf16(xd, m.router, rt.rlogits[:rows])
    Kc.moe_route(rt.rlogits[:rows], m.bias, cfg.top_k, cfg.routed_scale, cfg.norm_topk, rt.topk_ids[:rows],
                 rt.topk_w[:rows], rt.group_count, rt.group_expert[:G], rt.group_offset[:G + 1], rt.pair_token[:P],
                 rt.pair_expert[:P], rt.pair_w[:P], rt.pair_of[:P])
    assert torch.equal(rt.topk_ids[:rows].cpu().long(), ids)
    Kc.exl3_moe(xd, m.gate.trellis, m.gate.suh, m.gate.svh, m.up.trellis, m.up.suh, m.up.svh, m.down.trellis,
                m.down.suh, m.down.svh, rt.group_count, rt.group_expert[:G], rt.group_offset[:G + 1],
                rt.pair_token[:P], rt.pair_expert[:P], rt.pair_w[:P], rt.xh_g, rt.xh_u, rt.xd, rt.yd, cfg.limit)
    out = torch.empty(rows, cfg.hidden, device=DEV)
    Kc.moe_combine(rt.yd, rt.pair_of[:P], cfg.top_k, out, 0)
    torch.testing.assert_close(out.cpu(), ref, atol=2e-2, rtol=2e-2)
    # with the gate/up CTAs prefetching other weights into L2 (a hint): the same bits
    y1 = rt.yd[:P].clone()
    Kc.exl3_moe(xd, m.gate.trellis, m.gate.suh, m.gate.svh, m.up.trellis, m.up.suh, m.up.svh, m.down.trellis,
                m.down.suh, m.down.svh, rt.group_count, rt.group_expert[:G], rt.group_offset[:G + 1],
                rt.pair_token[:P], rt.pair_expert[:P], rt.pair_w[:P], rt.xh_g, rt.xh_u, rt.xd, rt.yd, cfg.limit,
                [m.down.trellis, m.router], 1 << 20)
    assert torch.equal(rt.yd[:P], y1)


def _to_dev(w):
    import copy
    from glm53.models import weights as W

    def conv(o):
        if isinstance(o, torch.Tensor):
            return o.to(DEV)
        if isinstance(o, list):
            return [conv(v) for v in o]
        if hasattr(o, "__dataclass_fields__"):
            o2 = copy.copy(o)
            for k in o.__dataclass_fields__:
                setattr(o2, k, conv(getattr(o, k)))
            return o2
        return o
    return conv(w)


def test_hc_post_pre(C, tiny_cfg, tiny_weights):
    from glm53.models import reference as R
    cfg = tiny_cfg
    lw = tiny_weights.layers[1]
    torch.manual_seed(5)
    Rr, S, D = 6, cfg.streams, cfg.hidden
    X = torch.randn(Rr, S, D).to(torch.bfloat16)
    branch = torch.randn(Rr, D)
    pre0, post0, comb0 = R.hc_mix(X.float(), lw.attn_hc.fn, lw.attn_hc.base, lw.attn_hc.scale, S, cfg.eps,
                                  cfg.hc_eps, cfg.hc_iters)
    Xn = R.hc_post(X.float(), branch, post0, comb0)
    normed_ref, post_ref, comb_ref = R.hc_pre(Xn, lw.ffn_hc, lw.post_norm, cfg)
    Xd = X.to(DEV).contiguous()
    normed = torch.empty(Rr, D, dtype=torch.bfloat16, device=DEV)
    post = torch.empty(Rr, S, device=DEV)
    comb = torch.empty(Rr, S, S, device=DEV)
    part = torch.empty(Rr, D // 64, 32, device=DEV)
    C.hc_post_pre(Xd, branch.to(DEV), post0.to(DEV), comb0.to(DEV), lw.ffn_hc.fn.to(DEV), lw.ffn_hc.base.to(DEV),
                  lw.ffn_hc.scale.to(DEV), lw.post_norm.to(DEV), normed, post, comb, part, cfg.eps, cfg.hc_eps,
                  cfg.hc_iters)
    torch.testing.assert_close(Xd.float().cpu(), Xn, atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(post.cpu(), post_ref, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(comb.cpu(), comb_ref, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(normed.float().cpu(), normed_ref, atol=3e-2, rtol=2e-2)


def test_dsa_select_radix(C):
    """Radix top-k over pool logits equals a stable sort (ties -> lower index), expanded to token slots."""
    torch.manual_seed(0)
    kp, P, bs = 4, 16, 64
    pos = 700
    c = pos // kp
    logits = torch.randn(1, 256)
    logits[0, 10] = logits[0, 11] = logits[0, 12] = 5.0      # ties
    from glm53.ops import kernels as Kk
    Kc = Kk.C()
    iproj = torch.zeros(1, 2 * 128 + 4, device=DEV)
    qi = torch.zeros(1, 4 * 128, dtype=torch.bfloat16, device=DEV)
    # run the select kernel alone by passing precomputed logits: zero pools give zero logits, so write the logits
    # after the logits kernel through a custom path: use pool cache = 0 and compare with the expected dense rule
    pool = torch.zeros(1024, 128, dtype=torch.uint8, device=DEV)
    ps = torch.ones(1024, device=DEV)
    bt = torch.arange(16, dtype=torch.int32, device=DEV).view(1, 16)
    out_l = torch.zeros(1, 256, device=DEV)
    sel = torch.zeros(1, P * kp, dtype=torch.int32, device=DEV)
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    positions = torch.tensor([pos], dtype=torch.int32, device=DEV)
    rs = torch.zeros(1, dtype=torch.int32, device=DEV)
    Kc.dsa_select(iproj, qi, torch.ones(128, device=DEV), pool, ps, positions, bt, rs, bs, 4, kp, P, out_l, sel, cnt)
    # all-zero logits: ties everywhere -> the lowest P-1 pools are chosen
    n = int(cnt.item())
    assert n == (P - 1) * kp + (pos % kp) + 1
    exp = list(range((P - 1) * kp)) + list(range(c * kp, pos + 1))
    assert sel[0, :n].cpu().tolist() == exp


@pytest.mark.parametrize("rows", [80, 300])
def test_moe_prefill_tcgen05_matches_oracle(C, tiny_cfg, tiny_weights, rows):
    """The prefill MoE path (scalable routing + tcgen05 grouped GEMMs with shared-memory trellis decode) against
    the fp32 oracle; 300 rows x top-4 over 16 experts gives experts > 64 tokens (several TMA boxes)."""
    from glm53.models.runtime import Runtime, RuntimeConfig
    cfg = tiny_cfg
    lw = next(l for l in tiny_weights.layers if l.moe is not None)
    torch.manual_seed(rows)
    x = torch.randn(rows, cfg.hidden).to(torch.bfloat16)
    ref, _ = _moe_ref(lw.moe, cfg, x.float())
    wd = _to_dev(tiny_weights)
    rt = Runtime(wd, RuntimeConfig(max_rows=512, kv_slots=256, max_blocks=4))
    rt.normed[:rows].copy_(x.to(DEV))
    rt.branch.zero_()
    rt._moe_prefill(wd.layers[lw.index], rows)
    torch.cuda.synchronize()
    assert C.gemm_error(rt.branch) == 0
    torch.testing.assert_close(rt.branch[:rows].cpu(), ref, atol=2e-2, rtol=2e-2)


def test_moe_prefill_many_tokens_per_expert(C, tiny_cfg, tiny_weights):
    """More than 256 tokens on one expert (two passes of the kernel): all rows routed to the same experts."""
    from glm53.models.runtime import Runtime, RuntimeConfig
    import dataclasses
    cfg = tiny_cfg
    lw = next(l for l in tiny_weights.layers if l.moe is not None)
    moe = dataclasses.replace(lw.moe, bias=lw.moe.bias.clone())
    moe.bias[:] = -100.0
    moe.bias[[1, 5, 9, 12]] = 100.0                 # every row picks experts 1, 5, 9, 12
    rows = 400
    torch.manual_seed(1)
    x = torch.randn(rows, cfg.hidden).to(torch.bfloat16)
    ref, ids = _moe_ref(moe, cfg, x.float())
    assert set(ids.flatten().tolist()) == {1, 5, 9, 12}
    wd = _to_dev(tiny_weights)
    lwd = wd.layers[lw.index]
    lwd.moe = dataclasses.replace(lwd.moe, bias=moe.bias.to(DEV))
    rt = Runtime(wd, RuntimeConfig(max_rows=512, kv_slots=256, max_blocks=4))
    rt.normed[:rows].copy_(x.to(DEV))
    rt._moe_prefill(lwd, rows)
    torch.cuda.synchronize()
    assert C.gemm_error(rt.branch) == 0
    torch.testing.assert_close(rt.branch[:rows].cpu(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("rows", [300, 1024])
@pytest.mark.parametrize("with_post", [True, False])
def test_hc_post_pre_tensor_cores(C, rows, with_post):
    """Prefill-sized mHC (4 streams, D = 4096): the tcgen05 partial pass (post + 24 mixing dots on the tensor
    cores, 512-column blocks) against the fp32 reference and against the CUDA-core kernel."""
    from types import SimpleNamespace
    from glm53.models import reference as R
    S, D = 4, 4096
    g = torch.Generator().manual_seed(7)
    X = (torch.randn(rows, S, D, generator=g)).to(torch.bfloat16)
    branch = torch.randn(rows, D, generator=g)
    fn = (torch.randn(2 * S + S * S, S * D, generator=g) * 0.02).to(torch.bfloat16)
    base = torch.randn(2 * S + S * S, generator=g) * 0.1
    scale = torch.tensor([1.0, 0.8, 1.2])
    norm_w = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    post0 = torch.rand(rows, S, generator=g) * 2
    comb0 = torch.softmax(torch.randn(rows, S, S, generator=g), -1)
    cfg = SimpleNamespace(streams=S, eps=1e-6, hc_eps=1e-6, hc_iters=20)
    Xn = R.hc_post(X.float(), branch, post0, comb0) if with_post else X.float()
    normed_ref, post_ref, comb_ref = R.hc_pre(Xn, SimpleNamespace(fn=fn, base=base, scale=scale), norm_w.float(),
                                              cfg)
    outs = {}
    for tcores in (1, 0):
        Xd = X.to(DEV).contiguous()
        normed = torch.empty(rows, D, dtype=torch.bfloat16, device=DEV)
        post = torch.empty(rows, S, device=DEV)
        comb = torch.empty(rows, S, S, device=DEV)
        part = torch.empty(rows, D // 64, 32, device=DEV)
        C.hc_post_pre(Xd, branch.to(DEV) if with_post else None, post0.to(DEV) if with_post else None,
                      comb0.to(DEV) if with_post else None, fn.to(DEV), base.to(DEV), scale.to(DEV), norm_w.to(DEV),
                      normed, post, comb, part, cfg.eps, cfg.hc_eps, cfg.hc_iters, tcores)
        torch.cuda.synchronize()
        outs[tcores] = (Xd.float().cpu(), normed.float().cpu(), post.cpu(), comb.cpu())
    Xt, nt, pt, ct = outs[1]
    torch.testing.assert_close(Xt, Xn, atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(Xt, outs[0][0], atol=0, rtol=0)          # same post arithmetic, bit for bit
    torch.testing.assert_close(pt, post_ref, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(ct, comb_ref, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(nt, normed_ref, atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(pt, outs[0][2], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("rows", [1, 8, 16])
@pytest.mark.parametrize("with_post", [True, False])
def test_hc_post_pre_decode_cluster(C, rows, with_post):
    """Decode-sized mHC (4 streams, D = 4096) in one cluster kernel (8 CTAs per row, the row reductions through
    distributed shared memory) against the fp32 reference, and the post arithmetic bit for bit against the
    two-kernel path (prefill-sized launch of the same rows padded to 300)."""
    from types import SimpleNamespace
    from glm53.models import reference as R
    S, D = 4, 4096
    g = torch.Generator().manual_seed(11 + rows)
    X = (torch.randn(rows, S, D, generator=g)).to(torch.bfloat16)
    branch = torch.randn(rows, D, generator=g)
    fn = (torch.randn(2 * S + S * S, S * D, generator=g) * 0.02).to(torch.bfloat16)
    base = torch.randn(2 * S + S * S, generator=g) * 0.1
    scale = torch.tensor([1.0, 0.8, 1.2])
    norm_w = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    post0 = torch.rand(rows, S, generator=g) * 2
    comb0 = torch.softmax(torch.randn(rows, S, S, generator=g), -1)
    cfg = SimpleNamespace(streams=S, eps=1e-6, hc_eps=1e-6, hc_iters=20)
    Xn = R.hc_post(X.float(), branch, post0, comb0) if with_post else X.float()
    normed_ref, post_ref, comb_ref = R.hc_pre(Xn, SimpleNamespace(fn=fn, base=base, scale=scale), norm_w.float(),
                                              cfg)
    Xd = X.to(DEV).contiguous()
    normed = torch.empty(rows, D, dtype=torch.bfloat16, device=DEV)
    post = torch.empty(rows, S, device=DEV)
    comb = torch.empty(rows, S, S, device=DEV)
    part = torch.empty(rows, D // 64, 32, device=DEV)
    C.hc_post_pre(Xd, branch.to(DEV) if with_post else None, post0.to(DEV) if with_post else None,
                  comb0.to(DEV) if with_post else None, fn.to(DEV), base.to(DEV), scale.to(DEV), norm_w.to(DEV),
                  normed, post, comb, part, cfg.eps, cfg.hc_eps, cfg.hc_iters, 0)
    torch.cuda.synchronize()
    torch.testing.assert_close(Xd.float().cpu(), Xn, atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(post.cpu(), post_ref, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(comb.cpu(), comb_ref, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(normed.float().cpu(), normed_ref, atol=3e-2, rtol=2e-2)
    # the same rows through the two-kernel path (a 300-row launch): identical post, close pre outputs
    pad = 300
    Xp = torch.zeros(pad, S, D, dtype=torch.bfloat16)
    Xp[:rows] = X
    bp, p0, c0 = torch.zeros(pad, D), torch.zeros(pad, S), torch.zeros(pad, S, S)
    bp[:rows], p0[:rows], c0[:rows] = branch, post0, comb0
    Xpd = Xp.to(DEV)
    n2 = torch.empty(pad, D, dtype=torch.bfloat16, device=DEV)
    po2, co2 = torch.empty(pad, S, device=DEV), torch.empty(pad, S, S, device=DEV)
    pa2 = torch.empty(pad, D // 64, 32, device=DEV)
    C.hc_post_pre(Xpd, bp.to(DEV) if with_post else None, p0.to(DEV) if with_post else None,
                  c0.to(DEV) if with_post else None, fn.to(DEV), base.to(DEV), scale.to(DEV), norm_w.to(DEV),
                  n2, po2, co2, pa2, cfg.eps, cfg.hc_eps, cfg.hc_iters, 0)
    torch.cuda.synchronize()
    assert torch.equal(Xpd[:rows].cpu(), Xd.cpu())
    torch.testing.assert_close(po2[:rows], post, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(co2[:rows], comb, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("M", [1, 8, 12])
@pytest.mark.parametrize("N,K", [(24896, 4096), (4100, 8192), (4096, 16384)])
def test_gemv_fp8_large_default_dispatch(C, M, N, K):
    """Large projections through the default dispatch (the bulk-copy kernel for up to 8 rows or K <= 4096, the
    split-K kernel otherwise; a partial last tile for N = 4100): all output modes against the fp32 reference, and
    two launches in a row give identical bits."""
    from glm53.models.weights import quantize_fp8_rows
    from glm53.ops import kernels as Kk
    g = torch.Generator(device=DEV).manual_seed(M * 13 + N)
    wf = torch.randn(N, K, device=DEV, generator=g) / math.sqrt(K)
    w = quantize_fp8_rows(wf)
    x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    ref = x.float() @ w.dequant().t()
    y = torch.empty(M, N, dtype=torch.float32, device=DEV)
    Kk.C().gemv(x, w.w, w.s, y, Kk.GEMV_F32, 0.0)
    torch.testing.assert_close(y, ref, atol=2e-3, rtol=2e-3)
    y2 = torch.empty_like(y)
    Kk.C().gemv(x, w.w, w.s, y2, Kk.GEMV_F32, 0.0)
    assert torch.equal(y, y2)
    yb = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    Kk.C().gemv(x, w.w, w.s, yb, Kk.GEMV_BF16, 0.0)
    torch.testing.assert_close(yb.float(), ref, atol=2e-2, rtol=2e-2)
    acc = torch.ones(M, N, dtype=torch.float32, device=DEV)
    Kk.C().gemv(x, w.w, w.s, acc, Kk.GEMV_F32_ACC, 0.0)
    torch.testing.assert_close(acc, ref + 1, atol=2e-3, rtol=2e-3)


def test_gemv_swiglu_large_default_dispatch(C):
    """The interleaved SwiGLU output mode at the dense MLP's size (100 MB of fp8 weights) through the default
    dispatch."""
    from glm53.models.runtime import interleave_gate_up
    from glm53.models.weights import quantize_fp8_rows
    from glm53.models.reference import swiglu
    from glm53.ops import kernels as Kk
    torch.manual_seed(1)
    Wd, Kd, M = 12288, 4096, 8
    gu = quantize_fp8_rows(torch.randn(2 * Wd, Kd) / math.sqrt(Kd))
    x = torch.randn(M, Kd).to(torch.bfloat16)
    full = x.float() @ gu.dequant().t()
    gg, uu = full[:, :Wd].to(torch.bfloat16).float(), full[:, Wd:].to(torch.bfloat16).float()
    ref = swiglu(gg, uu, 10.0)
    il = interleave_gate_up(gu)
    y = torch.empty(M, Wd, dtype=torch.bfloat16, device=DEV)
    Kk.C().gemv(x.to(DEV), il.w.to(DEV), il.s.to(DEV), y, Kk.GEMV_SWIGLU, 10.0)
    torch.testing.assert_close(y.float().cpu(), ref, atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("M", [1, 8, 13, 16])
@pytest.mark.parametrize("N,K", [(1000, 3072), (520, 1024), (272, 2048), (4096, 8192), (1000, 12288),
                                 (24896, 4096)])
def test_gemv_fp8_bulk(C, M, N, K):
    """The bulk-copy (TMA ring) decode projection, forced (ks=-1): every output mode against the fp32 reference
    (partial last tiles for N=1000, 520 and 272; 1, 2 and 4 KB stages; activations register-resident or streamed
    from L2 by K and row count), and two launches in a row give identical bits."""
    from glm53.models.weights import quantize_fp8_rows
    from glm53.ops import kernels as Kk
    g = torch.Generator(device=DEV).manual_seed(M * 31 + N + K)
    w = quantize_fp8_rows(torch.randn(N, K, device=DEV, generator=g) / math.sqrt(K))
    x = torch.randn(M, K, device=DEV, generator=g).to(torch.bfloat16)
    ref = x.float() @ w.dequant().t()
    y = torch.empty(M, N, dtype=torch.float32, device=DEV)
    Kk.C().gemv(x, w.w, w.s, y, Kk.GEMV_F32, 0.0, -1, 0)
    torch.testing.assert_close(y, ref, atol=2e-3, rtol=2e-3)
    y2 = torch.full_like(y, float("nan"))
    Kk.C().gemv(x, w.w, w.s, y2, Kk.GEMV_F32, 0.0, -1, 0)
    assert torch.equal(y, y2)
    yb = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    Kk.C().gemv(x, w.w, w.s, yb, Kk.GEMV_BF16, 0.0, -1, 0)
    torch.testing.assert_close(yb.float(), ref, atol=2e-2, rtol=2e-2)
    acc = torch.ones(M, N, dtype=torch.float32, device=DEV)
    Kk.C().gemv(x, w.w, w.s, acc, Kk.GEMV_F32_ACC, 0.0, -1, 0)
    torch.testing.assert_close(acc, ref + 1, atol=2e-3, rtol=2e-3)
    # a strided activation view (rows of a wider buffer) and an output with a row pitch
    xw = torch.zeros(M, K + 64, device=DEV, dtype=torch.bfloat16)
    xw[:, :K] = x
    yw = torch.zeros(M, N + 16, device=DEV)
    Kk.C().gemv(xw[:, :K], w.w, w.s, yw[:, :N], Kk.GEMV_F32, 0.0, -1, 0)
    assert torch.equal(yw[:, :N], y) and (yw[:, N:] == 0).all()
    assert Kk.C().gemm_error(x) == 0                     # no bounded wait ran out


@pytest.mark.parametrize("M", [1, 8, 16])
def test_gemv_swiglu_bulk(C, M):
    from glm53.models.runtime import interleave_gate_up
    from glm53.models.weights import quantize_fp8_rows
    from glm53.models.reference import swiglu
    from glm53.ops import kernels as Kk
    torch.manual_seed(2)
    Wd, Kd = 2048, 4096
    gu = quantize_fp8_rows(torch.randn(2 * Wd, Kd) / math.sqrt(Kd))
    x = torch.randn(M, Kd).to(torch.bfloat16)
    full = x.float() @ gu.dequant().t()
    gg, uu = full[:, :Wd].to(torch.bfloat16).float(), full[:, Wd:].to(torch.bfloat16).float()
    ref = swiglu(gg, uu, 10.0)
    il = interleave_gate_up(gu)
    y = torch.empty(M, Wd, dtype=torch.bfloat16, device=DEV)
    Kk.C().gemv(x.to(DEV), il.w.to(DEV), il.s.to(DEV), y, Kk.GEMV_SWIGLU, 10.0, -1, 0)
    torch.testing.assert_close(y.float().cpu(), ref, atol=3e-2, rtol=3e-2)


def test_l2_prefetch_leaves_results_unchanged(C):
    """The L2 prefetch paths are hints only: the standalone prefetch kernel and the MoE gate/up CTAs' prefetch of
    other weights change no result bit of the routed experts."""
    from glm53.ops import kernels as Kk
    g = torch.Generator(device=DEV).manual_seed(5)
    a = torch.randn(3000, 1024, device=DEV, generator=g).to(torch.bfloat16)
    b = torch.randn(777 * 16, device=DEV, generator=g)
    Kk.C().l2_prefetch([a, b], 1 << 30)
    Kk.C().l2_prefetch([a], 4096)
    torch.cuda.synchronize()
    assert Kk.C().gemm_error(a) == 0


@pytest.mark.parametrize("T,blk", [(8, 8), (12, 5), (1, 8)])
def test_dconv_matches_eager_chain(C, T, blk):
    """The drafter's grouped dynamic conv kernel equals the eager bf16 op chain bit for bit (per-row kernel deltas
    shared by channel groups, causal taps masked at draft-block boundaries)."""
    from glm53.ops import kernels as Kk
    H, taps, gs = 512, 3, 64
    g = torch.Generator(device=DEV).manual_seed(T * 7 + blk)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    delta = (0.1 * torch.randn(T, taps, H // gs, device=DEV, generator=g)).to(torch.bfloat16)
    base = (0.5 * torch.randn(taps, H, device=DEV, generator=g)).to(torch.bfloat16)
    out = torch.empty(T, H, device=DEV, dtype=torch.bfloat16)
    Kk.C().dconv(x, delta, base, out, gs, blk)
    pos = torch.arange(T, device=DEV) % blk
    ck = base[None] + delta.repeat_interleave(gs, -1)              # [T, taps, H] bf16
    ref = ck[:, 0] * x
    for k in range(1, taps):
        xs = torch.zeros_like(x)
        if T > k:
            xs[k:] = x[:-k]
        p = ck[:, k] * xs
        p = p * (pos >= k)[:, None].to(torch.bfloat16)
        ref = ref + p
    assert torch.equal(out, ref)


@pytest.mark.parametrize("K", [256, 4096])
def test_rot_in_wide_matches_narrow_bitexact(C, K):
    """The 16-byte rotated-input kernel of the prefill layout (a half-warp per 128-column block) against the
    warp-per-block kernel (taken for an x whose row stride is not a multiple of 8): bit-identical f16 outputs,
    including pairs that repeat a token and experts out of order."""
    g = torch.Generator(device=DEV).manual_seed(7)
    T, E, P = 37, 5, 150
    x_wide = torch.randn(T, K + 4, device=DEV, generator=g).to(torch.bfloat16)
    x_narrow = x_wide[:, :K]                      # row stride K + 4: the narrow kernel
    x_dense = x_narrow.contiguous()               # row stride K: the wide kernel
    suh_g = (torch.randn(E, K, device=DEV, generator=g) * 0.5).to(torch.float16)
    suh_u = (torch.randn(E, K, device=DEV, generator=g) * 0.5).to(torch.float16)
    pt = torch.randint(0, T, (P,), device=DEV, generator=g).to(torch.int32)
    pe = torch.randint(0, E, (P,), device=DEV, generator=g).to(torch.int32)
    outs = []
    for x in (x_narrow, x_dense):
        xg = torch.full((P, K), float("nan"), device=DEV, dtype=torch.float16)
        xu = torch.full((P, K), float("nan"), device=DEV, dtype=torch.float16)
        C.exl3_rot_in(x, suh_g, suh_u, pt, pe, xg, xu)
        outs.append((xg, xu))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][0].view(torch.int16), outs[1][0].view(torch.int16))
    assert torch.equal(outs[0][1].view(torch.int16), outs[1][1].view(torch.int16))
    # and the rotation itself: H128 (x * suh) per 128-column block, fp32 reference
    i = torch.arange(128)
    parity = torch.tensor([bin(v).count("1") & 1 for v in (i[:, None] & i[None, :]).flatten().tolist()])
    H = (1 - 2 * parity.view(128, 128)).float().to(DEV) / 128 ** 0.5    # Sylvester order: H[i, j] = (-1)^|i & j|
    xs = (x_dense.float()[pt.long()] * suh_g.float()[pe.long()]).view(P, K // 128, 128)
    ref = (xs @ H.T).view(P, K)
    torch.testing.assert_close(outs[1][0].float(), ref, rtol=2e-3, atol=2e-3)
