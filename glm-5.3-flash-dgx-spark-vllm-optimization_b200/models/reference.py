"""fp32 reference implementation of the GLM-5.3-Flash architecture (the oracle for every kernel and for the GPU
model).  It runs on any device in plain torch, one token at a time, using the same prepared weights as the GPU
runtime (fp8 per-channel dense projections, EXL3 routed experts) and rounding to bf16 / fp16 / fp8 at the same
points the GPU kernels store those types.

Math of one decoder layer (structure as in code/fork/docs/ref/tf_forward.py:278-301 and tf_glue.py:1-20):

  mHC pre   flat = X (S streams of D, bf16); r = rsqrt(mean(flat^2) + eps); mix = r * (fn @ flat)
            pre = sigmoid(mix[:S]*a0 + base) + hc_eps; post = 2*sigmoid(mix[S:2S]*a1 + base)
            comb = Sinkhorn(softmax_rows(mix[2S:]*a2 + base) + hc_eps), ``hc_iters`` alternations (cols first)
            normed = bf16(rmsnorm(bf16(sum_s pre_s X_s)) * w)
  mHC post  X_s = bf16(post_s * bf16(branch) + sum_j comb[j, s] X_j)
  KDA       p = in_proj(x) -> q,k,v (causal depthwise conv, 4 taps, SiLU), f = f_b(f_a), gate = g_b(g_a), b
            per head: q,k l2-normalised (q scaled by Dh^-1/2); g = lower * sigmoid(exp(A_log) * (f + dt_bias));
            S = S * exp(g) (per key channel); v' = sigmoid(b) * (v - S k); S += v' k^T; o = S q;
            o = rmsnorm(o) * o_norm * sigmoid(gate); out = o_proj(o)
            (recurrence: code/fork/glm53_kda_lazy.py:160-178)
  MLA       absorbed: q_lat_h = q_nope_h @ W_uk_h (per head, into the kv_lora latent), latent c = rmsnorm(kv_a(x))
            stored fp8 e4m3 with one fp32 scale per token, rope part (if any) bf16; scores over the DSA-selected
            keys, softmax, o_h = (sum p c) @ W_uv_h^T, out = o_proj(o)
  DSA       index key = LayerNorm(wk x); pools of ``kpool`` keys: per channel softmax(gate x + ape) weights ->
            pooled key -> Hadamard-128 -> e4m3 with a power-of-two scale; query = Hadamard(wq_b(q_res)) per head;
            pool logit = sum_h relu(q_h . k_pool) * w_h / sqrt(IH * ID); a query sees its own pool and the top
            (index_topk/kpool - 1) earlier complete pools (all keys while t < index_topk)
            (pool compression: code/fork/tests/kpoolring/ref/kpool_compress_vllm58454.py:139-257)
  MoE       scores = sigmoid(x @ router^T); top-k of scores + bias (ties: lower id); w = score / sum * scale;
            y = sum_k w_k E_k(x) + shared(x); E_k: EXL3 SwiGLU with clamp ``limit``
            (routing: code/fork/docs/ref/tf_glue.py:371-400)
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from ..config import ModelConfig
from ..ops import exl3 as exl3_ops
from .weights import Linear8, Weights, LayerW

bf16 = torch.bfloat16


def rb(x: torch.Tensor) -> torch.Tensor:
    """Round to bf16 and back to fp32."""
    return x.to(bf16).float()


def rh(x: torch.Tensor) -> torch.Tensor:
    return x.half().float()


def lin8(x: torch.Tensor, w: Linear8) -> torch.Tensor:
    """x [.., K] fp32 @ W^T with W = fp8 rows * scale: fp32 result (the GEMV accumulates in fp32)."""
    return (x.float() @ w.w.view(torch.float8_e4m3fn).float().t()) * w.s.float()


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def silu(x):
    return x * torch.sigmoid(x)


def swiglu(g: torch.Tensor, u: torch.Tensor, limit: float) -> torch.Tensor:
    g = torch.clamp(g, max=limit)
    u = torch.clamp(u, -limit, limit)
    return silu(g) * u


def fp8_quant_token(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row e4m3 quantisation with scale amax/448: (fp8 values as fp32, scale)."""
    amax = x.abs().amax(-1, keepdim=True).clamp_min(1e-8)
    s = amax / 448.0
    q = (x / s).clamp(-448, 448).to(torch.float8_e4m3fn).float()
    return q, s.squeeze(-1)


def fp8_quant_pow2(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row e4m3 quantisation with a power-of-two scale (ceil(log2(amax/448))), amax floored at 1e-4."""
    amax = x.abs().amax(-1, keepdim=True).clamp_min(1e-4)
    s = torch.exp2(torch.ceil(torch.log2(amax / 448.0)))
    q = (x / s).clamp(-448, 448).to(torch.float8_e4m3fn).float()
    return q, s.squeeze(-1)


def hadamard128(x: torch.Tensor) -> torch.Tensor:
    return exl3_ops.rotate(x.float(), -1)


def rope(x: torch.Tensor, pos: int | torch.Tensor, theta: float) -> torch.Tensor:
    """Rotate-half RoPE over the last dim (pairs (i, i + d/2))."""
    d = x.shape[-1]
    if d == 0:
        return x
    half = d // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float32, device=x.device) / half))
    pos_t = torch.as_tensor(pos, dtype=torch.float32, device=x.device)
    ang = pos_t[..., None] * inv
    cos, sin = torch.cos(ang), torch.sin(ang)
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)


# ---------------------------------------------------------------------------------------------------------------
# mHC
# ---------------------------------------------------------------------------------------------------------------
def sinkhorn(logits: torch.Tensor, iters: int, eps: float) -> torch.Tensor:
    """logits [.., S, S] -> doubly-(approximately) stochastic comb: softmax over each row + eps, then column
    normalisation, then (iters-1) x (row normalisation, column normalisation)."""
    c = torch.softmax(logits, -1) + eps
    c = c / (c.sum(-2, keepdim=True) + eps)
    for _ in range(iters - 1):
        c = c / (c.sum(-1, keepdim=True) + eps)
        c = c / (c.sum(-2, keepdim=True) + eps)
    return c


def hc_mix(X: torch.Tensor, fn: torch.Tensor, base: torch.Tensor, scale: torch.Tensor, S: int, eps: float,
           hc_eps: float, iters: int):
    """X [R, S, D] (bf16 values) -> pre [R, S], post [R, S], comb [R, S, S]."""
    R = X.shape[0]
    flat = X.reshape(R, -1).float()
    r = torch.rsqrt(flat.pow(2).mean(-1, keepdim=True) + eps)
    mix = (flat @ fn.float().t()) * r
    pre = torch.sigmoid(mix[:, :S] * scale[0] + base[:S]) + hc_eps
    post = 2.0 * torch.sigmoid(mix[:, S:2 * S] * scale[1] + base[S:2 * S])
    cl = (mix[:, 2 * S:] * scale[2] + base[2 * S:]).view(R, S, S)
    comb = sinkhorn(cl, iters, hc_eps)
    return pre, post, comb


def hc_pre(X, hcw, norm_w, cfg: ModelConfig):
    pre, post, comb = hc_mix(X, hcw.fn, hcw.base, hcw.scale, cfg.streams, cfg.eps, cfg.hc_eps, cfg.hc_iters)
    collapsed = rb((pre[:, :, None] * X.float()).sum(1))
    normed = rb(rmsnorm(collapsed, norm_w, cfg.eps))
    return normed, post, comb


def hc_post(X, branch, post, comb):
    """X [R, S, D]; branch [R, D] fp32; returns new X (bf16 values as fp32)."""
    b = rb(branch)
    mixed = torch.einsum("rjs,rjd->rsd", comb, X.float())
    return rb(post[:, :, None] * b[:, None, :] + mixed)


# ---------------------------------------------------------------------------------------------------------------
# state
# ---------------------------------------------------------------------------------------------------------------
@dataclass
class KDAState:
    conv: torch.Tensor          # [taps-1, C] fp32 (bf16 values): the last taps-1 conv inputs
    S: torch.Tensor             # [H, Dv, Dk] fp32


@dataclass
class MLAState:
    lat: list = field(default_factory=list)        # per token: fp8 latent (as fp32) [kv_lora]
    lat_s: list = field(default_factory=list)      # per token: scale
    kpe: list = field(default_factory=list)        # per token: rope key (bf16 values) [rope]
    ik: list = field(default_factory=list)         # per token: index key (bf16 values) [ID]
    ig: list = field(default_factory=list)         # per token: pool gate scores fp32 [ID]
    pool: list = field(default_factory=list)       # per complete pool: fp8 key (as fp32) [ID]
    pool_s: list = field(default_factory=list)     # per complete pool: pow2 scale


class RefState:
    def __init__(self, w: Weights):
        c = w.cfg
        self.pos = 0
        self.kda: dict[int, KDAState] = {}
        self.mla: dict[int, MLAState] = {}
        for lw in w.layers:
            if lw.kind == "kda":
                C = 3 * lw.kda.heads * c.lin_dim
                self.kda[lw.index] = KDAState(torch.zeros(c.conv - 1, C), torch.zeros(lw.kda.heads, c.lin_dim,
                                                                                         c.lin_dim))
            else:
                self.mla[lw.index] = MLAState()


# ---------------------------------------------------------------------------------------------------------------
# blocks (single token row x [D])
# ---------------------------------------------------------------------------------------------------------------
def kda_block(lw: LayerW, cfg: ModelConfig, st: KDAState, x: torch.Tensor) -> torch.Tensor:
    k = lw.kda
    H, Dh = k.heads, cfg.lin_dim
    p = rb(lin8(x[None], k.in_proj))[0]
    C = 3 * H * Dh
    u = p[:C]
    fa = p[C:C + Dh]
    ga = p[C + Dh:C + 2 * Dh]
    b = p[C + 2 * Dh:C + 2 * Dh + H]
    f = rb(lin8(fa[None], k.f_b))[0]
    gate = rb(lin8(ga[None], k.g_b))[0]
    hist = torch.cat([st.conv, u[None]], 0)                           # [taps, C]
    conv = rb(silu((hist.t() * k.conv).sum(-1)))                      # [C]
    st.conv = hist[1:].clone()
    q = conv[:H * Dh].view(H, Dh)
    kk = conv[H * Dh:2 * H * Dh].view(H, Dh)
    v = conv[2 * H * Dh:].view(H, Dh)
    q = q / torch.sqrt((q * q).sum(-1, keepdim=True) + 1e-6) * (Dh ** -0.5)
    kk = kk / torch.sqrt((kk * kk).sum(-1, keepdim=True) + 1e-6)
    g = cfg.lower * torch.sigmoid(torch.exp(k.a_log)[:, None] * (f.view(H, Dh) + k.dt_bias.view(H, Dh)))
    S = st.S * torch.exp(g)[:, None, :]
    beta = torch.sigmoid(b)
    vnew = beta[:, None] * (v - torch.einsum("hvk,hk->hv", S, kk))
    S = S + vnew[:, :, None] * kk[:, None, :]
    st.S = S
    o = torch.einsum("hvk,hk->hv", S, q)
    o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + cfg.eps) * k.o_norm.float() * torch.sigmoid(gate.view(H, Dh))
    o = rb(o).reshape(-1)
    return lin8(o[None], k.o_proj)[0]


def index_select(cfg: ModelConfig, st: MLAState, qi: torch.Tensor, hw: torch.Tensor, t: int) -> list[int]:
    """Token indices (ascending) the query at position t attends to."""
    kp = cfg.kpool
    cur = t // kp
    P = cfg.pools_selected
    if cur <= P - 1:
        return list(range(t + 1))
    pools = torch.stack(st.pool[:cur])                                # [cur, ID] fp8 values
    ps = torch.stack(st.pool_s[:cur])
    dots = torch.einsum("hd,pd->hp", qi, pools) * ps[None, :]
    logit = (torch.relu(dots) * hw[:, None]).sum(0) / math.sqrt(cfg.index_heads * cfg.index_dim)
    # top (P-1) by logit, ties -> lower pool id (stable sort on -logit)
    order = torch.sort(-logit, stable=True).indices[:P - 1]
    chosen = sorted(order.tolist())
    toks = [j * kp + i for j in chosen for i in range(kp)]
    toks += list(range(cur * kp, t + 1))
    return toks


def mla_block(lw: LayerW, cfg: ModelConfig, st: MLAState, x: torch.Tensor, t: int) -> torch.Tensor:
    a = lw.mla
    H = a.heads
    nope, rdim, vd, L = cfg.qk_nope, cfg.qk_rope, cfg.v_dim, cfg.kv_lora
    qkv = rb(lin8(x[None], a.qkv_a))[0]
    qa, kva = qkv[:cfg.q_lora], qkv[cfg.q_lora:]
    qr = rb(rmsnorm(qa, a.q_norm, cfg.eps))
    c = rb(rmsnorm(kva[:L], a.kv_norm, cfg.eps))
    kpe = rb(rope(kva[L:], t, cfg.rope_theta))
    q = rb(lin8(qr[None], a.q_b))[0].view(H, cfg.qk_dim)
    q_nope = q[:, :nope]
    q_pe = rb(rope(q[:, nope:], t, cfg.rope_theta))
    # absorbed query: [H, L]
    q_lat = rb(torch.einsum("hn,hln->hl", q_nope, a.w_uk_t.w.view(torch.float8_e4m3fn).float()
                            * a.w_uk_t.s[:, :, None]))
    c8, cs = fp8_quant_token(c)
    st.lat.append(c8)
    st.lat_s.append(cs)
    st.kpe.append(kpe)
    # indexer
    ix = a.index
    ip = x[None].float() @ ix.proj.float().t()
    ip = ip[0]
    ID, IH = cfg.index_dim, cfg.index_heads
    ik = ip[:ID]
    ik = (ik - ik.mean()) * torch.rsqrt(ik.var(unbiased=False) + cfg.eps) * ix.ln_w + ix.ln_b
    ik = rb(ik)
    hw = ip[ID:ID + IH]
    ig = ip[ID + IH:]
    st.ik.append(ik)
    st.ig.append(ig)
    kp = cfg.kpool
    if (t + 1) % kp == 0:
        j0 = t + 1 - kp
        sc = torch.stack(st.ig[j0:t + 1]) + ix.ape                     # [kp, ID]
        wts = torch.softmax(sc, 0)
        pooled = rb((wts * torch.stack(st.ik[j0:t + 1])).sum(0))
        rot = rb(hadamard128(pooled))
        q8, s8 = fp8_quant_pow2(rot)
        st.pool.append(q8)
        st.pool_s.append(s8)
    qi = rb(lin8(qr[None], ix.wq_b))[0].view(IH, ID)
    qi = rb(hadamard128(qi))
    sel = index_select(cfg, st, qi, hw, t)
    lat = torch.stack([st.lat[j] * st.lat_s[j] for j in sel])          # [n, L]
    scale = cfg.qk_dim ** -0.5
    s = q_lat @ lat.t()
    if rdim:
        kpes = torch.stack([st.kpe[j] for j in sel])
        s = s + q_pe @ kpes.t()
    p = torch.softmax(s * scale, -1)
    o_lat = p @ lat                                                  # [H, L]
    o = torch.einsum("hl,hvl->hv", rb(o_lat), a.w_uv.w.view(torch.float8_e4m3fn).float() * a.w_uv.s[:, :, None])
    o = rb(o).reshape(-1)
    return lin8(o[None], a.o_proj)[0]


def mlp_block(m, cfg: ModelConfig, x: torch.Tensor) -> torch.Tensor:
    gu = rb(lin8(x[None], m.gu))[0]
    W = m.width
    act = rb(swiglu(gu[:W], gu[W:], cfg.limit))
    return lin8(act[None], m.down)[0]


_WQ_CACHE: dict = {}


def _wq(stack, e: int, bits: int) -> torch.Tensor:
    """Decoded rotated-domain weight of expert e (cached: decoding is the oracle's slow part)."""
    key = (stack.trellis.data_ptr(), e)
    w = _WQ_CACHE.get(key)
    if w is None:
        w = exl3_ops.unpack(stack.trellis[e], bits).float()
        _WQ_CACHE[key] = w
    return w


def _exl3_linear(x, stack, e, bits):
    xh = exl3_ops.rotate(x.float() * stack.suh[e].float(), -1).half().float()
    return exl3_ops.rotate(xh @ _wq(stack, e, bits), -1) * stack.svh[e].float()


def expert_forward(moe, e: int, x: torch.Tensor, cfg: ModelConfig) -> torch.Tensor:
    """One EXL3 expert on rows x [R, D] -> [R, D] fp32 (rotated inputs rounded to fp16 as the kernels do;
    same arithmetic as ``ops.exl3.linear``)."""
    g = _exl3_linear(x, moe.gate, e, cfg.bits)
    u = _exl3_linear(x, moe.up, e, cfg.bits)
    act = swiglu(g, u, cfg.limit)
    return _exl3_linear(act, moe.down, e, cfg.bits)


def route(x: torch.Tensor, moe, cfg: ModelConfig) -> tuple[torch.Tensor, torch.Tensor]:
    """x [R, D] -> (ids [R, top_k] int64, weights [R, top_k] fp32)."""
    logits = x.float() @ moe.router.float().t()
    score = torch.sigmoid(logits)
    choice = score + moe.bias
    # ties -> lower id: stable sort on -choice
    ids = torch.sort(-choice, dim=-1, stable=True).indices[:, :cfg.top_k]
    w = torch.gather(score, 1, ids)
    if cfg.norm_topk:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return ids, w * cfg.routed_scale


def moe_block(lw: LayerW, cfg: ModelConfig, x: torch.Tensor) -> torch.Tensor:
    m = lw.moe
    xr = x[None]
    ids, w = route(xr, m, cfg)
    y = torch.zeros(cfg.hidden)
    for k in range(cfg.top_k):
        e = int(ids[0, k])
        y = y + w[0, k] * expert_forward(m, e, xr, cfg)[0]
    return y + mlp_block(m.shared, cfg, x)


# ---------------------------------------------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------------------------------------------
class ReferenceModel:
    """Single-sequence fp32 oracle (TP=1 weights)."""

    def __init__(self, w: Weights):
        if w.world != 1:
            raise ValueError("the reference model takes unsharded (world=1) weights")
        self.w = w
        self.cfg = w.cfg
        self.state = RefState(w)

    def reset(self):
        self.state = RefState(self.w)

    @torch.no_grad()
    def step(self, token: int, return_hidden: bool = False):
        c, w = self.cfg, self.w
        t = self.state.pos
        S = c.streams
        X = w.embed[token].float()[None, None, :].expand(1, S, c.hidden).clone()
        for lw in w.layers:
            normed, post, comb = hc_pre(X, lw.attn_hc, lw.in_norm, c)
            if lw.kind == "kda":
                br = kda_block(lw, c, self.state.kda[lw.index], normed[0])
            else:
                br = mla_block(lw, c, self.state.mla[lw.index], normed[0], t)
            X = hc_post(X, br[None], post, comb)
            normed, post, comb = hc_pre(X, lw.ffn_hc, lw.post_norm, c)
            br = mlp_block(lw.mlp, c, normed[0]) if lw.mlp is not None else moe_block(lw, c, normed[0])
            X = hc_post(X, br[None], post, comb)
        h = rb(X.float().mean(1))
        hn = rb(rmsnorm(h, w.norm, c.eps))
        logits = lin8(hn, w.head)[0]
        self.state.pos += 1
        if return_hidden:
            return logits, h[0]
        return logits

    @torch.no_grad()
    def prefill(self, tokens: list[int]) -> torch.Tensor:
        out = None
        for tok in tokens:
            out = self.step(int(tok))
        return out

    @torch.no_grad()
    def generate_greedy(self, prompt: list[int], n: int) -> tuple[list[int], list[torch.Tensor]]:
        logits = self.prefill(prompt)
        toks, all_logits = [], []
        for _ in range(n):
            nxt = int(torch.argmax(logits))
            toks.append(nxt)
            all_logits.append(logits)
            logits = self.step(nxt)
        return toks, all_logits
