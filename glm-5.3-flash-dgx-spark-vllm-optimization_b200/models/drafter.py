"""Block drafter for speculative decoding: one transformer layer that proposes K tokens in a single forward.

Role of the reference's DFlash2 drafter (code/fork/docs/DRAFTER_IMPL.md:46-52; README.md:40): it reads the
target's hidden state and drafts a block (block size 8, so K <= 7) that the target verifies in one window.  This
drafter is a 1-layer block model ("a random-init 1-layer block drafter with block size 8"):

  x_i   = fc([h ; emb(t_i)]) + slot_i          i = 0..K-1,  t_0 = last committed token, t_i = MASK (i > 0),
                                               h = the target's final hidden state (stream mean) of that token
  x    += o_proj(block_causal_attn(qkv(dconv_a(rmsnorm(x)))))
  x    += down(SwiGLU(gate_up(dconv_m(rmsnorm(x)))))
  logits_i = lm_head(rmsnorm(x_i))             the target's fp8 vocabulary-parallel head, shared
  draft_i  = argmax logits_i                   (row i proposes the token at position p + 1 + i)

  dconv(y)_i = sum_k (base_k + delta_k(y_i)) * y_{i-k}   grouped dynamic causal conv inside the draft block
                                               (taps 3, one kernel delta per group of 64 channels and row,
                                               delta = a small fp8 projection of y; csrc/dconv.cu), the role of the
                                               DFlash2 drafter's grouped conv around its attention and MLP
                                               (code/fork/docs/DEC_SMALLOPS.md:12)

Weights are fp8 e4m3 with per-row scales like the target's dense projections, random-initialised (seed-keyed), and
replicated on every tensor-parallel rank; only the shared head is vocabulary-sharded.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..config import ModelConfig
from ..ops import kernels as K
from .runtime import interleave_gate_up
from .weights import quantize_fp8_rows, _seed_of

MASK_TOKEN = 0


@dataclass
class DrafterConfig:
    block: int = 8              # K <= block - 1 drafts, plus the anchor row
    heads: int = 32
    head_dim: int = 128
    mlp_width: int = 8192
    conv_taps: int = 3          # grouped dynamic conv on the attention and MLP inputs
    conv_group: int = 64        # channels sharing one per-row kernel delta


class BlockDrafter:
    def __init__(self, cfg: ModelConfig, target_w, dc: DrafterConfig | None = None, seed: int = 1,
                 device="cuda", max_batch: int = 1):
        self.cfg, self.tw = cfg, target_w
        dc = dc or DrafterConfig(heads=max(1, cfg.hidden // 128), head_dim=min(128, cfg.hidden),
                                 mlp_width=2 * cfg.hidden)
        self.dc = dc
        D = cfg.hidden
        H, Dh = dc.heads, dc.head_dim
        dev = torch.device(device)

        def lin(name, n, k):
            g = torch.Generator(device=dev)
            g.manual_seed(_seed_of(seed, name))
            return quantize_fp8_rows(torch.randn(n, k, generator=g, device=dev) / math.sqrt(k))

        def norm(name, n):
            g = torch.Generator(device=dev)
            g.manual_seed(_seed_of(seed, name))
            return (1 + 0.05 * torch.randn(n, generator=g, device=dev)).to(torch.bfloat16)

        self.fc = lin("drafter.fc", D, 2 * D)
        self.qkv = lin("drafter.qkv", 3 * H * Dh, D)
        self.o = lin("drafter.o", D, H * Dh)
        self.gu = interleave_gate_up(lin("drafter.gate_up", 2 * dc.mlp_width, D))
        self.down = lin("drafter.down", D, dc.mlp_width)
        self.n1, self.n2, self.nf = norm("drafter.n1", D), norm("drafter.n2", D), norm("drafter.nf", D)
        taps, G = dc.conv_taps, D // dc.conv_group

        def conv_base(name):
            g = torch.Generator(device=dev)
            g.manual_seed(_seed_of(seed, name))
            b = 0.1 * torch.randn(taps, D, generator=g, device=dev)
            b[0] += 1.0                                   # near the identity: the current row dominates
            return b.to(torch.bfloat16)
        self.conv_a = (lin("drafter.conv_attn.delta", taps * G, D), conv_base("drafter.conv_attn.base"))
        self.conv_m = (lin("drafter.conv_mlp.delta", taps * G, D), conv_base("drafter.conv_mlp.base"))
        # several requests draft in one pass (max_batch blocks of rows, request b's rows at [b k, (b+1) k))
        self.max_batch = max(1, max_batch)
        R = dc.block * self.max_batch
        self.delta = torch.zeros(R, taps * G, dtype=torch.bfloat16, device=dev)
        self.xc = torch.zeros(R, D, dtype=torch.bfloat16, device=dev)
        g = torch.Generator(device=dev)
        g.manual_seed(_seed_of(seed, "drafter.slot"))
        self.slot_emb = (torch.randn(dc.block, D, generator=g, device=dev) * 0.1).float()
        bf = torch.bfloat16
        self.inp = torch.zeros(R, 2 * D, dtype=bf, device=dev)
        self.emb = torch.zeros(R, 1, D, dtype=bf, device=dev)
        self.x = torch.zeros(R, D, dtype=torch.float32, device=dev)
        self.xn = torch.zeros(R, D, dtype=bf, device=dev)
        self.qkv_buf = torch.zeros(R, 3 * H * Dh, dtype=bf, device=dev)
        self.att = torch.zeros(R, H * Dh, dtype=bf, device=dev)
        self.act = torch.zeros(R, dc.mlp_width, dtype=bf, device=dev)
        self.logits = torch.zeros(R, target_w.head.n, dtype=torch.float32, device=dev)
        self.ids = torch.full((R,), MASK_TOKEN, dtype=torch.int32, device=dev)
        self.hid = torch.zeros(self.max_batch, D, dtype=bf, device=dev)
        self._k = 1

    def _dconv(self, conv, R: int, k: int) -> None:
        """xc[:R] = grouped dynamic conv of xn[:R] within each request's block of k rows (the kernel deltas projected
        from xn itself)."""
        proj, base = conv
        K.linear8(self.xn[:R], proj.w, proj.s, self.delta[:R])
        K.C().dconv(self.xn[:R], self.delta[:R], base, self.xc[:R], self.dc.conv_group, k)

    @torch.no_grad()
    def forward(self, last_token: torch.Tensor, hidden: torch.Tensor, k: int) -> torch.Tensor:
        """last_token: int32 [1] (device); hidden: bf16 [D] target hidden of that token. Returns logits [k, V_local]
        (the caller samples / argmaxes them through the tensor-parallel sampler)."""
        self.stage(last_token, hidden)
        return self.run(k)

    def stage(self, last_token, hidden: torch.Tensor) -> None:
        """Inputs of the next draft into the drafter's static buffers (outside any CUDA graph): the last token (a
        device int32 [1] tensor or a Python int) and the target hidden state of that token."""
        if isinstance(last_token, int):
            self.ids[:1].fill_(last_token)
        else:
            self.ids[:1].copy_(last_token)
        self.hid[0].copy_(hidden.view(-1))

    def stage_batch(self, last_tokens: list[int], hiddens: list[torch.Tensor], k: int) -> None:
        """Inputs of one draft pass for several requests (outside any CUDA graph): request b's last token goes to
        row b k of its block (the other rows of the block are MASK) and its target hidden state to hid[b]."""
        B = len(last_tokens)
        if B > self.max_batch or k > self.dc.block:
            raise ValueError("draft batch exceeds the drafter's buffers")
        ids = torch.full((B, k), MASK_TOKEN, dtype=torch.int32)
        ids[:, 0] = torch.tensor(last_tokens, dtype=torch.int32)
        self.ids[:B * k].copy_(ids.view(-1), non_blocking=True)
        for b, h in enumerate(hiddens):
            self.hid[b].copy_(h.view(-1))

    @torch.no_grad()
    def run(self, k: int) -> torch.Tensor:
        """The draft block of one request from the staged inputs (static buffers only: capturable as a CUDA graph
        per k)."""
        return self.run_batch(1, k)

    @torch.no_grad()
    def run_batch(self, B: int, k: int) -> torch.Tensor:
        """Draft blocks of B requests in one pass (rows [b k, (b+1) k) of request b; the block attention and the
        dynamic convolutions stay inside each request's block, the projections read their weights once for all
        rows).  Returns logits [B k, V_local]; capturable as a CUDA graph per (B, k).  With B = 1 this is the
        single-request draft, bit for bit."""
        Kc = K.C()
        D = self.cfg.hidden
        k = max(k, 1)
        R = B * k
        # [h ; emb(t_i)]
        Kc.embed(self.ids[:R], self.tw.embed, self.emb[:R])
        self.inp[:R, D:].copy_(self.emb[:R, 0])
        self.inp[:R, :D].view(B, k, D).copy_(self.hid[:B].view(B, 1, D).expand(B, k, D))
        self.x[:R].view(B, k, D).copy_(self.slot_emb[:k].view(1, k, D).expand(B, k, D))
        K.linear8(self.inp[:R], self.fc.w, self.fc.s, self.x[:R], K.GEMV_F32_ACC)
        Kc.rmsnorm_f32(self.x[:R], self.n1, self.cfg.eps, self.xn[:R])
        self._dconv(self.conv_a, R, k)
        K.linear8(self.xc[:R], self.qkv.w, self.qkv.s, self.qkv_buf[:R])
        Kc.block_attn(self.qkv_buf[:R], self.dc.heads, self.dc.head_dim, k, self.dc.head_dim ** -0.5, self.att[:R])
        K.linear8(self.att[:R], self.o.w, self.o.s, self.x[:R], K.GEMV_F32_ACC)
        Kc.rmsnorm_f32(self.x[:R], self.n2, self.cfg.eps, self.xn[:R])
        self._dconv(self.conv_m, R, k)
        K.linear8(self.xc[:R], self.gu.w, self.gu.s, self.act[:R], K.GEMV_SWIGLU, self.cfg.limit)
        K.linear8(self.act[:R], self.down.w, self.down.s, self.x[:R], K.GEMV_F32_ACC)
        Kc.rmsnorm_f32(self.x[:R], self.nf, self.cfg.eps, self.xn[:R])
        K.linear8(self.xn[:R], self.tw.head.w, self.tw.head.s, self.logits[:R], K.GEMV_F32)
        return self.logits[:R]
