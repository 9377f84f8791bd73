"""GPU model runtime: the GLM-5.3-Flash forward pass on this engine's sm_100a kernels.

One ``Runtime`` per rank.  Every forward reads its inputs from static device buffers (``Batch``) and writes into
preallocated scratch, so a decode step can be captured once in a CUDA graph and replayed.  A forward covers R rows
that belong to B sequences (a decode window of K+1 rows per request, or one prefill chunk); per row it needs the
token id, position, KV token slot and sequence index, per sequence the page table, the KDA state-pool indices (read
/ write) and the conv-window slot.

Layer structure (code/fork/docs/ref/tf_forward.py:278-301): mHC pre -> KDA or MLA/DSA -> [all-reduce] -> mHC post
fused with the next mHC pre -> dense MLP or MoE -> [all-reduce] -> ...; the final mHC post is followed by the
stream mean, the final RMSNorm and the vocabulary-parallel lm_head.

KDA verify windows: the recurrent kernel reads state ``s_in`` and writes the state after the window's last row to
``s_out``; ``commit`` keeps the first ``keep`` rows of each sequence (re-running the recurrence over them when
keep < rows, from the layer's saved window inputs) and shifts the conv windows.
"""

from __future__ import annotations

import os
from array import array
from dataclasses import dataclass

import numpy as np
import torch

from ..ops import kernels as K
from ..utils.canary import Scratch
from .weights import Linear8, Weights

bf16, f32, i32 = torch.bfloat16, torch.float32, torch.int32
KDA_CHUNK_MIN_ROWS = 32     # prefill windows longer than this use the chunked KDA kernel
MOE_PREFILL_MIN_ROWS = 64   # forwards with more rows route the experts through the tcgen05 prefill kernels


@dataclass
class RuntimeConfig:
    max_rows: int = 16            # rows of one forward
    max_seqs: int = 1             # sequences with KDA state / conv windows
    kv_slots: int = 8192          # token slots of the paged caches (a multiple of block_size)
    block_size: int = 64
    max_blocks: int = 128         # page-table width per sequence
    decode_rows: int = 16         # forwards of at most this many rows keep per-layer KDA window inputs (replay)
    mla_splits: int = 16          # most key splits of the decode attention (rows x splits fill the SMs)
    moe_chunk: int = 256          # rows per routed-MoE launch group of the decode path (routing kernel capacity)
    moe_prefill_rows: int = 8192  # rows per routed-MoE launch group of the prefill (tcgen05) path
    attn_chunk: int = 1024        # rows per attention launch group (scratch bound)
    logit_rows: int = 16


def interleave_gate_up(gu: Linear8) -> Linear8:
    """[gate; up] rows -> 16-row tiles of (8 gate rows, the matching 8 up rows): the layout the GEMV SwiGLU
    epilogue expects."""
    n = gu.w.shape[0] // 2
    assert n % 8 == 0
    g, u = gu.w[:n].view(n // 8, 8, -1), gu.w[n:].view(n // 8, 8, -1)
    gs, us = gu.s[:n].view(n // 8, 8), gu.s[n:].view(n // 8, 8)
    w = torch.stack([g, u], 1).reshape(2 * n, -1).contiguous()
    s = torch.stack([gs, us], 1).reshape(2 * n).contiguous()
    return Linear8(w, s)


class Batch:
    """Static device buffers describing the rows and sequences of a forward."""

    def __init__(self, rc: RuntimeConfig, device):
        R, B = rc.max_rows, rc.max_seqs
        self.ids = torch.zeros(R, dtype=i32, device=device)
        self.positions = torch.zeros(R, dtype=i32, device=device)
        self.slots = torch.zeros(R, dtype=i32, device=device)
        self.row_seq = torch.zeros(R, dtype=i32, device=device)
        self.kda_seq = torch.zeros(5, B, dtype=i32, device=device)        # row0, nrows, s_in, s_out, conv_slot
        self.commit_seq = torch.zeros(5, B, dtype=i32, device=device)     # same with nrows = kept rows
        self.block_table = torch.zeros(B, rc.max_blocks, dtype=i32, device=device)
        self.logit_rows = torch.zeros(rc.logit_rows, dtype=torch.int64, device=device)
        self.host = torch.zeros(4 * R + 10 * B + rc.logit_rows, dtype=i32, pin_memory=torch.cuda.is_available())
        self.R = 0
        self.B = 0
        self.commit_B = 0
        self.max_rows_per_seq = 0
        self.n_logits = 0


class Runtime:
    def __init__(self, w: Weights, rc: RuntimeConfig, comm=None):
        self.w, self.rc, self.comm = w, rc, comm
        c = self.cfg = w.cfg
        dev = self.device = w.device
        self.tp = w.world
        R = rc.max_rows
        D, S = c.hidden, c.streams
        self.batch = Batch(rc, dev)
        self.px = None
        self._fused = False
        # side stream for work that does not feed the next kernel (decode windows): the shared expert runs beside the
        # routed experts (ALU-bound trellis decode vs a bandwidth-bound GEMV), the KDA output-gate projection beside
        # the convolution and recurrence; forked and joined with events, so CUDA-graph capture records both branches
        self.overlap = dev.type == "cuda" and os.environ.get("GLM53_OVERLAP", "1") == "1"
        # decode windows run the KDA block tail (f_b, g_b, conv, recurrence, gated norm) as one kernel
        # (GLM53_KDA_FUSED=0: the five-kernel path)
        self.kda_fused = os.environ.get("GLM53_KDA_FUSED", "1") == "1"
        if self.overlap:
            self.side = torch.cuda.Stream(device=dev)
            self.ev_fork, self.ev_join = torch.cuda.Event(), torch.cuda.Event()
        # L2 prefetch (decode windows, GLM53_L2_PREFETCH=1): the routed experts' gate/up CTAs prefetch the next
        # layer's first projections into L2 while their ALU-bound trellis decode leaves HBM idle (the trellis loads
        # are marked evict-first); GLM53_L2_PREFETCH_MB caps the bytes.  Off by default: measured on the TP1 decode
        # step it is neutral (+0.5 % at 32 MiB, -0.7 % at 96 MiB), the bulk-copy GEMV already streaming near HBM rate
        self.l2pf = dev.type == "cuda" and os.environ.get("GLM53_L2_PREFETCH", "0") == "1"
        self.l2pf_bytes = int(float(os.environ.get("GLM53_L2_PREFETCH_MB", "32")) * 2 ** 20)
        # prefill chunks (rows >= GEMM_MIN_M) can push their partials from the tcgen05 GEMM epilogue as well
        # (GLM53_FUSED_TP_PREFILL=1).  Off by default: measured on 8192-row chunks it is slower than NCCL's ring
        # all-reduce (32k prefill 10.1k vs 11.3k tok/s at TP2, 10.5k vs 15.3k at TP4) -- every rank stores its whole
        # partial into every peer, (W-1) x the ring's bytes per rank, from the GEMM epilogue's 4 warps
        self._fused_prefill = os.environ.get("GLM53_FUSED_TP_PREFILL", "0") == "1"
        # sequence parallelism for prefill chunks (tensor parallel, at least GLM53_SP_MIN_ROWS rows, a multiple of the
        # world size): rank j keeps the residual streams of rows [j R/W, (j+1) R/W) and runs mHC on them only; the
        # normalised rows are all-gathered before each block and the block's fp32 partials reduce-scattered after
        # it (the all-reduce's two halves, with the mHC work divided by W between them).  Measured on an 8192-row
        # chunk at TP2: 451 ms against 475 ms with the all-reduce
        self.sp = dev.type == "cuda" and os.environ.get("GLM53_SP", "1") == "1"
        self.sp_min_rows = int(os.environ.get("GLM53_SP_MIN_ROWS", "256"))
        # with W8A8 on the KDA input projection, sequence-parallel chunks all-gather its e4m3 rows (and row scales)
        # instead of bf16 rows: half the bytes, the same codes (per-row quantisation is row-local)
        self.sp_fp8ag = os.environ.get("GLM53_SP_FP8AG", "1") == "1"
        self._qin = None
        self._sp = None
        if comm is not None and self.tp > 1 and getattr(comm, "fused", False):
            from ..parallel.fused import PeerExchange
            rows = R if (self._fused_prefill and R >= K.GEMM_MIN_M) else min(R, rc.decode_rows, K.GEMV_MAX_M)
            self.px = PeerExchange(rows, D, dev)
        # --- GPU-layout weights (SwiGLU-interleaved gate/up) ---
        self.gu_il = {}
        for lw in w.layers:
            m = lw.mlp if lw.mlp is not None else lw.moe.shared
            self.gu_il[lw.index] = interleave_gate_up(m.gu)
        # scratch: guard bands around every buffer in the bounds-checked build (utils/canary.py)
        self.scratch = Scratch(dev)
        self.scratch.attach(self)
        z = self.scratch.zeros
        # --- activations ---
        self.X = z(R, S, D, dtype=bf16, device=dev)
        self.normed = z(R, D, dtype=bf16, device=dev)
        self.post = [z(R, S, dtype=f32, device=dev) for _ in range(2)]
        self.comb = [z(R, S, S, dtype=f32, device=dev) for _ in range(2)]
        self.part = z(R, D // 64, 32, dtype=f32, device=dev)
        self.branch = z(R, D, dtype=f32, device=dev)
        self.hidden = z(R, D, dtype=bf16, device=dev)
        # reduce-scatter output of the sequence-parallel prefill (this rank's rows of the block sum)
        self.rs = z((R + self.tp - 1) // self.tp, D, dtype=f32, device=dev) if self.tp > 1 else None
        sp_q = self.tp > 1 and self.sp and self.sp_fp8ag and R >= K.GEMM_MIN_M
        self.q_rows = z(R, D, dtype=torch.uint8, device=dev) if sp_q else None
        self.q_scale = z(R, dtype=f32, device=dev) if sp_q else None
        self.fnormed = z(R, D, dtype=bf16, device=dev)
        self.lrows = z(rc.logit_rows, D, dtype=bf16, device=dev)
        self.logits = z(rc.logit_rows, w.head.n, dtype=f32, device=dev)
        # --- KDA ---
        kda = [lw for lw in w.layers if lw.kind == "kda"]
        self.kda_index = {lw.index: i for i, lw in enumerate(kda)}
        if kda:
            k0 = kda[0].kda
            H, Dh = k0.heads, c.lin_dim
            self.kH, self.kDh = H, Dh
            width = k0.in_proj.n
            self.kda_width = width
            width = (width + 63) // 64 * 64          # padded row stride: 16-byte aligned rows for vector loads
            C3 = 3 * H * Dh
            self.S_pool = [z(2 * rc.max_seqs, H, Dh, Dh, dtype=f32, device=dev) for _ in kda]
            self.conv_pool = [z(rc.max_seqs, c.conv - 1, C3, dtype=bf16, device=dev) for _ in kda]
            dr = min(rc.decode_rows, R)
            self.kproj_l = [z(dr, width, dtype=bf16, device=dev) for _ in kda]
            self.kf_l = [z(dr, H * Dh, dtype=bf16, device=dev) for _ in kda]
            self.kqkv_l = [z(dr, C3, dtype=bf16, device=dev) for _ in kda]
            self.kproj = z(R, width, dtype=bf16, device=dev)
            self.kf = z(R, H * Dh, dtype=bf16, device=dev)
            self.kqkv = z(R, C3, dtype=bf16, device=dev)
            self.kg = z(R, H * Dh, dtype=bf16, device=dev)
            # chunked prefill records per (64-row chunk slot, head): Q~, K~, K^ [64, Dh] (fp16), T, P [64, 64],
            # e^{G_C} [Dh] (slots = chunks of the longest launch + sequences + 1; layout in csrc/kda_chunk.cu)
            self.kda_scr = None
            if R > KDA_CHUNK_MIN_ROWS:
                n = K.C().kda_chunk_scratch_floats(R, rc.max_seqs, H, Dh)
                self.kda_scr = z(n, dtype=f32, device=dev)
            self.ko = z(R, H * Dh, dtype=f32, device=dev)
            self.kout = z(R, H * Dh, dtype=bf16, device=dev)
        # --- MLA / DSA ---
        mla = [lw for lw in w.layers if lw.kind == "mla"]
        self.mla_index = {lw.index: i for i, lw in enumerate(mla)}
        if mla:
            a0 = mla[0].mla
            H = self.mH = a0.heads
            L, rope = c.kv_lora, c.qk_rope
            ns = rc.kv_slots
            assert ns % rc.block_size == 0 and rc.block_size % c.kpool == 0
            self.kv = [z(ns, L, dtype=torch.uint8, device=dev) for _ in mla]
            self.kv_scale = [z(ns, dtype=f32, device=dev) for _ in mla]
            self.kpe = [z(ns, max(rope, 1), dtype=bf16, device=dev) for _ in mla]
            # raw index keys / pool gate scores live only until their pool of kpool tokens is complete: this
            # forward's rows in shared row buffers, earlier tokens of open pools in a per-sequence tail ring per layer
            # (indexed by the sequence's state slot); the paged cache holds pooled keys only
            ring = K.DSA_RING
            self.ik_rows = z(R, c.index_dim, dtype=bf16, device=dev)
            self.ig_rows = z(R, c.index_dim, dtype=f32, device=dev)
            self.ik_ring = [z(rc.max_seqs * ring, c.index_dim, dtype=bf16, device=dev) for _ in mla]
            self.ig_ring = [z(rc.max_seqs * ring, c.index_dim, dtype=f32, device=dev) for _ in mla]
            self.pool = [z(ns // c.kpool, c.index_dim, dtype=torch.uint8, device=dev) for _ in mla]
            self.pool_scale = [z(ns // c.kpool, dtype=f32, device=dev) for _ in mla]
            AR = min(R, rc.attn_chunk)
            self.qkv_a = z(R, a0.qkv_a.n, dtype=bf16, device=dev)
            self.qr = z(R, c.q_lora, dtype=bf16, device=dev)
            self.q = z(R, H, c.qk_dim, dtype=bf16, device=dev)
            self.q_lat = z(R, H, L, dtype=bf16, device=dev)
            self.o_lat = z(R, H, L, dtype=bf16, device=dev)
            self.obuf = z(R, H * c.v_dim, dtype=bf16, device=dev)
            self.iproj = z(R, 2 * c.index_dim + c.index_heads, dtype=f32, device=dev)
            self.qi = z(R, c.index_heads * c.index_dim, dtype=bf16, device=dev)
            self.max_pools = rc.max_blocks * rc.block_size // c.kpool
            self.dsa_logits = z(AR, self.max_pools, dtype=f32, device=dev)
            self.max_sel = max(c.index_topk, 1)
            self.sel = z(AR, max(self.max_sel, c.index_topk), dtype=i32, device=dev)
            self.sel_count = z(AR, dtype=i32, device=dev)
            self.splits = rc.mla_splits
            self.sms = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 148
            # partials: decode-sized forwards split the keys; the CUDA-core kernel also stages unsplit rows here
            PR = max(min(AR, rc.decode_rows) * rc.mla_splits, AR)
            self.part_o = z(PR * H * L, dtype=f32, device=dev)
            self.part_ml = z(PR * H * 2, dtype=f32, device=dev)
        # --- MLP / MoE ---
        MR = min(R, rc.moe_chunk)
        tk = c.top_k
        P = MR * tk
        widths = [self.gu_il[i].w.shape[0] // 2 for i in self.gu_il]
        self.act = z(R, max(widths), dtype=bf16, device=dev)
        self.rlogits = z(MR, c.experts, dtype=f32, device=dev)
        self.topk_ids = z(MR, tk, dtype=i32, device=dev)
        self.topk_w = z(MR, tk, dtype=f32, device=dev)
        self.max_groups = min(P, c.experts)
        self.group_count = z(1, dtype=i32, device=dev)
        self.group_expert = z(self.max_groups, dtype=i32, device=dev)
        self.group_offset = z(self.max_groups + 1, dtype=i32, device=dev)
        self.pair_token = z(P, dtype=i32, device=dev)
        self.pair_expert = z(P, dtype=i32, device=dev)
        self.pair_w = z(P, dtype=f32, device=dev)
        self.pair_of = z(P, dtype=i32, device=dev)
        moe0 = next((lw.moe for lw in w.layers if lw.moe is not None), None)
        self.prefill_moe = R > MOE_PREFILL_MIN_ROWS and moe0 is not None
        if self.prefill_moe:
            # prefill path: one routing group of up to moe_prefill_rows rows
            PR = min(R, rc.moe_prefill_rows)
            self.p_rows = PR
            PP = PR * tk
            self.p_logits = z(PR, c.experts, dtype=f32, device=dev)
            self.p_topk_ids = z(PR, tk, dtype=i32, device=dev)
            self.p_topk_w = z(PR, tk, dtype=f32, device=dev)
            self.p_groups = c.experts
            self.p_group_expert = z(c.experts, dtype=i32, device=dev)
            self.p_group_offset = z(c.experts + 1, dtype=i32, device=dev)
            self.p_pair_token = z(PP, dtype=i32, device=dev)
            self.p_pair_expert = z(PP, dtype=i32, device=dev)
            self.p_pair_w = z(PP, dtype=f32, device=dev)
            self.p_pair_of = z(PP, dtype=i32, device=dev)
            self.p_counts = z(c.experts, dtype=i32, device=dev)
            self.p_fill = z(c.experts, dtype=i32, device=dev)
            P = max(P, PP)
        # expert parallelism (weights prepared with ep=True): each rank routes its own share of the rows, dispatches
        # them to the ranks owning their experts and receives their outputs (parallel/ep.py, one exchange and one
        # scratch for all MoE layers); the shared expert and everything else stay tensor-parallel
        self.ep = None
        if moe0 is not None and w.meta.get("ep") and self.tp > 1 and comm is not None:
            from ..parallel.ep import EPBuffers, EPMoE
            self.ep_bufs = EPBuffers(c, moe0.gate.n, (R + self.tp - 1) // self.tp, w.rank, w.world, device=dev)
            self.ep = {lw.index: EPMoE(c, lw.moe.router, lw.moe.bias, lw.moe.gate, lw.moe.up, lw.moe.down, 0,
                                       w.rank, w.world, bufs=self.ep_bufs)
                       for lw in w.layers if lw.moe is not None}
            self.prefill_moe = False
        if moe0 is not None and self.ep is None:
            # the decode path stores its rotated inputs as duplicated f16 pairs (2 halves per element)
            PX = max(P, 2 * MR * tk)
            self.xh_g = z(PX, D, dtype=torch.float16, device=dev)
            self.xh_u = z(PX, D, dtype=torch.float16, device=dev)
            self.xd = z(PX, moe0.gate.n, dtype=torch.float16, device=dev)
            self.yd = z(P, D, dtype=f32, device=dev)

    # ------------------------------------------------------------------------------------------------------------
    # host-side batch staging (pinned buffer -> one H2D copy per array)
    # ------------------------------------------------------------------------------------------------------------
    def stage(self, ids, positions, slots, row_seq, seqs, block_tables, logit_rows) -> int:
        """ids/positions/slots/row_seq: per-row ints; seqs: per sequence (row0, nrows, s_in, s_out, conv_slot);
        block_tables: per sequence list of page ids; logit_rows: rows whose logits are computed.  Everything is
        packed into one pinned host buffer and copied to the static device buffers asynchronously."""
        b = self.batch
        R, B = len(ids), len(seqs)
        if R > self.rc.max_rows or B > self.rc.max_seqs or len(logit_rows) > self.rc.logit_rows:
            raise ValueError("batch exceeds the runtime's static buffers")
        nbt = max((len(t) for t in block_tables), default=0)
        if nbt > self.rc.max_blocks:
            raise ValueError("page table wider than max_blocks")
        n_needed = 4 * R + 5 * B + B * nbt + 2 * len(logit_rows) + 1
        if b.host.numel() < n_needed:
            b.host = torch.zeros(2 * n_needed, dtype=i32, pin_memory=torch.cuda.is_available())
        # the previous staging copies must have left the pinned buffer before it is rewritten
        if getattr(b, "staged", None) is not None:
            b.staged.synchronize()
        h = b.host.numpy()
        o = 0
        segs = []
        for arr in (ids, positions, slots, row_seq):
            h[o:o + R] = arr
            segs.append((o, R))
            o += R
        sq = [list(col) for col in zip(*seqs)]          # 5 rows of B
        for row in sq:
            h[o:o + B] = row
            o += B
        sq_off = o - 5 * B
        bt_off = o
        for t in block_tables:
            # int32 arrays (the engine's page tables) copy as one buffer; lists convert element by element
            h[o:o + len(t)] = np.frombuffer(t, dtype=np.int32) if isinstance(t, array) and t.itemsize == 4 else t
            o += nbt
        o += o & 1                                        # 8-byte alignment of the int64 logit-row indices
        lr = h[o:o + 2 * len(logit_rows)].view("int64")
        lr[:] = logit_rows
        lr_off = o
        hb = b.host
        for dst, (off, n) in zip((b.ids, b.positions, b.slots, b.row_seq), segs):
            dst[:n].copy_(hb[off:off + n], non_blocking=True)
        b.kda_seq[:, :B].copy_(hb[sq_off:sq_off + 5 * B].view(5, B), non_blocking=True)
        if nbt:
            b.block_table[:B, :nbt].copy_(hb[bt_off:bt_off + B * nbt].view(B, nbt), non_blocking=True)
        if logit_rows:
            b.logit_rows[:len(logit_rows)].copy_(hb[lr_off:lr_off + 2 * len(logit_rows)].view(torch.int64),
                                                 non_blocking=True)
        if torch.cuda.is_available():
            b.staged = torch.cuda.Event()
            b.staged.record()
        b.R, b.B = R, B
        b.max_rows_per_seq = max(s[1] for s in seqs)
        b.n_logits = len(logit_rows)
        b.h2d_bytes = 4 * n_needed
        return R

    # ------------------------------------------------------------------------------------------------------------
    # forward
    # ------------------------------------------------------------------------------------------------------------
    def allreduce(self, t: torch.Tensor):
        if self.comm is not None and self.tp > 1:
            self.comm.all_reduce(t)

    def forward(self, R: int | None = None, keep_window: bool | None = None, logits: bool = True):
        b = self.batch
        R = b.R if R is None else R
        c = self.cfg
        if keep_window is None:
            keep_window = R <= self.rc.decode_rows
        self._keep_window = keep_window
        Kc = K.C()
        X = self.X[:R]
        # sequence-parallel prefill: this rank's rows [r0, r1) of the residual streams (see __init__)
        self._sp = None
        if (getattr(self, "sp", False) and self.tp > 1 and self.comm is not None and not keep_window
                and R >= self.sp_min_rows and R % self.tp == 0):
            Rl = R // self.tp
            self._sp = (self.w.rank * Rl, (self.w.rank + 1) * Rl)
        rows = slice(*self._sp) if self._sp else slice(0, R)
        Kc.embed(b.ids[rows], self.w.embed, X[rows])
        cur = 0
        first = True
        # tensor parallelism: block partials are pushed to the peers by the block's last projection (GEMV epilogue
        # for decode windows, tcgen05 GEMM epilogue for prefill chunks) and reduced inside the next mHC kernel
        # (parallel/fused.py); rows between the two kernels' ranges, or with the switch off, all-reduce by NCCL
        self._fused = self._sp is None and self.px is not None and R <= self.px.rows and (
            R <= K.GEMV_MAX_M or (self._fused_prefill and R >= K.GEMM_MIN_M and K.GEMM_ENABLED))
        self._point = 0
        for lw in self.w.layers:
            # post of the previous FFN (none before layer 0) fused with this layer's attention pre
            nxt = 1 - cur
            if first:
                Kc.hc_post_pre(X[rows], None, None, None, lw.attn_hc.fn, lw.attn_hc.base, lw.attn_hc.scale,
                               lw.in_norm, self.normed[rows], self.post[nxt][rows], self.comb[nxt][rows],
                               self.part[:rows.stop - rows.start], c.eps, c.hc_eps, c.hc_iters)
            else:
                self._post_pre(X, R, cur, nxt, lw.attn_hc, lw.in_norm)
            if lw.kind == "kda" and self._sp_fp8(R):
                self._sp_gather_q(R)
            else:
                self._sp_gather(self.normed, R)
            cur = nxt
            first = False
            if lw.kind == "kda":
                self._kda(lw, R)
            else:
                self._mla(lw, R)
            nxt = 1 - cur
            self._post_pre(X, R, cur, nxt, lw.ffn_hc, lw.post_norm)
            self._sp_gather(self.normed, R)
            cur = nxt
            if lw.mlp is not None:
                self._mlp(lw, R)
            else:
                self._moe(lw, R)
        self._post_pre(X, R, cur, None, None, None)
        Kc.stream_mean_norm(X[rows], self.w.norm, c.eps, self.hidden[rows], self.fnormed[rows])
        self._sp_gather(self.hidden, R)
        self._sp_gather(self.fnormed, R)
        if not logits:
            return None
        n = b.n_logits
        torch.index_select(self.fnormed[:R], 0, b.logit_rows[:n], out=self.lrows[:n])
        K.linear8(self.lrows[:n], self.w.head.w, self.w.head.s, self.logits[:n], K.GEMV_F32)
        return self.logits[:n]

    def _sp_fp8(self, R) -> bool:
        """Whether this sequence-parallel chunk all-gathers the KDA input rows in e4m3 (see __init__)."""
        return (self._sp is not None and self.q_rows is not None and R <= self.q_rows.shape[0]
                and R >= K.GEMM_MIN_M and K.w8a8_large_m("kda_in_proj"))

    def _sp_gather_q(self, R):
        """This rank's normalised rows quantised to the W8A8 row format, then every rank's codes and scales to every
        rank; the KDA input projection consumes them (self._qin) instead of bf16 rows."""
        r0, r1 = self._sp
        K.C().quant_rows(self.normed[r0:r1], self.q_rows[r0:r1], self.q_scale[r0:r1])
        self.comm.all_gather(self.q_rows[:R].view(-1), self.q_rows[r0:r1].reshape(-1))
        self.comm.all_gather(self.q_scale[:R], self.q_scale[r0:r1])
        self._qin = (self.q_rows[:R], self.q_scale[:R])

    def _sp_gather(self, buf, R):
        """Sequence-parallel prefill: every rank's rows of ``buf`` to every rank (``buf[:R]`` in row order)."""
        if self._sp is not None:
            r0, r1 = self._sp
            self.comm.all_gather(buf[:R].view(-1), buf[r0:r1].reshape(-1))

    def _post_pre(self, X, R, cur, nxt, hc, norm_w):
        """mHC post of the block just computed (reducing the tensor-parallel partials) fused with the next pre
        (hc None: post only)."""
        c = self.cfg
        Kc = K.C()
        if self._sp is not None:
            # this rank's rows: reduce-scatter of the block's partials, then post + pre on those rows only
            r0, r1 = self._sp
            n = r1 - r0
            if getattr(self, "_branch_local", False):     # the block computed this rank's rows completely
                rs = self.branch[r0:r1]
                self._branch_local = False
            else:
                rs = self.rs[:n]
                self.comm.reduce_scatter(rs, self.branch[:R])
            pre = (hc.fn, hc.base, hc.scale, norm_w, self.normed[r0:r1], self.post[nxt][r0:r1],
                   self.comb[nxt][r0:r1]) if hc is not None else (None,) * 7
            Kc.hc_post_pre(X[r0:r1], rs, self.post[cur][r0:r1], self.comb[cur][r0:r1], *pre, self.part[:n], c.eps,
                           c.hc_eps, c.hc_iters)
            self._point += 1
            return
        pre = (hc.fn, hc.base, hc.scale, norm_w, self.normed[:R], self.post[nxt][:R], self.comb[nxt][:R]) \
            if hc is not None else (None,) * 7
        if self._fused:
            px, p = self.px, self._point % 2
            Kc.hc_post_pre_tp(X, px.gath[p], px.slot, px.world, px.flags[p], px.epoch[p:p + 1],
                              px.done_cons[p:p + 1], px.err, self.post[cur][:R], self.comb[cur][:R], *pre,
                              self.part[:R], c.eps, c.hc_eps, c.hc_iters)
        else:
            self.allreduce(self.branch[:R])
            Kc.hc_post_pre(X, self.branch[:R], self.post[cur][:R], self.comb[cur][:R], *pre, self.part[:R], c.eps,
                           c.hc_eps, c.hc_iters)
        self._point += 1

    def _final_linear(self, x, lin, R, mode=K.GEMV_F32, proj=None):
        """The row-parallel projection that ends a block: writes the block's fp32 partial into ``branch``; in the
        fused tensor-parallel mode it also pushes it into every rank's receive slot."""
        if self._fused and R <= K.GEMV_MAX_M:
            px, p = self.px, self._point % 2
            K.C().gemv_push(x, lin.w, lin.s, self.branch[:R], mode, px.push_ptrs[p], px.push_flags[p],
                            px.done_prod[p:p + 1], px.slot, px.rank, px.world, px.err)
        elif self._fused:
            px, p = self.px, self._point % 2
            K.C().gemm_w8a16_push(x, lin.w, lin.s, self.branch[:R], mode, K._w_scratch(lin.w.numel(), x.device),
                                  px.push_ptrs[p], px.push_flags[p], px.done_prod[p:p + 1], px.slot, px.rank,
                                  px.world)
        else:
            K.linear8(x, lin.w, lin.s, self.branch[:R], mode, proj=proj)

    def _moe_prefetch(self, lw, R):
        """(tensors, bytes) the routed experts' gate/up CTAs prefetch into L2: the next layer's first projections."""
        if getattr(self, "l2pf", False) and R <= K.GEMV_MAX_M:
            return self._next_layer_weights(lw), self.l2pf_bytes
        return [], 0

    def _next_layer_weights(self, lw):
        """The first bandwidth-bound projections of the layer after `lw` (none after the last layer)."""
        i = lw.index + 1
        if i >= len(self.w.layers):
            return []
        nl = self.w.layers[i]
        if nl.kind == "kda":
            return [nl.kda.in_proj.w, nl.kda.f_b.w]
        a = nl.mla
        return [a.qkv_a.w, a.q_b.w, a.index.wq_b.w]

    # ---- blocks ------------------------------------------------------------------------------------------------
    def _kda(self, lw, R):
        c, k, b = self.cfg, lw.kda, self.batch
        Kc = K.C()
        li = self.kda_index[lw.index]
        H, Dh = self.kH, self.kDh
        if self._keep_window:
            proj, fb, qkv = self.kproj_l[li][:R], self.kf_l[li][:R], self.kqkv_l[li][:R]
        else:
            proj, fb, qkv = self.kproj[:R], self.kf[:R], self.kqkv[:R]
        C3 = 3 * H * Dh
        if self._qin is not None:         # sequence-parallel chunk: rows arrived as e4m3 codes and row scales
            q, qs = self._qin
            self._qin = None
            Kc.gemm_w8q(q, qs, k.in_proj.w, k.in_proj.s, proj, K.GEMV_BF16, 0.0)
        else:
            K.linear8(self.normed[:R], k.in_proj.w, k.in_proj.s, proj, proj="kda_in_proj")
        if self._keep_window and self.kda_fused and Dh == 128 and c.conv == 4 and 1 <= b.max_rows_per_seq <= 16:
            # decode window: f_b, g_b, conv, recurrence and gated norm in one kernel (conv outputs and decay
            # logits stored for the commit replay)
            Kc.kda_decode(proj, b.kda_seq[:, :b.B], b.max_rows_per_seq, k.f_b.w, k.f_b.s, k.g_b.w, k.g_b.s, k.conv,
                          self.conv_pool[li], qkv, fb, k.a_log, k.dt_bias, k.o_norm, self.S_pool[li], self.kout[:R],
                          H, Dh, C3, C3 + 2 * Dh, c.lower, c.eps)
            self._final_linear(self.kout[:R], k.o_proj, R)
            return
        K.linear8(proj[:, C3:C3 + Dh], k.f_b.w, k.f_b.s, fb)
        side = getattr(self, "overlap", False) and R <= K.GEMV_MAX_M
        if side:        # output gate (read only by the gated norm) beside the convolution and recurrence
            self.ev_fork.record()
            with torch.cuda.stream(self.side):
                self.side.wait_event(self.ev_fork)
                K.linear8(proj[:, C3 + Dh:C3 + 2 * Dh], k.g_b.w, k.g_b.s, self.kg[:R])
                self.ev_join.record()
        else:
            K.linear8(proj[:, C3 + Dh:C3 + 2 * Dh], k.g_b.w, k.g_b.s, self.kg[:R])
        seq = b.kda_seq[:, :b.B]
        Kc.kda_conv(proj, seq, b.max_rows_per_seq, k.conv, self.conv_pool[li], qkv, H, Dh)
        if not self._keep_window:       # prefill chunk: every row is kept, shift the conv window now
            Kc.kda_conv_commit(proj, seq, self.conv_pool[li], H, Dh, c.conv)
        if self._keep_window or b.max_rows_per_seq <= KDA_CHUNK_MIN_ROWS:
            Kc.kda_recurrent(proj, seq, fb, qkv, k.a_log, k.dt_bias, self.S_pool[li], self.ko[:R], H, Dh,
                             C3 + 2 * Dh, c.lower)
        else:       # prefill: 64-token chunked form of the same recurrence
            Kc.kda_chunk(proj, seq, fb, qkv, k.a_log, k.dt_bias, self.S_pool[li], self.ko[:R], H, Dh,
                         C3 + 2 * Dh, c.lower, self.kda_scr)
        if side:
            torch.cuda.current_stream().wait_event(self.ev_join)
        Kc.kda_gated_norm(self.ko[:R], self.kg[:R], k.o_norm, self.kout[:R], H, Dh, c.eps)
        self._final_linear(self.kout[:R], k.o_proj, R)

    def _mla_rows(self, lw, R):
        """Row-parallel MLA for a sequence-parallel prefill chunk: the latent / index caches and the indexer keys
        for every row (each rank's rows attend to all earlier tokens), then the query, DSA selection, sparse
        attention and output projection of this rank's rows over all heads, with the full-head projections
        (``MLAW.full``).  The rows come out complete, so the block needs no reduce-scatter; the per-row key gathers
        of the attention are divided by the world size.  Measured at TP2 on the 32k cold prefill: 20,139 tok/s
        against 18,390 with head-parallel MLA blocks."""
        c, a, b = self.cfg, lw.mla, self.batch
        f = a.full
        Kc = K.C()
        li = self.mla_index[lw.index]
        H, L, rope, nope, qd = c.heads, c.kv_lora, c.qk_rope, c.qk_nope, c.qk_dim
        r0, r1 = self._sp
        n = r1 - r0
        K.linear8(self.normed[:R], a.qkv_a.w, a.qkv_a.s, self.qkv_a[:R])
        Kc.mla_prep(self.qkv_a[:R], a.q_norm, a.kv_norm, self.qr[:R], self.kv[li], self.kv_scale[li],
                    self.kpe[li] if rope else None, b.slots[:R], b.positions[:R], c.q_lora, L, rope, c.eps,
                    c.rope_theta)
        K.linear_bf16(self.normed[:R], a.index.proj, self.iproj[:R])
        Kc.dsa_update(self.iproj[:R], a.index.ln_w, a.index.ln_b, a.index.ape, self.ik_rows, self.ig_rows,
                      self.ik_ring[li], self.ig_ring[li], self.pool[li], self.pool_scale[li], b.slots[:R],
                      b.positions[:R], b.block_table, b.row_seq[:R], b.kda_seq[:, :b.B], self.rc.block_size,
                      c.index_heads, c.kpool, c.eps)
        # this rank's rows x all heads fit the per-rank buffers (R x H/W elements per row = n x H)
        q = self.q.view(-1)[:n * H * qd].view(n, H, qd)
        q_lat = self.q_lat.view(-1)[:n * H * L].view(n, H, L)
        o_lat = self.o_lat.view(-1)[:n * H * L].view(n, H, L)
        ob = self.obuf.view(-1)[:n * H * c.v_dim].view(n, H, c.v_dim)
        K.linear8(self.qr[r0:r1], f.q_b.w, f.q_b.s, q.view(n, H * qd))
        if rope:
            Kc.rope_q(q, b.positions[r0:r1], nope, rope, c.rope_theta)
        K.linear8(q[:, :, :nope].transpose(0, 1), f.w_uk_t.w, f.w_uk_t.s, q_lat.transpose(0, 1))
        K.linear8(self.qr[r0:r1], a.index.wq_b.w, a.index.wq_b.s, self.qi[r0:r1])
        AR = self.sel.shape[0]
        sm_scale = qd ** -0.5
        for s0 in range(0, n, AR):
            s1 = min(n, s0 + AR)
            m = s1 - s0
            g0, g1 = r0 + s0, r0 + s1
            Kc.dsa_select(self.iproj[g0:g1], self.qi[g0:g1], a.index.ln_w, self.pool[li], self.pool_scale[li],
                          b.positions[g0:g1], b.block_table, b.row_seq[g0:g1], self.rc.block_size, c.index_heads,
                          c.kpool, c.pools_selected, self.dsa_logits[:m], self.sel[:m], self.sel_count[:m])
            qpe = q[s0:s1, :, nope:] if rope else None
            Kc.mla_decode(q_lat[s0:s1], qpe, H * qd, qd, self.kv[li], self.kv_scale[li],
                          self.kpe[li] if rope else None, self.sel[:m], self.sel_count[:m], rope, sm_scale, 1,
                          self.part_o, self.part_ml, o_lat[s0:s1])
        K.linear8(o_lat.transpose(0, 1), f.w_uv.w, f.w_uv.s, ob.transpose(0, 1))
        K.linear8(ob.view(n, H * c.v_dim), f.o_proj.w, f.o_proj.s, self.branch[r0:r1], K.GEMV_F32,
                  proj="mla_o_proj")
        self._branch_local = True

    def _mla(self, lw, R):
        c, a, b = self.cfg, lw.mla, self.batch
        Kc = K.C()
        if self._sp is not None and a.full is not None:
            self._mla_rows(lw, R)
            return
        li = self.mla_index[lw.index]
        H, L, rope, nope = self.mH, c.kv_lora, c.qk_rope, c.qk_nope
        K.linear8(self.normed[:R], a.qkv_a.w, a.qkv_a.s, self.qkv_a[:R])
        Kc.mla_prep(self.qkv_a[:R], a.q_norm, a.kv_norm, self.qr[:R], self.kv[li], self.kv_scale[li],
                    self.kpe[li] if rope else None, b.slots[:R], b.positions[:R], c.q_lora, L, rope, c.eps,
                    c.rope_theta)
        K.linear8(self.qr[:R], a.q_b.w, a.q_b.s, self.q[:R].view(R, H * c.qk_dim))
        if rope:
            Kc.rope_q(self.q[:R], b.positions[:R], nope, rope, c.rope_theta)
        # absorbed query: q_lat[r, h] = q_nope[r, h] @ W_uk[h]   (batched over heads)
        K.linear8(self.q[:R, :, :nope].transpose(0, 1), a.w_uk_t.w, a.w_uk_t.s, self.q_lat[:R].transpose(0, 1))
        # indexer
        K.linear_bf16(self.normed[:R], a.index.proj, self.iproj[:R])
        Kc.dsa_update(self.iproj[:R], a.index.ln_w, a.index.ln_b, a.index.ape, self.ik_rows, self.ig_rows,
                      self.ik_ring[li], self.ig_ring[li], self.pool[li], self.pool_scale[li], b.slots[:R],
                      b.positions[:R], b.block_table, b.row_seq[:R], b.kda_seq[:, :b.B], self.rc.block_size,
                      c.index_heads, c.kpool, c.eps)
        K.linear8(self.qr[:R], a.index.wq_b.w, a.index.wq_b.s, self.qi[:R])
        AR = self.sel.shape[0]
        sm_scale = c.qk_dim ** -0.5
        # decode: split each row's keys so that rows x splits covers the SMs about twice (partials merged after)
        splits = max(1, min(self.splits, 2 * self.sms // max(R, 1))) if R <= self.rc.decode_rows else 1
        for r0 in range(0, R, AR):
            r1 = min(R, r0 + AR)
            n = r1 - r0
            Kc.dsa_select(self.iproj[r0:r1], self.qi[r0:r1], a.index.ln_w, self.pool[li], self.pool_scale[li],
                          b.positions[r0:r1], b.block_table, b.row_seq[r0:r1], self.rc.block_size, c.index_heads,
                          c.kpool, c.pools_selected, self.dsa_logits[:n], self.sel[:n], self.sel_count[:n])
            qpe = self.q[r0:r1, :, nope:] if rope else None
            Kc.mla_decode(self.q_lat[r0:r1], qpe, H * c.qk_dim, c.qk_dim, self.kv[li], self.kv_scale[li],
                          self.kpe[li] if rope else None, self.sel[:n], self.sel_count[:n], rope, sm_scale, splits,
                          self.part_o, self.part_ml, self.o_lat[r0:r1])
        ob = self.obuf[:R].view(R, H, c.v_dim)
        K.linear8(self.o_lat[:R].transpose(0, 1), a.w_uv.w, a.w_uv.s, ob.transpose(0, 1))
        self._final_linear(self.obuf[:R], a.o_proj, R, proj="mla_o_proj")

    def _mlp(self, lw, R):
        m = lw.mlp
        gu = self.gu_il[lw.index]
        act = self.act[:R, :m.width]
        K.linear8(self.normed[:R], gu.w, gu.s, act, K.GEMV_SWIGLU, self.cfg.limit)
        self._final_linear(act, m.down, R)

    def _moe_prefill(self, lw, R):
        """Routed experts of a prefill chunk: scalable routing, rotated inputs, tcgen05 gate/up and down with the
        trellis decoded into shared memory once per (expert, 128-channel block), then the slot-ordered combine."""
        c, m = self.cfg, lw.moe
        Kc = K.C()
        for r0 in range(0, R, self.p_rows):
            r1 = min(R, r0 + self.p_rows)
            n = r1 - r0
            P = n * c.top_k
            x = self.normed[r0:r1]
            K.linear_bf16(x, m.router, self.p_logits[:n])
            Kc.moe_route_large(self.p_logits[:n], m.bias, c.top_k, c.routed_scale, c.norm_topk, self.p_topk_ids[:n],
                               self.p_topk_w[:n], self.group_count, self.p_group_expert, self.p_group_offset,
                               self.p_pair_token[:P], self.p_pair_expert[:P], self.p_pair_w[:P],
                               self.p_pair_of[:P], self.p_counts, self.p_fill)
            Kc.exl3_rot_in(x, m.gate.suh, m.up.suh, self.p_pair_token[:P], self.p_pair_expert[:P], self.xh_g,
                           self.xh_u)
            Kc.moe_prefill(m.gate.trellis, m.up.trellis, m.gate.svh, m.up.svh, m.down.suh, None, self.group_count,
                           self.p_group_expert, self.p_group_offset, self.xh_g[:P], self.xh_u[:P], self.xd[:P],
                           c.limit, True)
            Kc.moe_prefill(m.down.trellis, None, m.down.svh, None, None, self.p_pair_w[:P], self.group_count,
                           self.p_group_expert, self.p_group_offset, self.xd[:P], None, self.yd[:P], c.limit, False)
            Kc.moe_combine(self.yd, self.p_pair_of[:P], c.top_k, self.branch[r0:r1], 0)

    def _moe_ep(self, lw, R):
        """Expert-parallel routed experts: rank j owns rows [j R / W, (j+1) R / W) of the layer input; its routed
        outputs land in those rows of the branch (zero elsewhere), so the tensor-parallel reduction of the branch
        (shared expert partials added) assembles every row."""
        W, j = self.tp, self.w.rank
        r0, r1 = R * j // W, R * (j + 1) // W
        self.branch[:R].zero_()
        self.ep[lw.index].forward(self.normed[r0:r1], out=self.branch[r0:r1])
        self._shared_expert(lw, R)

    def _moe(self, lw, R):
        c, m = self.cfg, lw.moe
        Kc = K.C()
        if getattr(self, "ep", None) is not None:
            self._moe_ep(lw, R)
            return
        if self.prefill_moe and R > MOE_PREFILL_MIN_ROWS:
            self._moe_prefill(lw, R)
            self._shared_expert(lw, R)
            return
        MR = self.rlogits.shape[0]
        if getattr(self, "overlap", False) and not self._fused and R <= MR:
            # the shared expert writes the branch on the side stream while the routed experts run; the routed
            # slot-ordered sum is formed first and the shared output added last (the same fp32 operations as the
            # sequential routed-then-shared order)
            s = m.shared
            self.ev_fork.record()
            with torch.cuda.stream(self.side):
                self.side.wait_event(self.ev_fork)
                act = self.act[:R, :s.width]
                K.linear8(self.normed[:R], self.gu_il[lw.index].w, self.gu_il[lw.index].s, act, K.GEMV_SWIGLU,
                          c.limit)
                K.linear8(act, s.down.w, s.down.s, self.branch[:R], K.GEMV_F32)
                self.ev_join.record()
            P = R * c.top_k
            x = self.normed[:R]
            K.linear_bf16(x, m.router, self.rlogits[:R])
            groups = min(P, c.experts)
            Kc.moe_route(self.rlogits[:R], m.bias, c.top_k, c.routed_scale, c.norm_topk, self.topk_ids[:R],
                         self.topk_w[:R], self.group_count, self.group_expert[:groups],
                         self.group_offset[:groups + 1], self.pair_token[:P], self.pair_expert[:P], self.pair_w[:P],
                         self.pair_of[:P])
            Kc.exl3_moe(x, m.gate.trellis, m.gate.suh, m.gate.svh, m.up.trellis, m.up.suh, m.up.svh,
                        m.down.trellis, m.down.suh, m.down.svh, self.group_count, self.group_expert[:groups],
                        self.group_offset[:groups + 1], self.pair_token[:P], self.pair_expert[:P], self.pair_w[:P],
                        self.xh_g, self.xh_u, self.xd, self.yd, c.limit, *self._moe_prefetch(lw, R))
            torch.cuda.current_stream().wait_event(self.ev_join)
            Kc.moe_combine(self.yd, self.pair_of[:P], c.top_k, self.branch[:R], 2)
            return
        for r0 in range(0, R, MR):
            r1 = min(R, r0 + MR)
            n = r1 - r0
            P = n * c.top_k
            x = self.normed[r0:r1]
            K.linear_bf16(x, m.router, self.rlogits[:n])
            groups = min(P, c.experts)
            Kc.moe_route(self.rlogits[:n], m.bias, c.top_k, c.routed_scale, c.norm_topk, self.topk_ids[:n],
                         self.topk_w[:n], self.group_count, self.group_expert[:groups],
                         self.group_offset[:groups + 1], self.pair_token[:P], self.pair_expert[:P], self.pair_w[:P],
                         self.pair_of[:P])
            pf = self._moe_prefetch(lw, R) if r0 == 0 else ([], 0)
            Kc.exl3_moe(x, m.gate.trellis, m.gate.suh, m.gate.svh, m.up.trellis, m.up.suh, m.up.svh,
                        m.down.trellis, m.down.suh, m.down.svh, self.group_count, self.group_expert[:groups],
                        self.group_offset[:groups + 1], self.pair_token[:P], self.pair_expert[:P], self.pair_w[:P],
                        self.xh_g, self.xh_u, self.xd, self.yd, c.limit, *pf)
            Kc.moe_combine(self.yd, self.pair_of[:P], c.top_k, self.branch[r0:r1], 0)
        self._shared_expert(lw, R)

    def _shared_expert(self, lw, R):
        """The shared expert (fp8 SwiGLU MLP), accumulated into the branch."""
        c, m = self.cfg, lw.moe
        s = m.shared
        gu = self.gu_il[lw.index]
        act = self.act[:R, :s.width]
        K.linear8(self.normed[:R], gu.w, gu.s, act, K.GEMV_SWIGLU, c.limit)
        self._final_linear(act, s.down, R, K.GEMV_F32_ACC)

    # ------------------------------------------------------------------------------------------------------------
    # commit of a verify window
    # ------------------------------------------------------------------------------------------------------------
    def stage_commit(self, seqs_keep):
        """Stage the per-sequence (row0, keep, s_in, s_out, conv_slot) of a commit (outside any graph)."""
        b = self.batch
        B = len(seqs_keep)
        sq = torch.as_tensor(seqs_keep, dtype=i32).t().contiguous()
        b.commit_seq[:, :B].copy_(sq)
        b.commit_B = B

    def commit(self, seqs_keep=None, replay: bool = True):
        """Keep rows of the last forward (run with keep_window): ``seqs_keep`` per sequence (row0, keep, s_in,
        s_out, conv_slot), or None to use the staged descriptor (graph replays).  ``replay`` re-runs the KDA
        recurrence over the kept rows (needed when a sequence keeps fewer rows than its window) so s_out holds
        the state after the last kept row; the conv windows shift by the kept rows."""
        b = self.batch
        Kc = K.C()
        if seqs_keep is not None:
            self.stage_commit(seqs_keep)
        seq = b.commit_seq[:, :b.commit_B]
        for lw in self.w.layers:
            if lw.kind != "kda":
                continue
            li = self.kda_index[lw.index]
            k = lw.kda
            H, Dh = self.kH, self.kDh
            C3 = 3 * H * Dh
            proj = self.kproj_l[li]
            if replay:
                Kc.kda_recurrent(proj, seq, self.kf_l[li], self.kqkv_l[li], k.a_log, k.dt_bias, self.S_pool[li],
                                 None, H, Dh, C3 + 2 * Dh, self.cfg.lower)
            Kc.kda_conv_commit(proj, seq, self.conv_pool[li], H, Dh, self.cfg.conv)


class Graphed:
    """A CUDA graph of one runtime call with fixed shapes (the batch buffers it reads are static).  Capture needs
    the batch staged with a valid window; warm-up runs on a side stream first, as CUDA graph capture requires."""

    def __init__(self, fn, warmup: int = 2):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = fn()

    def __call__(self):
        self.graph.replay()
        return self.out
