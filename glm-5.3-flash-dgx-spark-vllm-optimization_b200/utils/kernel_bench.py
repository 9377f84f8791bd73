"""Kernel microbenchmarks (one GPU): each case builds random inputs of the full model's shapes, times the kernel with
CUDA events after warm-up (an L2 flush -- a 256 MB write -- between timed iterations) and prints one JSON line with
the time and the achieved rate against the measured peaks (MEASURED_PEAKS.json when present).

  python -m glm53.utils.kernel_bench moe --tokens 1 8 64 512 8192 [--tp 1]      (BASELINE configs[1])
  python -m glm53.utils.kernel_bench gemv|gemm|kda|mla|all
  torchrun --nproc-per-node N -m glm53.utils.kernel_bench ag --rows 1024 4096    (fused all-gather + GEMM vs NCCL)
  torchrun --nproc-per-node N -m glm53.utils.kernel_bench ep --tokens 1 8 64 512   (experts
      EP-sharded over N GPUs, tokens per rank; dispatch/combine fused into the kernels)
  --iters 1 --warmup 1 makes a case small enough to capture under ncu
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0)
    return 6650.0, 1590.0


class Timer:
    def __init__(self, warmup: int, iters: int, flush: bool = True):
        self.warmup, self.iters = warmup, iters
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if flush else None

    def __call__(self, fn) -> float:
        for _ in range(self.warmup):
            fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(self.iters):
            if self.flush is not None:
                self.flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
        return tot / self.iters


def emit(d):
    print(json.dumps(d), flush=True)


def bench_moe(args, T: Timer):
    """One MoE layer: routing + routed EXL3 experts (+ combine), hidden 4096, 288 experts of width 2048/tp."""
    import glm53
    from glm53.models.runtime import Runtime, RuntimeConfig
    from glm53.models.weights import MoEW, MLPW, LayerW, Weights, quantize_fp8_rows
    from glm53.ops import exl3
    cfg = glm53.full_config(4)
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    D, W, E = cfg.hidden, cfg.moe_width // args.tp, cfg.experts
    from glm53.models.weights import Exl3Stack
    gate = Exl3Stack(*exl3.random_linear(D, W, generator=g, device=dev, lead=(E,)))
    up = Exl3Stack(*exl3.random_linear(D, W, generator=g, device=dev, lead=(E,)))
    down = Exl3Stack(*exl3.random_linear(W, D, generator=g, device=dev, lead=(E,)))
    router = (torch.randn(E, D, generator=g, device=dev) / math.sqrt(D)).to(torch.bfloat16)
    shared = MLPW(quantize_fp8_rows(torch.randn(2 * W, D, device=dev) / 64), quantize_fp8_rows(
        torch.randn(D, W, device=dev) / 45), W)
    moe = MoEW(router, torch.zeros(E, device=dev), gate, up, down, shared)
    hbm, _ = peaks()
    for n in args.tokens:
        rc = RuntimeConfig(max_rows=max(n, 16), kv_slots=64, block_size=64, max_blocks=1, moe_chunk=256,
                           moe_prefill_rows=8192)
        lw = LayerW(3, "mla", "moe", None, None, None, None, moe=moe)
        w = Weights(cfg, torch.zeros(16, D, dtype=torch.bfloat16, device=dev), [lw],
                    torch.ones(D, dtype=torch.bfloat16, device=dev), quantize_fp8_rows(torch.randn(16, D, device=dev)))
        rt = Runtime.__new__(Runtime)
        _moe_only_runtime(rt, w, rc, dev)
        rt.normed[:n].copy_(torch.randn(n, D, generator=g, device=dev).to(torch.bfloat16))
        ms = T(lambda: rt._moe(lw, n))
        # bytes: trellis of the distinct experts touched (4 bits/weight) + the shared expert
        distinct = int(min(E, E * (1 - (1 - 1 / E) ** (n * cfg.top_k))))
        wbytes = distinct * 3 * D * W // 2 + 3 * D * W
        emit({"case": "moe_layer", "tokens": n, "tp": args.tp, "ms": ms, "distinct_experts_est": distinct,
              "weight_GBps": wbytes / ms / 1e6, "frac_of_hbm": wbytes / ms / 1e6 / hbm,
              "path": "decode (in-register trellis, mma.sync)" if n <= 64 else "prefill (tcgen05, smem trellis)"})
        del rt


def _moe_only_runtime(rt, w, rc, dev):
    """A Runtime holding only the MoE scratch (no attention / KDA caches)."""
    from glm53.models import runtime as RT
    c = w.cfg
    rt.w, rt.rc, rt.comm, rt.cfg, rt.device, rt.tp = w, rc, None, c, dev, 1
    rt.px, rt._fused = None, False
    R = rc.max_rows
    D = c.hidden
    rt.gu_il = {lw.index: RT.interleave_gate_up(lw.moe.shared.gu) for lw in w.layers}
    rt.normed = torch.zeros(R, D, dtype=torch.bfloat16, device=dev)
    rt.branch = torch.zeros(R, D, dtype=torch.float32, device=dev)
    rt.act = torch.zeros(R, max(g.w.shape[0] // 2 for g in rt.gu_il.values()), dtype=torch.bfloat16, device=dev)
    MR = min(R, rc.moe_chunk)
    tk = c.top_k
    P = MR * tk
    rt.rlogits = torch.zeros(MR, c.experts, device=dev)
    rt.topk_ids = torch.zeros(MR, tk, dtype=torch.int32, device=dev)
    rt.topk_w = torch.zeros(MR, tk, device=dev)
    rt.max_groups = min(P, c.experts)
    rt.group_count = torch.zeros(1, dtype=torch.int32, device=dev)
    rt.group_expert = torch.zeros(rt.max_groups, dtype=torch.int32, device=dev)
    rt.group_offset = torch.zeros(rt.max_groups + 1, dtype=torch.int32, device=dev)
    for n in ("pair_token", "pair_expert", "pair_of"):
        setattr(rt, n, torch.zeros(P, dtype=torch.int32, device=dev))
    rt.pair_w = torch.zeros(P, device=dev)
    moe0 = w.layers[0].moe
    rt.prefill_moe = R > RT.MOE_PREFILL_MIN_ROWS
    if rt.prefill_moe:
        PR = min(R, rc.moe_prefill_rows)
        rt.p_rows = PR
        PP = PR * tk
        rt.p_logits = torch.zeros(PR, c.experts, device=dev)
        rt.p_topk_ids = torch.zeros(PR, tk, dtype=torch.int32, device=dev)
        rt.p_topk_w = torch.zeros(PR, tk, device=dev)
        rt.p_group_expert = torch.zeros(c.experts, dtype=torch.int32, device=dev)
        rt.p_group_offset = torch.zeros(c.experts + 1, dtype=torch.int32, device=dev)
        for n in ("p_pair_token", "p_pair_expert", "p_pair_of"):
            setattr(rt, n, torch.zeros(PP, dtype=torch.int32, device=dev))
        rt.p_pair_w = torch.zeros(PP, device=dev)
        rt.p_counts = torch.zeros(c.experts, dtype=torch.int32, device=dev)
        rt.p_fill = torch.zeros(c.experts, dtype=torch.int32, device=dev)
        P = max(P, PP)
    PX = max(P, 2 * MR * tk)          # the decode path's rotated inputs are duplicated f16 pairs
    rt.xh_g = torch.zeros(PX, D, dtype=torch.float16, device=dev)
    rt.xh_u = torch.zeros(PX, D, dtype=torch.float16, device=dev)
    rt.xd = torch.zeros(PX, moe0.gate.n, dtype=torch.float16, device=dev)
    rt.yd = torch.zeros(P, D, device=dev)


def bench_gemv(args, T: Timer):
    from glm53.models.weights import quantize_fp8_rows
    from glm53.ops import kernels as K
    hbm, _ = peaks()
    for (N, Kd, name) in [(24896, 4096, "kda_in_proj"), (4096, 8192, "kda_o_proj"), (4096, 16384, "mla_o_proj"),
                          (2048, 4096, "mla_qkv_a"), (154880, 4096, "lm_head"), (288, 4096, "router_bf16"),
                          (16384, 1536, "mla_q_b"), (4096, 4096, "shared_gate_up"), (4096, 2048, "shared_down"),
                          (24576, 4096, "dense_gate_up"), (4096, 12288, "dense_down")]:
        if args.proj and name not in args.proj:
            continue
        if args.tp > 1:
            # per-rank shape: row-parallel projections split K, replicated ones keep both, the rest split N
            if name in ("kda_o_proj", "mla_o_proj", "shared_down", "dense_down"):
                Kd //= args.tp
            elif name not in ("mla_qkv_a", "router_bf16"):
                N //= args.tp
        for M in args.rows:
            x = torch.randn(M, Kd, device="cuda").to(torch.bfloat16)
            y = torch.empty(M, N, device="cuda")
            if name == "router_bf16":
                w = (torch.randn(N, Kd, device="cuda") / 64).to(torch.bfloat16)
                ms = T(lambda: K.C().gemv(x, w, None, y, K.GEMV_F32, 0.0))
                nbytes = N * Kd * 2
            else:
                q = quantize_fp8_rows(torch.randn(N, Kd, device="cuda") / 64)
                nbytes = N * Kd
                if args.sweep:
                    # split-K shapes: warps per tile (ks) x cluster split (cl)
                    for ks in (1, 2, 4, 8):
                        for cl in (1, 2, 4, 8):
                            if Kd // 64 < ks * cl * 2:
                                continue
                            ms = T(lambda: K.C().gemv(x, q.w, q.s, y, K.GEMV_F32, 0.0, ks, cl))
                            emit({"case": "gemv_sweep", "proj": name, "M": M, "ks": ks, "cl": cl, "ms": ms,
                                  "frac_of_hbm": nbytes / ms / 1e6 / hbm})
                # size calibration: a device copy of the weight bytes (read + write) at this size
                dst = torch.empty_like(q.w)
                msc = T(lambda: dst.copy_(q.w))
                emit({"case": "gemv_copy_ref", "proj": name, "bytes": nbytes, "ms": msc,
                      "copy_GBps": 2 * nbytes / msc / 1e6})
                del dst
                # the two fp8 kernels: load-per-lane split-K (ks=-2: its own shape choice) and the bulk-copy ring
                # (ks=-1); "ms" is the default dispatch
                for kind, ks in (("loads", -2), ("bulk", -1)):
                    if kind == "bulk" and Kd % 512:
                        continue
                    msk = T(lambda: K.C().gemv(x, q.w, q.s, y, K.GEMV_F32, 0.0, ks, 0))
                    emit({"case": "gemv_kernel", "kernel": kind, "proj": name, "M": M, "ms": msk,
                          "frac_of_hbm": nbytes / msk / 1e6 / hbm})
                ms = T(lambda: K.C().gemv(x, q.w, q.s, y, K.GEMV_F32, 0.0))
            emit({"case": "gemv", "proj": name, "tp": args.tp, "M": M, "N": N, "K": Kd, "ms": ms, "GBps": nbytes / ms / 1e6,
                  "frac_of_hbm": nbytes / ms / 1e6 / hbm})


def bench_gemm(args, T: Timer):
    from glm53.models.weights import quantize_fp8_rows
    from glm53.ops import kernels as K
    _, tflops = peaks()
    for (M, N, Kd) in [(8192, 24896, 4096), (8192, 4096, 8192), (8192, 24576, 4096), (4096, 4096, 4096)]:
        x = torch.randn(M, Kd, device="cuda").to(torch.bfloat16)
        q = quantize_fp8_rows(torch.randn(N, Kd, device="cuda") / 64)
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        scratch = torch.empty(N * Kd, dtype=torch.bfloat16, device="cuda")
        ms = T(lambda: K.C().gemm_w8a16(x, q.w, q.s, y, K.GEMV_BF16, 0.0, scratch))
        wb = scratch[:N * Kd].view(N, Kd)
        ms_bf = T(lambda: K.C().gemm_bf16(x, wb, q.s, y, K.GEMV_BF16, 0.0))
        fl = 2.0 * M * N * Kd
        emit({"case": "gemm_tcgen05", "M": M, "N": N, "K": Kd, "ms_w8a16": ms, "ms_bf16_only": ms_bf,
              "tflops": fl / ms_bf / 1e9, "frac_of_bf16_peak": fl / ms_bf / 1e9 / tflops})


def bench_kda(args, T: Timer):
    from glm53.ops import kernels as K
    H, Dh = 64 // args.tp, 128
    for Tn in args.kda_rows:
        HD = H * Dh
        ldp = (3 * HD + 2 * Dh + H + 63) // 64 * 64
        proj = (torch.randn(Tn, ldp, device="cuda") * 0.5).to(torch.bfloat16)
        qkv = torch.randn(Tn, 3 * HD, device="cuda").to(torch.bfloat16)
        f = torch.randn(Tn, HD, device="cuda").to(torch.bfloat16)
        a_log = torch.zeros(H, device="cuda")
        dt = torch.zeros(HD, device="cuda")
        S = torch.zeros(2, H, Dh, Dh, device="cuda")
        o = torch.empty(Tn, HD, device="cuda")
        seq = torch.tensor([[0], [Tn], [0], [1], [0]], dtype=torch.int32, device="cuda")
        if Tn > 32:
            scr = torch.empty(K.C().kda_chunk_scratch_floats(Tn, 1, H, Dh), device="cuda")
            ms = T(lambda: K.C().kda_chunk(proj, seq, f, qkv, a_log, dt, S, o, H, Dh, 3 * HD + 2 * Dh, -5.0, scr))
        else:
            ms = T(lambda: K.C().kda_recurrent(proj, seq, f, qkv, a_log, dt, S, o, H, Dh, 3 * HD + 2 * Dh, -5.0))
        emit({"case": "kda_chunk" if Tn > 32 else "kda_recurrent", "rows": Tn, "heads": H, "ms": ms,
              "tokens_per_s": Tn / ms * 1e3})
        if Tn <= 16:
            # the decode window's whole KDA block tail: fused kernel against the five-kernel sequence
            from glm53.models.weights import quantize_fp8_rows
            fb = quantize_fp8_rows(torch.randn(HD, Dh, device="cuda") / Dh ** 0.5)
            gb = quantize_fp8_rows(torch.randn(HD, Dh, device="cuda") / Dh ** 0.5)
            conv_w = torch.randn(3 * HD, 4, device="cuda") * 0.3
            conv_pool = (torch.randn(2, 3, 3 * HD, device="cuda") * 0.5).to(torch.bfloat16)
            o_norm = torch.ones(Dh, device="cuda", dtype=torch.bfloat16)
            out = torch.empty(Tn, HD, device="cuda", dtype=torch.bfloat16)
            gate = torch.empty(Tn, HD, device="cuda", dtype=torch.bfloat16)
            C3 = 3 * HD
            ms_f = T(lambda: K.C().kda_decode(proj, seq, Tn, fb.w, fb.s, gb.w, gb.s, conv_w, conv_pool, qkv, f, a_log,
                                              dt, o_norm, S, out, H, Dh, C3, C3 + 2 * Dh, -5.0, 1e-6))

            def five():
                K.linear8(proj[:, C3:C3 + Dh], fb.w, fb.s, f)
                K.linear8(proj[:, C3 + Dh:C3 + 2 * Dh], gb.w, gb.s, gate)
                K.C().kda_conv(proj, seq, Tn, conv_w, conv_pool, qkv, H, Dh)
                K.C().kda_recurrent(proj, seq, f, qkv, a_log, dt, S, o, H, Dh, C3 + 2 * Dh, -5.0)
                K.C().kda_gated_norm(o, gate, o_norm, out, H, Dh, 1e-6)
            ms_5 = T(five)
            emit({"case": "kda_decode_window", "rows": Tn, "heads": H, "ms_fused": ms_f, "ms_five_kernels": ms_5})


def bench_mla(args, T: Timer):
    from glm53.ops import kernels as K
    H, L = 64 // args.tp, 512
    for R in args.mla_rows:
        slots = 8192
        q = torch.randn(R, H, L, device="cuda").to(torch.bfloat16)
        kv = torch.randint(0, 120, (slots, L), dtype=torch.uint8, device="cuda")
        sc = torch.rand(slots, device="cuda") * 0.01
        sel = torch.randint(0, slots, (R, 2048), dtype=torch.int32, device="cuda")
        cnt = torch.full((R,), 2048, dtype=torch.int32, device="cuda")
        fl = 4.0 * R * H * 2048 * L
        for tcores in (0, 1):
            # decode rows: key splits so that rows x splits fills the SMs (merged by a second kernel)
            splits = (4 if not tcores else max(1, min(16, 148 // R))) if R <= 16 else 1
            po = torch.empty(R * splits * H * L, device="cuda")
            pm = torch.empty(R * splits * H * 2, device="cuda")
            o = torch.empty_like(q)
            ms = T(lambda: K.C().mla_decode(q, None, 0, 0, kv, sc, None, sel, cnt, 0, 0.0625, splits, po, pm, o,
                                            tcores))
            emit({"case": "mla_sparse_attn", "kernel": "tcgen05" if tcores else "mma.sync", "rows": R, "heads": H,
                  "keys": 2048, "splits": splits, "ms": ms, "tflops": fl / ms / 1e9})


def bench_ep(args, T: Timer):
    """One routed-MoE layer, experts sharded over the ranks; per step: route -> dispatch (peer stores) -> expert
    GEMMs -> combine (peer stores from the down epilogue) -> slot-ordered sum.  Time = max over ranks of the CUDA
    event time per step; roofline = slower of the expert-weight bytes at measured HBM bandwidth and the bytes a
    rank sends over NVLink (dispatch bf16 rows + combine fp32 rows to other ranks) at 770 GB/s per direction."""
    import torch.distributed as dist
    from glm53 import full_config
    from glm53.models import weights as W
    from glm53.parallel import dist as D
    from glm53.parallel.ep import EPMoE, local_experts
    rank, local, world = D.init(timeout_s=120)
    cfg = full_config(layers=4)
    dev = torch.device("cuda", local)
    src = W.RandomSource(cfg, seed=0, device=dev)
    li = next(i for i, m in enumerate(cfg.mlp_kinds) if m == "moe") if hasattr(cfg, "mlp_kinds") else 3
    stacks = {p: src.experts(li, p, cfg.experts) for p in ("gate_proj", "up_proj", "down_proj")}
    g = torch.Generator(device=dev).manual_seed(7)
    router = (torch.randn(cfg.experts, cfg.hidden, generator=g, device=dev) / math.sqrt(cfg.hidden)).to(torch.bfloat16)
    bias = torch.zeros(cfg.experts, device=dev)
    ep = EPMoE(cfg, router, bias, local_experts(stacks["gate_proj"], rank, world),
               local_experts(stacks["up_proj"], rank, world), local_experts(stacks["down_proj"], rank, world),
               max_tokens=max(args.tokens), rank=rank, world=world)
    del stacks
    hbm, _ = peaks()
    gx = torch.Generator(device=dev).manual_seed(100 + rank)
    for Tn in args.tokens:
        x = torch.randn(Tn, cfg.hidden, generator=gx, device=dev).to(torch.bfloat16)
        for _ in range(args.warmup):
            ep.forward(x)
        torch.cuda.synchronize()
        ep.x_ex.check()
        dist.barrier() if world > 1 else None
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            ep.forward(x)
        e1.record()
        torch.cuda.synchronize()
        ep.x_ex.check()
        ms = e0.elapsed_time(e1) / args.iters
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        P = Tn * cfg.top_k
        # distinct local experts hit (expected, uniform routing over all ranks' tokens)
        E, El = cfg.experts, cfg.experts // world
        hits = El * (1 - (1 - 1 / E) ** (P * world))
        w_bytes = hits * 3 * cfg.hidden * cfg.moe_width * cfg.bits / 8
        nv_bytes = P * (world - 1) / world * cfg.hidden * (2 + 4)
        roof_ms = max(w_bytes / (hbm * 1e6), nv_bytes / (770.0 * 1e6))
        if rank == 0:
            emit({"case": "ep_moe_layer", "world": world, "tokens_per_rank": Tn, "ms": ms,
                  "tokens_per_s": Tn * world / ms * 1e3, "path": "tcgen05" if ep.tensor_core_experts(Tn) else
                  "register-decode", "hbm_weight_bytes": w_bytes, "nvlink_bytes_per_rank": nv_bytes,
                  "roofline_ms": roof_ms, "frac_of_roofline": roof_ms / ms})
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def bench_ag(args, T: Timer):
    """All-gather + GEMM of a column-parallel projection (KDA in_proj: K 4096 -> N 24896 / W) over the ranks'
    row shards: fused (the GEMM's TMA producer loads peer shards) vs NCCL all_gather_into_tensor + the same GEMM.
    Roofline: slower of the GEMM at measured bf16 peak and the (W-1) shards over NVLink at 770 GB/s."""
    import torch.distributed as dist
    from glm53.models.weights import quantize_fp8_rows
    from glm53.ops import kernels as K
    from glm53.parallel import dist as D
    from glm53.parallel.ag_gemm import AGGemm
    rank, local, world = D.init(timeout_s=120)
    dev = torch.device("cuda", local)
    _, peak = peaks()
    Kd, N = 4096, (24896 // world + 15) // 16 * 16
    w = quantize_fp8_rows(torch.randn(N, Kd, device=dev) / math.sqrt(Kd))
    for rows in args.rows:
        bufs = [AGGemm(rows, Kd, dev), AGGemm(rows, Kd, dev)]
        y = torch.empty(world * rows, N, device=dev, dtype=torch.bfloat16)
        mine = torch.randn(rows, Kd, device=dev).to(torch.bfloat16)
        gathered = torch.empty(world * rows, Kd, device=dev, dtype=torch.bfloat16)
        step = [0]

        def fused():
            ag = bufs[step[0] % 2]
            step[0] += 1
            ag.shard.copy_(mine)
            ag.publish()
            ag.gemm(w.w, w.s, y, K.GEMV_BF16)

        def nccl():
            if world > 1:
                dist.all_gather_into_tensor(gathered, mine)
            else:
                gathered.copy_(mine)
            K.linear8(gathered, w.w, w.s, y, K.GEMV_BF16)

        res = {}
        for name, fn in (("fused", fused), ("nccl", nccl)):
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.iters
            if world > 1:
                t = torch.tensor([ms], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = t.item()
            res[name] = ms
        flops = 2.0 * world * rows * N * Kd
        nv = (world - 1) * rows * Kd * 2
        roof = max(flops / (peak * 1e9), nv / (770.0 * 1e6))
        if rank == 0:
            emit({"case": "ag_gemm", "world": world, "rows_per_rank": rows, "N": N, "K": Kd, "ms_fused": res["fused"],
                  "ms_nccl_allgather_plus_gemm": res["nccl"], "roofline_ms": roof,
                  "frac_of_roofline_fused": roof / res["fused"]})
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def bench_hc(args, T: Timer):
    """mHC post (4 streams) fused with the next pre (24 mixing logits, Sinkhorn, collapse, rmsnorm) for R rows."""
    from glm53.ops import kernels as K
    S, D, NM = 4, 4096, 24
    dev = "cuda"
    for R in args.rows:
        X = torch.randn(R, S, D, device=dev).to(torch.bfloat16)
        branch = torch.randn(R, D, device=dev)
        post = torch.rand(R, S, device=dev)
        comb = torch.rand(R, S, S, device=dev) / S
        fn = (torch.randn(NM, S * D, device=dev) / math.sqrt(S * D)).to(torch.bfloat16)
        base = torch.zeros(NM, device=dev)
        hscale = torch.ones(3, device=dev)
        norm_w = torch.ones(D, device=dev).to(torch.bfloat16)
        normed = torch.empty(R, D, device=dev).to(torch.bfloat16)
        post_o, comb_o = torch.empty(R, S, device=dev), torch.empty(R, S, S, device=dev)
        part = torch.empty(R * (D // 64) * 32, device=dev)
        for tcores in ((1, 0) if R >= 256 else (0,)):
            ms = T(lambda: K.C().hc_post_pre(X, branch, post, comb, fn, base, hscale, norm_w, normed, post_o,
                                              comb_o, part, 1e-5, 1e-6, 20, tcores))
            fused = R <= 16 and os.environ.get("GLM53_HC_FUSED", "1") == "1"
            path = "tcgen05" if tcores else ("cluster, one kernel" if fused else "cuda-core, two kernels")
            emit({"case": "hc_post_pre", "path": path, "rows": R, "ms": ms,
                  "GBps": (R * S * D * 2 * 2 + R * D * 4 + NM * S * D * 2 + R * D * 2 * 2) / ms / 1e6})


def bench_dsa(args, T: Timer):
    """DSA indexer at decode: pool logits (CUDA-core kernel, the decode path) and the radix top-k selection for R
    query rows at the end of a `--context`-token sequence (full config: 32 index heads x 128, pools of 4 tokens,
    top 512 pools); the e4m3 pool cache is random, one page table of 64-token pages."""
    from glm53.ops import kernels as K
    C = K.C()
    dev = "cuda"
    IH, ID, kpool, bs, topk_pools = 32, 128, 4, 64, 2048 // 4
    g = torch.Generator(device=dev).manual_seed(0)
    for ctx in args.context:
        for R in args.rows:
            pages = (ctx + bs - 1) // bs
            npools = pages * bs // kpool
            raw = torch.randint(0, 256, (npools, ID), generator=g, device=dev, dtype=torch.int32)
            raw[(raw == 0x7F) | (raw == 0xFF)] = 0
            pool_cache = raw.to(torch.uint8)
            pool_scale = torch.ones(npools, device=dev)
            bt = torch.randperm(pages, device=dev, generator=g).to(torch.int32).view(1, pages)
            iproj = torch.randn(R, ID + IH + ID, device=dev, generator=g)
            qi = torch.randn(R, IH * ID, device=dev, generator=g).to(torch.bfloat16)
            positions = torch.arange(ctx - R, ctx, device=dev, dtype=torch.int32)
            row_seq = torch.zeros(R, device=dev, dtype=torch.int32)
            ln_w = torch.ones(ID, device=dev)
            logits = torch.empty(R, npools, device=dev)
            sel = torch.empty(R, topk_pools * kpool, device=dev, dtype=torch.int32)
            cnt = torch.empty(R, device=dev, dtype=torch.int32)
            ms_l = T(lambda: C.dsa_logits(iproj, qi, ln_w, pool_cache, pool_scale, positions, bt, row_seq, bs, IH,
                                          kpool, logits, False))
            ms_t = T(lambda: C.dsa_logits(iproj, qi, ln_w, pool_cache, pool_scale, positions, bt, row_seq, bs, IH,
                                          kpool, logits, True))
            ms_s = T(lambda: C.dsa_select(iproj, qi, ln_w, pool_cache, pool_scale, positions, bt, row_seq, bs, IH,
                                          kpool, topk_pools, logits, sel, cnt))
            emit({"case": "dsa_decode", "context": ctx, "rows": R, "pools": npools, "ms_logits_cuda_cores": ms_l,
                  "ms_logits_tcgen05": ms_t, "ms_select_default_path": ms_s,
                  "pool_cache_GBps_cuda_cores": npools * ID / ms_l / 1e6})


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["moe", "gemv", "gemm", "kda", "mla", "ep", "hc", "ag", "dsa", "all"])
    ap.add_argument("--tokens", type=int, nargs="+", default=[1, 8, 64, 512, 8192])
    ap.add_argument("--rows", type=int, nargs="+", default=[8])
    ap.add_argument("--kda-rows", type=int, nargs="+", default=[8, 8192])
    ap.add_argument("--mla-rows", type=int, nargs="+", default=[8, 1024])
    ap.add_argument("--context", type=int, nargs="+", default=[4096, 131072, 524288],
                    help="dsa: context lengths (tokens)")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--no-flush", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="gemv: every split-K shape")
    ap.add_argument("--proj", nargs="+", default=None, help="gemv: only these projections")
    args = ap.parse_args(argv)
    import sys
    sys.path.insert(0, ROOT)
    import glm53  # noqa: F401
    T = Timer(args.warmup, args.iters, flush=not args.no_flush)
    cases = ["moe", "gemv", "gemm", "kda", "mla"] if args.case == "all" else [args.case]
    for c in cases:
        globals()["bench_" + c](args, T)


if __name__ == "__main__":
    main()
