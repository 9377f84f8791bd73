"""Expert-parallel routed MoE with the all-to-all dispatch and combine inside the kernels (csrc/ep_moe.cu).

Rank d of the group owns the experts [d*El, (d+1)*El) at full width (El = experts / world).  Every rank routes
its own tokens, pushes each (token, expert) row to the owner's receive buffer with peer stores, the owner runs its
experts once over all rows it received (grouped by expert, so each expert's trellis is decoded once per step), and
the down projection's epilogue stores every weighted output row straight into the source rank's combine buffer;
the source then sums each token's top-k rows in slot order.  Flags (release / bounded acquire) replace NCCL's
all-to-all; two buffer parities let a rank run one step ahead.

Symmetric buffer of one rank (one set per parity p; peers see it through torch symmetric memory):

    recv_x     bf16 [world src][cap][K]     rows dispatched to this rank
    recv_meta  int4 [world src][cap]        {local expert, source pair index, routing weight bits, 0}
    recv_cnt   i32  [world src][El]         rows per local expert from each source
    comb       f32  [cap][K]                this rank's pair outputs, written by the owner ranks
    disp_flag  u32  [world]                 steps dispatched to this rank, per source
    comb_flag  u32  [world]                 steps whose outputs arrived here, per owner rank

Reference: the reference's EP path (expert_map with a sentinel for non-local experts,
code/fork/docs/prod_exl3_reference.py:924-958) is implemented but not deployed; it would use NCCL all2all.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..models.weights import Exl3Stack
from ..ops import kernels as K


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


def local_experts(stack: Exl3Stack, rank: int, world: int) -> Exl3Stack:
    """The experts owned by `rank` (contiguous block of E / world)."""
    E = stack.trellis.shape[0]
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    el = E // world
    s = slice(rank * el, (rank + 1) * el)
    return Exl3Stack(stack.trellis[s].contiguous(), stack.suh[s].contiguous(), stack.svh[s].contiguous())


class EPExchange:
    """Symmetric receive / combine buffers and the peer address tables of both parities."""

    def __init__(self, world: int, rank: int, El: int, cap: int, K: int, device, group=None):
        self.world, self.rank, self.El, self.cap, self.K = world, rank, El, cap, K
        W = world
        sizes = [("recv_x", W * cap * K * 2), ("meta", W * cap * 16), ("cnt", W * El * 4), ("comb", cap * K * 4),
                 ("disp", W * 4), ("combf", W * 4)]
        self.off = {}
        o = 0
        for p in range(2):
            for name, n in sizes:
                self.off[(p, name)] = o
                o += _align(n)
        total = o
        dev = torch.device(device)
        if W == 1:
            self.buf = torch.zeros(total, dtype=torch.uint8, device=dev)
            ptrs = [self.buf.data_ptr()]
        else:
            import torch.distributed._symmetric_memory as symm_mem
            group = group or dist.group.WORLD
            try:
                symm_mem.enable_symm_mem_for_group(group.group_name)
            except Exception:
                pass
            self.buf = symm_mem.empty(total, dtype=torch.uint8, device=dev)
            self.handle = symm_mem.rendezvous(self.buf, group.group_name)
            self.buf.zero_()
            ptrs = list(self.handle.buffer_ptrs)
        self.peer, self.local = [], []
        for p in range(2):
            f = lambda name, d: ptrs[d] + self.off[(p, name)]
            tab = [[f("recv_x", d) for d in range(W)], [f("meta", d) for d in range(W)],
                   [f("cnt", d) for d in range(W)], [f("disp", d) + 4 * rank for d in range(W)],
                   [f("comb", d) for d in range(W)], [f("combf", d) + 4 * rank for d in range(W)]]
            self.peer.append(torch.tensor(tab, dtype=torch.int64, device=dev))
            own = ptrs[rank]
            self.local.append(torch.tensor([own + self.off[(p, "disp")], own + self.off[(p, "combf")],
                                            own + self.off[(p, "cnt")], own + self.off[(p, "meta")],
                                            own + self.off[(p, "comb")], own + self.off[(p, "recv_x")]],
                                           dtype=torch.int64))
        # per parity: counters, pair count, received rows, epoch, error word
        self.state = torch.zeros(2, 16, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        if W > 1:
            dist.barrier(group)

    def check(self) -> None:
        e = self.state[:, 8].tolist()
        if any(e):
            self.state[:, 8].zero_()
            raise RuntimeError(f"expert-parallel exchange error codes {e} (51/54: a peer did not arrive in time, "
                               f"52/53: a receive buffer overflowed)")


class EPBuffers:
    """The exchange and the scratch of the expert-parallel MoE, shared by every MoE layer of a model (the layers run
    one after another, each step alternating the exchange's parity)."""

    def __init__(self, cfg, N: int, max_tokens: int, rank: int = 0, world: int = 1, group=None, device="cuda"):
        dev = torch.device(device)
        E, tk = cfg.experts, cfg.top_k
        self.El = E // world
        Kd = cfg.hidden
        self.max_tokens = max_tokens
        self.cap = max(1, max_tokens) * tk
        self.recv_cap = world * self.cap
        self.x_ex = EPExchange(world, rank, self.El, self.cap, Kd, dev, group)
        i32, f32 = torch.int32, torch.float32
        T, P = max(1, max_tokens), self.cap
        self.logits = torch.zeros(T, E, dtype=f32, device=dev)
        self.topk_ids = torch.zeros(T, tk, dtype=i32, device=dev)
        self.topk_w = torch.zeros(T, tk, dtype=f32, device=dev)
        G = min(P, E)
        self.group_count = torch.zeros(1, dtype=i32, device=dev)
        self.group_expert = torch.zeros(max(G, E), dtype=i32, device=dev)
        self.group_offset = torch.zeros(max(G, E) + 1, dtype=i32, device=dev)
        self.pair_token = torch.zeros(P, dtype=i32, device=dev)
        self.pair_expert = torch.zeros(P, dtype=i32, device=dev)
        self.pair_w = torch.zeros(P, dtype=f32, device=dev)
        self.pair_of = torch.zeros(P, dtype=i32, device=dev)
        self.counts = torch.zeros(E, dtype=i32, device=dev)
        self.fill = torch.zeros(E, dtype=i32, device=dev)
        W, El, RC = world, self.El, self.recv_cap
        self.seg = torch.zeros(3 * W * El, dtype=i32, device=dev)
        self.groups = torch.zeros(2 + 2 * El, dtype=i32, device=dev)
        self.rp_i = torch.zeros(2 * RC, dtype=i32, device=dev)
        self.rp_w = torch.zeros(RC, dtype=f32, device=dev)
        self.rp_out = torch.zeros(RC, dtype=torch.int64, device=dev)
        self.xh_g = torch.zeros(RC * 2 * Kd, dtype=torch.float16, device=dev)
        self.xh_u = torch.zeros(RC * 2 * Kd, dtype=torch.float16, device=dev)
        self.xd = torch.zeros(RC * 2 * N, dtype=torch.float16, device=dev)
        self.out = torch.zeros(T, Kd, dtype=f32, device=dev)
        self.step = 0


class EPMoE:
    """One routed-MoE layer, experts sharded over the process group; forward(x [T, K] bf16) -> [T, K] fp32.  The
    exchange and scratch come from ``bufs`` (shared by the layers of a model) or are allocated for this layer."""

    def __init__(self, cfg, router: torch.Tensor, bias: torch.Tensor, gate: Exl3Stack, up: Exl3Stack,
                 down: Exl3Stack, max_tokens: int, rank: int = 0, world: int = 1, group=None, device="cuda",
                 bufs: EPBuffers | None = None):
        self.cfg, self.rank, self.world = cfg, rank, world
        self.gate, self.up, self.down = gate, up, down           # local experts (El)
        self.router, self.bias = router, bias
        self.b = bufs or EPBuffers(cfg, gate.n, max_tokens, rank, world, group, device)
        self.El = self.b.El
        self.max_tokens = self.b.max_tokens
        self.cap, self.recv_cap = self.b.cap, self.b.recv_cap
        self.x_ex = self.b.x_ex

    def __getattr__(self, name):
        # scratch tensors live in the shared buffers
        b = self.__dict__.get("b")
        if b is not None and hasattr(b, name):
            return getattr(b, name)
        raise AttributeError(name)

    @property
    def step(self) -> int:
        return self.b.step

    @step.setter
    def step(self, v: int) -> None:
        self.b.step = v

    def tensor_core_experts(self, T: int) -> bool:
        """tcgen05 grouped GEMMs (trellis decoded into shared memory) once the rows per local expert reach 16;
        the register-decode (mma.sync) kernels below that.  Each rank decides for the rows it receives (about
        T * top_k with balanced routing)."""
        return T * self.cfg.top_k >= 16 * self.El and self.gate.n % 128 == 0

    @torch.no_grad()
    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """x [T, K] bf16 -> [T, K] fp32 (into ``out`` when given: a contiguous fp32 [T, K] view)."""
        c = self.cfg
        Kc = K.C()
        T = x.shape[0]
        dst = self.out[:T] if out is None else out
        if T > self.max_tokens:
            raise ValueError("more tokens than the exchange buffers hold")
        tk = c.top_k
        P = T * tk
        p = self.step & 1
        if T > 0:
            K.linear_bf16(x, self.router, self.logits[:T])
        if T == 0:
            pass
        elif P <= 2048:
            G = min(P, c.experts)
            Kc.moe_route(self.logits[:T], self.bias, tk, c.routed_scale, c.norm_topk, self.topk_ids[:T],
                         self.topk_w[:T], self.group_count, self.group_expert[:G], self.group_offset[:G + 1],
                         self.pair_token[:P], self.pair_expert[:P], self.pair_w[:P], self.pair_of[:P])
        else:
            Kc.moe_route_large(self.logits[:T], self.bias, tk, c.routed_scale, c.norm_topk, self.topk_ids[:T],
                               self.topk_w[:T], self.group_count, self.group_expert[:c.experts],
                               self.group_offset[:c.experts + 1], self.pair_token[:P], self.pair_expert[:P],
                               self.pair_w[:P], self.pair_of[:P], self.counts, self.fill)
        ex = self.x_ex
        st = ex.state[p]
        st[3].fill_(P)
        Kc.ep_moe_step(x, dst, self.pair_token[:P], self.pair_expert[:P], self.pair_w[:P],
                       self.pair_of[:P], self.gate.trellis, self.gate.suh, self.gate.svh, self.up.trellis,
                       self.up.suh, self.up.svh, self.down.trellis, self.down.suh, self.down.svh, ex.peer[p],
                       ex.local[p], st, self.seg, self.groups, self.rp_i, self.rp_w, self.rp_out, self.xh_g,
                       self.xh_u, self.xd, self.El, self.rank, self.world, self.cap, self.recv_cap, tk, c.limit,
                       self.tensor_core_experts(T))
        self.step += 1
        return dst
