"""Receive buffers for the fused tensor-parallel reduction of decode windows.

Every rank owns one symmetric buffer (mapped into every peer's address space; torch symmetric memory does the
mapping, the kernels do all the traffic):

  data   [2 parities][world slots][rows * D] fp32    slot j of parity p = rank j's partial of the p-th reduction
  flags  [2 parities][world] u32                     flags[p][j] counts rank j's completed pushes into parity p

Producer (csrc/gemv.cu, push mode): the row-parallel GEMV that ends a block stores its fp32 partial into slot
`rank` of parity p on every rank (peer stores over NVLink) and its last CTA raises flags[p][rank] on every rank
(release).  Consumer (csrc/mhc.cu, hc_post_pre with gath): waits until flags[p][j] >= epoch[p] + 1 for every j
(acquire, bounded), sums the slots in rank order -- identical bits on every rank -- and bumps its local epoch[p].
Reductions alternate parity, so a rank that runs ahead writes the other buffer; it can only come back to this one
after consuming the next reduction, which every peer produces after finishing its own read of this one.

This replaces the all-reduce the reference issues per block (NCCL AllReduce_Sum_bf16_RING_LL, 102 per decode
step: code/fork/docs/DEC_AR1SHOT.md:10-14; its one-shot variant is all-gather + local add,
code/fork/glm53_ar1shot.py:100-140, which is what this does inside the kernels).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class PeerExchange:
    def __init__(self, rows: int, D: int, device, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.D = rows, D
        self.slot = rows * D
        W = self.world
        data_bytes = 2 * W * self.slot * 4
        flag_bytes = 2 * W * 4
        total = data_bytes + ((flag_bytes + 255) // 256) * 256
        group = group or dist.group.WORLD
        try:
            symm_mem.enable_symm_mem_for_group(group.group_name)
        except Exception:
            pass
        self.buf = symm_mem.empty(total, dtype=torch.uint8, device=device)
        self.handle = symm_mem.rendezvous(self.buf, group.group_name)
        self.buf.zero_()
        ptrs = list(self.handle.buffer_ptrs)
        dev = torch.device(device)
        self.push_ptrs = [torch.tensor([ptrs[j] + p * W * self.slot * 4 for j in range(W)], dtype=torch.int64,
                                       device=dev) for p in range(2)]
        self.push_flags = [torch.tensor([ptrs[j] + data_bytes + p * W * 4 for j in range(W)], dtype=torch.int64,
                                        device=dev) for p in range(2)]
        f32 = self.buf[:data_bytes].view(torch.float32).view(2, W * self.slot)
        self.gath = [f32[p] for p in range(2)]
        fl = self.buf[data_bytes:data_bytes + flag_bytes].view(torch.int32).view(2, W)
        self.flags = [fl[p] for p in range(2)]
        self.epoch = torch.zeros(2, dtype=torch.int32, device=dev)
        self.done_cons = torch.zeros(2, dtype=torch.int32, device=dev)
        self.done_prod = torch.zeros(2, dtype=torch.int32, device=dev)
        self.err = torch.zeros(4, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        dist.barrier(group)

    def check(self) -> None:
        """Raise if a bounded wait of a fused kernel ran out (a peer did not arrive)."""
        e = int(self.err[0].item())
        if e:
            self.err.zero_()
            raise RuntimeError(f"fused tensor-parallel exchange timed out waiting for a peer (code {e})")
