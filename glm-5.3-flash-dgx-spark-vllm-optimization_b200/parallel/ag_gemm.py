"""All-gather + GEMM on a column-parallel input (the input rows are sharded over the ranks, e.g. sequence-parallel
prefill): y [W * rows, N_local] = concat_j(A_j) @ W_local^T inside one tcgen05 GEMM.  A rank publishes its shard
by writing it into its symmetric buffer and raising flag [rank] on every rank (release).  In the GEMM, the epilogue
warps of every CTA first copy a share of the peers' 128-row blocks over NVLink into a local staging buffer (each
remote block crosses NVLink once) and mark each block ready; the TMA producer reads this rank's own tiles straight
away and a peer's tiles from the staging buffer once their block is ready, so the gather overlaps the math of the
local tiles instead of running as a separate NCCL all-gather.  All waits are bounded.  A shard must not be
rewritten before every rank's GEMM of that epoch has run: callers alternate two instances (a rank can reach the
same instance again only after its peers published the next epoch, i.e. finished this one).

Reference: the reference all-gathers the sequence-parallel residual with NCCL before its column-parallel GEMMs
(code/fork/overlay/patch_mhc_sp.py:14-26; FP8 variant code/fork/fp8_w8a8.py:1171-1205).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import kernels as K


class AGGemm:
    def __init__(self, rows: int, K_dim: int, device, group=None):
        self.rows, self.K = rows, K_dim
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        W = self.world
        data = rows * K_dim * 2
        total = data + 256
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
        self.shard = self.buf[:data].view(torch.bfloat16).view(rows, K_dim)     # this rank's rows (write here)
        self.flags = self.buf[data:data + 4 * W].view(torch.int32)              # flag [j]: shard j published
        self.ptrs = torch.tensor(ptrs, dtype=torch.int64)                        # host: shard base of each rank
        self.ptrs_dev = self.ptrs.to(dev)
        # local staging of the peers' rows (each remote row block crosses NVLink once per epoch) and its flags
        self.stage = torch.empty(W * rows, K_dim, dtype=torch.bfloat16, device=dev)
        self.ready = torch.zeros((W * rows + 127) // 128, dtype=torch.int32, device=dev)
        self.flag_addrs = torch.tensor([p + data for p in ptrs], dtype=torch.int64, device=dev)
        self.epoch = 0
        torch.cuda.synchronize()
        if W > 1:
            dist.barrier(group)

    def publish(self) -> None:
        """Call after this rank's rows are in `shard` (stream order)."""
        K.C().signal_peers(self.flag_addrs, self.rank)
        self.epoch += 1

    def gemm(self, w: torch.Tensor, s: torch.Tensor, y: torch.Tensor, mode: int = K.GEMV_BF16) -> torch.Tensor:
        """y [W * rows, N] = all rows of every rank's shard @ (w8 * s)^T (waits for the shards of this epoch)."""
        K.C().gemm_ag_w8a16(self.ptrs, self.ptrs_dev, self.rank, self.rows, self.K, self.K, w, s, y, mode,
                            K._w_scratch(w.numel(), y.device), self.flags, self.epoch, self.stage, self.ready)
        return y
