"""Process-group bootstrap and the NCCL baseline collectives.

One process per GPU; ``init()`` reads RANK / LOCAL_RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT (torchrun's
environment), binds the rank to ``cuda:LOCAL_RANK`` and creates the NCCL group (gloo on CPU) with a short timeout,
so ranks that wait for a peer that is gone end with an error instead of hanging.

``NcclComm`` is the baseline communicator the runtime uses for the tensor-parallel partial sums (all-reduce of the
fp32 block outputs) and the vocabulary-parallel argmax (all-gather of per-rank (value, id) pairs).  The reference
uses vLLM's PyNccl all-reduce for the same call sites (code/fork/docs/DEC_AR1SHOT.md:10-12).
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def env_world() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def init(backend: str | None = None, timeout_s: float = 120.0):
    """Initialise torch.distributed when WORLD_SIZE > 1; returns (rank, local_rank, world)."""
    rank, local, world = env_world()
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, local, world


class NcclComm:
    """Baseline collectives over the default process group."""

    def __init__(self, group=None, fused: bool | None = None):
        self.group = group
        # decode windows reduce the tensor-parallel partials inside the kernels (parallel/fused.py) unless disabled
        self.fused = (os.environ.get("GLM53_FUSED_TP", "1") == "1") if fused is None else fused
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def all_gather(self, out: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        """out [world * n] <- every rank's t [n] in rank order."""
        if self.world > 1:
            dist.all_gather_into_tensor(out, t, group=self.group)
        else:
            out.copy_(t)
        return out

    def reduce_scatter(self, out: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        """out [n / world, ...] <- rank's block of the elementwise sum over ranks of t [n, ...] (rows in rank
        order)."""
        if self.world > 1:
            dist.reduce_scatter_tensor(out, t, group=self.group)
        else:
            out.copy_(t)
        return out

    def max_scalar(self, x: float) -> float:
        if self.world == 1:
            return x
        dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())

    def barrier(self):
        if self.world > 1:
            dist.barrier(group=self.group)
