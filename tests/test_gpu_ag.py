"""All-gather + GEMM with the gather inside the tcgen05 GEMM (TMA loads of peer shards): one GPU (world 1) and two
GPUs (skipped with fewer) against an fp32 reference of the gathered matrix product (GPU only)."""

import math
import os

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run(rank, world, steps=3):
    from glm53.models.weights import quantize_fp8_rows
    from glm53.parallel.ag_gemm import AGGemm
    rows, K, N = 256, 512, 384
    bufs = [AGGemm(rows, K, DEV), AGGemm(rows, K, DEV)]     # two parities: a shard is rewritten two steps later
    w = quantize_fp8_rows(torch.randn(N, K, generator=torch.Generator().manual_seed(5)) / math.sqrt(K))
    wd, sd = w.w.to(DEV), w.s.to(DEV)
    worst = 0.0
    for step in range(steps):
        ag = bufs[step % 2]
        g = torch.Generator(device=DEV).manual_seed(1000 * step + rank)
        mine = torch.randn(rows, K, generator=g, device=DEV).to(torch.bfloat16)
        ag.shard.copy_(mine)
        ag.publish()
        y = torch.zeros(world * rows, N, device=DEV)
        ag.gemm(wd, sd, y, 1)                                   # GEMV_F32 (staged peer rows)
        # reference: every rank's rows regenerated from the seeds
        allrows = torch.cat([torch.randn(rows, K, generator=torch.Generator(device=DEV).manual_seed(1000 * step + j),
                                         device=DEV).to(torch.bfloat16) for j in range(world)])
        ref = allrows.float() @ w.dequant().to(DEV).t()
        torch.cuda.synchronize()
        worst = max(worst, ((y - ref).abs().max() / ref.abs().max()).item())
    return worst


def test_ag_gemm_world1():
    assert _run(0, 1) < 2e-3


def _worker(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from glm53.parallel import dist as D
    D.init(timeout_s=60)
    try:
        result[rank] = _run(rank, world)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ag_gemm_two_gpus():
    import torch.multiprocessing as mp
    result = mp.Manager().dict()
    mp.spawn(_worker, args=(2, 29551, result), nprocs=2, join=True)
    assert len(result) == 2 and max(result.values()) < 2e-3, dict(result)
