"""Tensor parallelism on 2, 4 and 8 GPUs (each world size skipped with fewer GPUs): the fused reduction (partials pushed to the peers from the
projection's epilogue -- GEMV for decode windows, tcgen05 GEMM for prefill chunks -- and summed in rank order
inside the next mHC kernel) gives the same logits as the NCCL all-reduce path, for a prefill chunk and for decode
windows (GPU only)."""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from glm53.config import tiny_config
    from glm53.models import weights as W
    from glm53.models.runtime import Runtime, RuntimeConfig
    from glm53.models.session import Sequence
    from glm53.parallel import dist as D
    D.init(timeout_s=60)
    try:
        cfg = tiny_config()
        dev = torch.device("cuda", rank)
        w = W.prepare(W.RandomSource(cfg, seed=0, device=dev), cfg, rank=rank, world=world, device=dev)
        rc = RuntimeConfig(max_rows=128, max_seqs=1, kv_slots=64 * 8, block_size=64, max_blocks=8)
        g = torch.Generator().manual_seed(3)
        prompt = torch.randint(16, cfg.vocab, (200,), generator=g).tolist()
        outs = []
        for fused in (False, True):
            rt = Runtime(w, rc, comm=D.NcclComm(fused=fused))
            seq = Sequence(rt)
            lg = [seq.prefill(prompt, chunk=128).clone()]          # chunks of 128 and 72 rows (tcgen05 GEMMs)
            toks = [1, 2, 3, 4, 5, 6, 7, 8]
            seq.stage(toks, list(range(8)))
            lg.append(rt.forward(8, keep_window=True).clone())    # a decode window (GEMV epilogue push)
            if rt.px is not None:
                rt.px.check()
            outs.append(torch.cat([x.flatten() for x in lg]))
        result[rank] = (outs[0] - outs[1]).abs().max().item()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_tp_matches_nccl(world):
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    result = mp.Manager().dict()
    mp.spawn(_worker, args=(world, 29541 + world, result), nprocs=world, join=True)
    assert len(result) == world
    if world == 2:
        # two ranks: a + b is the same fp32 sum in either order, so the paths agree bit for bit
        assert max(result.values()) == 0.0, dict(result)
    else:
        # more ranks: the fused path sums in rank order, NCCL in its ring order -- fp32 rounding only
        assert max(result.values()) < 5e-2, dict(result)


def _push_worker(rank, world, port, result):
    """Row-parallel decode projection with the fused push (bulk-copy GEMV for these sizes): every rank's fp32
    partial must land in its slot of every rank's receive buffer and the arrival flags must count one launch."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from glm53.models.weights import quantize_fp8_rows
    from glm53.ops import kernels as Kk
    from glm53.parallel import dist as D
    from glm53.parallel.fused import PeerExchange
    D.init(timeout_s=60)
    try:
        dev = torch.device("cuda", rank)
        errs = []
        for N, K in ((4096, 2048), (4096, 4096)):
            rows = 8
            px = PeerExchange(rows, N, dev)
            g = torch.Generator(device=dev).manual_seed(11)
            x = torch.randn(rows, K, device=dev, generator=g).to(torch.bfloat16)
            ws = [quantize_fp8_rows(torch.randn(N, K, device=dev, generator=torch.Generator(device=dev).manual_seed(
                100 + j)) / K ** 0.5) for j in range(world)]
            y = torch.empty(rows, N, device=dev)
            Kk.C().gemv_push(x, ws[rank].w, ws[rank].s, y, Kk.GEMV_F32, px.push_ptrs[0], px.push_flags[0],
                             px.done_prod[0:1], px.slot, rank, world, px.err)
            torch.cuda.synchronize()
            dist.barrier()
            for j in range(world):
                ref = torch.empty(rows, N, device=dev)
                Kk.C().gemv(x, ws[j].w, ws[j].s, ref, Kk.GEMV_F32, 0.0)
                got = px.gath[0][j * px.slot:(j + 1) * px.slot].view(rows, N)
                errs.append((got - ref).abs().max().item())
            errs.append(float((px.flags[0] != 1).sum().item()))
            px.check()
            dist.barrier()
        result[rank] = max(errs)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gemv_push_bulk(world):
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    result = mp.Manager().dict()
    mp.spawn(_push_worker, args=(world, 29557 + world, result), nprocs=world, join=True)
    assert len(result) == world
    assert max(result.values()) == 0.0, dict(result)


def _sp_worker(rank, world, port, result):
    """Sequence-parallel prefill (mHC on each rank's rows, all-gather before and reduce-scatter after each block),
    also with the MLA blocks row-parallel over all heads, against the all-reduce path: logits of the prefill chunks
    and of a decode window after them."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0", GLM53_SP_MIN_ROWS="64",
                      GLM53_PREFILL_W8A8="none")       # exact W8A16 projections: the paths differ by fp32 order only
    import torch.distributed as dist
    from glm53.config import tiny_config
    from glm53.models import weights as W
    from glm53.models.runtime import Runtime, RuntimeConfig
    from glm53.models.session import Sequence
    from glm53.parallel import dist as D
    D.init(timeout_s=60)
    try:
        cfg = tiny_config()
        dev = torch.device("cuda", rank)
        w = W.prepare(W.RandomSource(cfg, seed=0, device=dev), cfg, rank=rank, world=world, device=dev)
        w_rows = W.prepare(W.RandomSource(cfg, seed=0, device=dev), cfg, rank=rank, world=world, device=dev,
                           sp_mla=True)
        rc = RuntimeConfig(max_rows=128, max_seqs=1, kv_slots=64 * 8, block_size=64, max_blocks=8)
        g = torch.Generator().manual_seed(5)
        prompt = torch.randint(16, cfg.vocab, (256,), generator=g).tolist()
        outs = []
        # all-reduce path; sequence parallel; sequence parallel with the row-parallel (all-head) MLA blocks
        for sp, wts in (("0", w), ("1", w), ("1", w_rows)):
            os.environ["GLM53_SP"] = sp
            rt = Runtime(wts, rc, comm=D.NcclComm(fused=False))
            seq = Sequence(rt)
            lg = [seq.prefill(prompt, chunk=128).clone()]          # two 128-row chunks
            lg.append(rt.hidden[:128].float().clone())
            toks = [1, 2, 3, 4, 5, 6, 7, 8]
            seq.stage(toks, list(range(8)))
            lg.append(rt.forward(8, keep_window=True).clone())
            outs.append(torch.cat([x.flatten() for x in lg]))
        result[rank] = ((outs[0] - outs[1]).abs().max().item(), (outs[0] - outs[2]).abs().max().item())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sequence_parallel_prefill_matches_allreduce(world):
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    result = mp.Manager().dict()
    mp.spawn(_sp_worker, args=(world, 29571 + world, result), nprocs=world, join=True)
    assert len(result) == world
    # reduce-scatter + all-gather instead of the all-reduce, and all heads of a row in one projection instead of
    # per-rank head groups summed: fp32 summation order only
    assert max(v[0] for v in result.values()) < 5e-2, ("sequence parallel", dict(result))
    assert max(v[1] for v in result.values()) < 5e-2, ("row-parallel MLA", dict(result))


def _sp_fp8_worker(rank, world, port, result):
    """Sequence-parallel prefill with W8A8 on the KDA input projection: all-gathering the rows as e4m3 codes and
    row scales against all-gathering bf16 rows and quantising after the gather.  Per-row quantisation is row-local,
    so the two must agree bit for bit (and the all-reduce path is the W8A8 reference)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0", GLM53_SP_MIN_ROWS="64",
                      GLM53_PREFILL_W8A8="kda_in_proj")
    import torch.distributed as dist
    from glm53.config import tiny_config
    from glm53.models import weights as W
    from glm53.models.runtime import Runtime, RuntimeConfig
    from glm53.models.session import Sequence
    from glm53.parallel import dist as D
    D.init(timeout_s=60)
    try:
        cfg = tiny_config()
        dev = torch.device("cuda", rank)
        w = W.prepare(W.RandomSource(cfg, seed=0, device=dev), cfg, rank=rank, world=world, device=dev)
        rc = RuntimeConfig(max_rows=128, max_seqs=1, kv_slots=64 * 8, block_size=64, max_blocks=8)
        g = torch.Generator().manual_seed(6)
        prompt = torch.randint(16, cfg.vocab, (256,), generator=g).tolist()
        outs, used = [], []
        for fp8ag in ("0", "1"):
            os.environ["GLM53_SP"] = "1"
            os.environ["GLM53_SP_FP8AG"] = fp8ag
            rt = Runtime(w, rc, comm=D.NcclComm(fused=False))
            seq = Sequence(rt)
            lg = [seq.prefill(prompt, chunk=128).clone(), rt.hidden[:128].float().clone()]
            used.append(rt._sp is not None and rt._sp_fp8(128))     # the last chunk ran sequence parallel
            outs.append(torch.cat([x.flatten() for x in lg]))
        result[rank] = ((outs[0] - outs[1]).abs().max().item(), used[1], rt.q_rows is not None)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sequence_parallel_fp8_allgather_bit_exact(world):
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    result = mp.Manager().dict()
    mp.spawn(_sp_fp8_worker, args=(world, 29591 + world, result), nprocs=world, join=True)
    assert len(result) == world
    assert all(v[1] and v[2] for v in result.values()), ("the e4m3 all-gather path was not taken", dict(result))
    assert max(v[0] for v in result.values()) == 0.0, dict(result)


def _ep_worker(rank, world, port, result):
    """The model with its routed experts expert-parallel (weights sharded by expert, rows of each layer split over
    the ranks, dispatch and combine through the peers' buffers) against the tensor-parallel model: logits of a
    prefill chunk and of two decode windows (one captured as a CUDA graph and replayed)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from glm53.config import tiny_config
    from glm53.models import weights as W
    from glm53.models.runtime import Graphed, Runtime, RuntimeConfig
    from glm53.models.session import Sequence
    from glm53.parallel import dist as D
    D.init(timeout_s=60)
    try:
        cfg = tiny_config()
        dev = torch.device("cuda", rank)
        rc = RuntimeConfig(max_rows=128, max_seqs=1, kv_slots=64 * 8, block_size=64, max_blocks=8)
        g = torch.Generator().manual_seed(9)
        prompt = torch.randint(16, cfg.vocab, (160,), generator=g).tolist()
        outs = []
        for ep in (False, True):
            w = W.prepare(W.RandomSource(cfg, seed=0, device=dev), cfg, rank=rank, world=world, device=dev, ep=ep)
            rt = Runtime(w, rc, comm=D.NcclComm())
            assert (rt.ep is not None) == ep
            seq = Sequence(rt)
            lg = [seq.prefill(prompt, chunk=128).clone()]
            toks = [3, 1, 4, 1, 5, 9, 2, 6]
            seq.stage(toks, list(range(8)))
            lg.append(rt.forward(8, keep_window=True).clone())
            graph = Graphed(lambda: rt.forward(8, keep_window=True))
            graph()
            lg.append(graph().clone())
            if rt.px is not None:
                rt.px.check()
            if rt.ep is not None:
                rt.ep_bufs.x_ex.check()
            outs.append(torch.cat([x.flatten() for x in lg]))
            del rt, w
        result[rank] = (outs[0] - outs[1]).abs().max().item()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_expert_parallel_model_matches_tensor_parallel(world):
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    result = mp.Manager().dict()
    mp.spawn(_ep_worker, args=(world, 29591 + world, result), nprocs=world, join=True)
    assert len(result) == world
    # full-width experts on the owner vs width-sharded experts summed over ranks: fp32 summation order only
    assert max(result.values()) < 5e-2, dict(result)
