"""Multi-process tests on CPU (gloo, world size 2): the baseline collectives the runtime uses, tensor-parallel
sharding of the tiny proxy (the rank partials of each row-parallel block add up to the unsharded block), and
host-side failure detection (a rank that fails or never arrives surfaces as an error on its peer within the
process-group timeout instead of hanging)."""

import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(fn, world, *args, timeout=120):
    port = _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, q, args)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, ok, payload = q.get(timeout=timeout)
        results[r] = (ok, payload)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


def _entry(fn, rank, world, port, q, args):
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    try:
        out = fn(rank, world, *args)
        q.put((rank, True, out))
    except Exception:
        q.put((rank, False, traceback.format_exc()))


def _collectives(rank, world):
    import torch.distributed as dist
    from glm53.parallel import dist as D
    D.init(backend="gloo", timeout_s=30)
    comm = D.NcclComm()
    t = torch.full((4,), float(rank + 1))
    comm.all_reduce(t)
    out = torch.empty(world * 2)
    comm.all_gather(out, torch.tensor([rank * 10.0, rank * 10.0 + 1]))
    m = comm.max_scalar(float(rank) * 3.5)
    dist.destroy_process_group()
    return t.tolist(), out.tolist(), m


def test_gloo_collectives():
    res = _run(_collectives, 2)
    for r in (0, 1):
        ok, (t, g, m) = res[r]
        assert ok
        assert t == [3.0] * 4 and g == [0.0, 1.0, 10.0, 11.0] and m == 3.5


def _sharded_blocks(rank, world):
    """Each rank computes its partial of the row-parallel blocks of the tiny proxy on the same input; the sum over
    ranks (all-reduce) must match the unsharded block."""
    import torch.distributed as dist
    import glm53
    from glm53.models import weights as W
    from glm53.models import reference as Rf
    from glm53.parallel import dist as D
    D.init(backend="gloo", timeout_s=60)
    cfg = glm53.tiny_config()
    ck = W.random_checkpoint(cfg, seed=0)
    full = W.prepare(W.DictSource(ck), cfg)
    part = W.prepare(W.DictSource(ck), cfg, rank=rank, world=world)
    torch.manual_seed(0)
    x = torch.randn(cfg.hidden).to(torch.bfloat16).float()
    errs = {}
    # dense MLP (layer 0) and shared expert (layer 1): column-parallel gate/up, row-parallel down
    for name, fm, pm in (("mlp", full.layers[0].mlp, part.layers[0].mlp),
                         ("shared", full.layers[1].moe.shared, part.layers[1].moe.shared)):
        y = Rf.mlp_block(pm, cfg, x)
        dist.all_reduce(y)
        ref = Rf.mlp_block(fm, cfg, x)
        errs[name] = float((y - ref).abs().max() / ref.abs().max())
    # routed experts: gate/up split by output columns, down by input rows (EXL3 whole 128-blocks)
    lf, lp = full.layers[1], part.layers[1]
    y = Rf.moe_block(lp, cfg, x) - Rf.mlp_block(lp.moe.shared, cfg, x)
    dist.all_reduce(y)
    ref = Rf.moe_block(lf, cfg, x) - Rf.mlp_block(lf.moe.shared, cfg, x)
    errs["experts"] = float((y - ref).abs().max() / ref.abs().max())
    dist.destroy_process_group()
    return errs


def test_tensor_parallel_partials_sum_to_full():
    res = _run(_sharded_blocks, 2, timeout=300)
    for r in (0, 1):
        ok, errs = res[r]
        assert ok, errs
        # row-parallel weights are slices of the unsharded fp8 weights: only the fp32 summation order differs
        assert errs["mlp"] < 1e-4 and errs["shared"] < 1e-4, errs
        assert errs["experts"] < 1e-3, errs


def _failing_peer(rank, world):
    import torch.distributed as dist
    from glm53.parallel import dist as D
    D.init(backend="gloo", timeout_s=5)
    if rank == 1:
        raise RuntimeError("injected failure on rank 1 before the collective")
    t = torch.ones(2)
    try:
        dist.all_reduce(t)
        return "no error"
    except Exception as e:                            # the peer never arrives: the collective times out
        return f"detected: {type(e).__name__}"


def test_peer_failure_is_detected_on_host():
    res = _run(_failing_peer, 2, timeout=120)
    assert res[1][0] is False and "injected failure" in res[1][1]
    ok, msg = res[0]
    assert ok and msg.startswith("detected"), msg
