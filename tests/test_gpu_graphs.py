"""CUDA-graph replay of a decode verify window and of the block drafter (tiny proxy): replays do no implicit host
synchronisation (torch sync debug mode "error"), allocate nothing, and read the inputs staged before each replay."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_verify_and_draft_graphs_replay_without_sync_or_allocation():
    import glm53
    from glm53.models import weights as W
    from glm53.models.drafter import BlockDrafter
    from glm53.models.runtime import Graphed, Runtime, RuntimeConfig
    from glm53.models.session import Sequence
    cfg = glm53.tiny_config()
    dev = torch.device("cuda", 0)
    w = W.prepare(W.RandomSource(cfg, seed=0, device=dev), cfg, device=dev)
    rt = Runtime(w, RuntimeConfig(max_rows=64, kv_slots=64 * 8, block_size=64, max_blocks=8))
    seq = Sequence(rt)
    g = torch.Generator().manual_seed(1)
    seq.prefill(torch.randint(16, cfg.vocab, (100,), generator=g).tolist(), chunk=64)
    R = 8
    toks_a = torch.randint(16, cfg.vocab, (R,), generator=g).tolist()
    toks_b = torch.randint(16, cfg.vocab, (R,), generator=g).tolist()
    seq.stage(toks_a, list(range(R)))
    graph = Graphed(lambda: rt.forward(R, keep_window=True))
    drafter = BlockDrafter(cfg, w, device=dev)
    hid = [rt.hidden[0].clone(), (rt.hidden[0].float() * 0.5).to(rt.hidden.dtype)]   # drafter inputs per key
    drafter.stage(5, hid[0])
    dgraph = Graphed(lambda: drafter.run(7))
    torch.cuda.synchronize()
    outs = {}
    base_mem = None
    for i in range(20):
        toks = toks_a if i % 2 == 0 else toks_b
        seq.stage(toks, list(range(R)))                   # host staging outside the checked region
        drafter.stage(toks[0], hid[i % 2])
        torch.cuda.synchronize()
        if base_mem is None:
            base_mem = torch.cuda.memory_allocated()
        torch.cuda.set_sync_debug_mode("error")
        try:
            lg = graph()
            dl = dgraph()
        finally:
            torch.cuda.set_sync_debug_mode(0)
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == base_mem
        key = i % 2
        snap = (lg.float().sum().item(), dl.float().sum().item())
        if key in outs:
            assert outs[key] == snap                       # the same inputs replay to the same bits
        outs[key] = snap
    assert outs[0][0] != outs[1][0] and outs[0][1] != outs[1][1]   # the staged inputs reach both graphs
