"""Tensor-parallel serving control plane on CPU (gloo, world size 2): rank 0 publishes each step's new requests and
aborts, the follower applies them in the same order and steps, and both ranks' engines emit the same tokens (greedy,
seeded and unseeded sampled requests; an unseeded request's noise key is the same in both processes), reject the
same over-long request, abort the same request, and stop together. The server aborts a request whose answer hit a
stop string."""

import time

import pytest

from test_dist_cpu import _run


def _plane(rank, world, transport):
    import torch.distributed as dist
    from glm53.api.server import ControlPlane
    from glm53.engine.llm import EngineConfig, LLMEngine, SamplingParams
    from glm53.parallel import dist as D
    from tests.fake_backend import FakeBackend
    D.init(backend="gloo", timeout_s=30)
    group = dist.new_group(backend="gloo")
    eng = LLMEngine(FakeBackend(max_seqs=4, checkpoints=0),
                    EngineConfig(max_seqs=4, page_size=16, num_pages=128, max_model_len=256, prefill_chunk=32,
                                 cuda_graphs=False))
    plane = ControlPlane(eng, group, heartbeat_s=0.05, transport=transport)
    errors = []
    if rank == 0:
        first = [("a", list(range(20, 60)), SamplingParams(max_tokens=30)),
                 ("b", list(range(30, 50)), SamplingParams(max_tokens=40, temperature=3.0)),
                 ("c", list(range(40, 90)), SamplingParams(max_tokens=25, temperature=1.0, seed=5))]
        err, step = plane.lead(first)
        errors += err
        n = 0
        while step:
            eng.step()
            n += 1
            late = [("d", list(range(16, 36)), SamplingParams(max_tokens=12)),
                    ("long", list(range(300)), SamplingParams(max_tokens=8))] if n == 3 else []
            err, step = plane.lead(late, ["c"] if n == 5 else [])
            errors += err
        time.sleep(0.2)
        plane.lead()                                   # idle heartbeat
        plane.lead(stop=True)
    else:
        plane.follow()
    plane.close()
    out = {rid: (r.output, r.finish_reason) for rid, r in eng.done.items()}
    hist = {s: list(h) for s, h in eng.b.hist.items()}
    dist.destroy_process_group()
    return out, hist, errors


@pytest.mark.parametrize("transport", ["shm", "gloo"])
def test_control_plane_keeps_ranks_in_lockstep(transport):
    res = _run(_plane, 2, transport)
    (ok0, p0), (ok1, p1) = res[0], res[1]
    assert ok0, p0
    assert ok1, p1
    out0, hist0, err0 = p0
    out1, hist1, _ = p1
    assert out0 == out1 and hist0 == hist1
    assert set(out0) == {"a", "b", "c", "d"}
    assert out0["c"][1] == "abort" and out0["a"][1] == "length" and len(out0["b"][0]) == 40
    assert [rid for rid, _ in err0] == ["long"]


def test_stop_string_aborts_the_engine_request():
    from fastapi.testclient import TestClient
    from glm53.api.server import build_app
    from glm53.engine.tokenizer import ByteTokenizer
    from tests.fake_backend import reference_greedy
    from test_api import FakeLLM
    llm = FakeLLM()
    tok = ByteTokenizer(512)
    prompt = list(range(20, 60))
    text = tok.decode(reference_greedy(prompt, 200))
    stop = next(text[i:i + 2] for i in range(4, len(text) - 2) if text[i:i + 2].strip() and text[i:i + 2] not in
                text[:i + 1])
    with TestClient(build_app(llm, "glm-test", reasoning=False)) as c:
        body = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 200, "stop": [stop]}).json()
        assert body["choices"][0]["finish_reason"] == "stop"
        t0 = time.time()
        while llm.engine.running and time.time() - t0 < 5:
            time.sleep(0.02)
        assert not llm.engine.running
        done = list(llm.engine.done.values())
        assert done and done[-1].finish_reason == "abort" and len(done[-1].output) < 200


def _lost_peer(rank, world, who_leaves):
    import datetime

    import torch.distributed as dist
    from glm53.api.server import ControlPlane
    from glm53.engine.llm import EngineConfig, LLMEngine, SamplingParams
    from glm53.parallel import dist as D
    from tests.fake_backend import FakeBackend
    D.init(backend="gloo", timeout_s=30)
    group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=3))
    eng = LLMEngine(FakeBackend(max_seqs=2, checkpoints=0),
                    EngineConfig(max_seqs=2, page_size=16, num_pages=32, max_model_len=128, prefill_chunk=32,
                                 cuda_graphs=False))
    plane = ControlPlane(eng, group, heartbeat_s=0.05, timeout_s=3)
    if rank == 0:
        plane.lead([("a", list(range(20, 40)), SamplingParams(max_tokens=4))])
        if who_leaves == 0:
            return "left"                              # the leader goes away between steps
        t0 = time.time()
        try:
            for _ in range(100):
                plane.lead()
                time.sleep(0.05)
        except Exception as e:
            return ("error", type(e).__name__, time.time() - t0)
        return ("no error", None, time.time() - t0)
    plane._bcast(None)                                 # the first plan
    if who_leaves == 1:
        return "left"                                  # the follower goes away between steps
    t0 = time.time()
    try:
        plane.follow()
    except Exception as e:
        return ("error", type(e).__name__, time.time() - t0)
    return ("no error", None, time.time() - t0)


def test_follower_ends_when_the_leader_is_gone():
    res = _run(_lost_peer, 2, 0, timeout=60)
    ok, payload = res[1]
    assert ok, payload
    assert payload[0] == "error" and payload[2] < 20, payload


def test_leader_ends_when_a_follower_is_gone():
    res = _run(_lost_peer, 2, 1, timeout=60)
    ok, payload = res[0]
    assert ok, payload
    assert payload[0] == "error" and payload[2] < 20, payload


def _big_and_many(rank, world):
    import torch.distributed as dist
    from glm53.parallel import dist as D
    from glm53.parallel.control import ShmChannel
    D.init(backend="gloo", timeout_s=30)
    group = dist.new_group(backend="gloo")
    ch = ShmChannel(group, timeout_s=10, capacity=1 << 12)
    msgs = [{"i": i, "blob": list(range(i * 300))} for i in range(40)]       # up to ~40 KB: many parts
    got = []
    for m in msgs:
        if rank == 0:
            ch.publish(m)
        else:
            got.append(ch.receive())
    ch.close()
    dist.destroy_process_group()
    return got == msgs if rank else True


def test_shm_channel_multi_part_messages_arrive_in_order():
    res = _run(_big_and_many, 3)
    assert all(ok and payload for ok, payload in res.values()), res


def _loop_and_follower(rank, world):
    import asyncio

    import torch.distributed as dist
    from glm53.api.server import ControlPlane, EngineLoop
    from glm53.engine.llm import EngineConfig, LLMEngine, SamplingParams
    from glm53.parallel import dist as D
    from tests.fake_backend import FakeBackend

    class L:
        engine = LLMEngine(FakeBackend(max_seqs=4, checkpoints=0),
                           EngineConfig(max_seqs=4, page_size=16, num_pages=128, max_model_len=256,
                                        prefill_chunk=32, cuda_graphs=False))
    D.init(backend="gloo", timeout_s=30)
    group = dist.new_group(backend="gloo")
    if rank != 0:
        ControlPlane(L.engine, group, timeout_s=20).follow()
    else:
        el = EngineLoop(L, group)

        async def one(prompt, params):
            q = asyncio.Queue()
            rid = el.submit(prompt, params, asyncio.get_running_loop(), q)
            toks = []
            while True:
                item = await q.get()
                toks += item.get("tokens", [])
                if item.get("finished"):
                    return rid, toks

        async def many():
            return await asyncio.gather(
                one(list(range(20, 60)), SamplingParams(max_tokens=20)),
                one(list(range(25, 45)), SamplingParams(max_tokens=30, temperature=2.0)),
                one(list(range(30, 90)), SamplingParams(max_tokens=15, temperature=2.0, seed=9)))
        got = asyncio.run(many())
        time.sleep(1.5)                                # idle: heartbeats keep the follower waiting
        el.close()
        assert [len(t) for _, t in got] == [20, 30, 15]
    out = {rid: r.output for rid, r in L.engine.done.items()}
    dist.destroy_process_group()
    return out


def test_engine_loop_drives_a_follower_rank():
    res = _run(_loop_and_follower, 2, timeout=90)
    (ok0, out0), (ok1, out1) = res[0], res[1]
    assert ok0, out0
    assert ok1, out1
    assert out0 == out1 and len(out0) == 3
