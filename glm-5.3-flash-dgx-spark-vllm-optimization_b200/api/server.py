"""OpenAI-compatible HTTP server.

  GET  /health                 200 when the engine loop is alive
  GET  /v1/models              the served model
  POST /v1/completions         prompt (string or token ids), max_tokens, temperature, top_p, top_k, seed, stop,
                               stream (server-sent events)
  POST /v1/chat/completions    messages (chat template of the byte tokenizer), same sampling fields, stream;
                               reasoning_effort (placed before the first user turn); the answer is split into
                               reasoning_content (<think> ... </think>) and content, and tool calls are parsed
                               into message.tool_calls (api/parsers.py)
  POST /v1/responses           Responses API: input (string or items; unknown item types skipped), instructions,
                               max_output_tokens; output items reasoning / message / function_call
  POST /tokenize, /detokenize  token ids of a prompt or of chat messages; text of token ids
  GET  /metrics                Prometheus text: requests running / waiting, prompt / generation tokens, speculative
                               drafts / accepted tokens, prefix-cache hits / queries, finished requests

One engine thread owns the GPU and steps the engine whenever requests are pending; HTTP handlers hand requests to
it through a queue and receive tokens through per-request queues. A request whose answer hits a stop string, or
whose client goes away, is aborted in the engine so its slot and pages are freed. The reference serves the same API
through vLLM (code/kit/launcher/start.sh:2666-2684; Responses-input robustness: code/vllm-patches/responses_utils.patch).

Tensor parallel (one process per GPU under torchrun): every rank loads its shard and runs the same engine; rank 0
serves HTTP and, before each engine step, broadcasts that step's new requests and aborts over a CPU (gloo) group
(``ControlPlane``); the other ranks apply them in the same order and step, so the schedulers stay in lockstep and
every step's collectives line up (the reference's head serves and its workers run headless:
code/kit/launcher/start.sh:2741, :2821).

  python -m glm53.api.server --model tiny --port 8000
  torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m glm53.api.server --model full --port 8000
"""

from __future__ import annotations

import argparse
import asyncio
import json
import queue
import threading
import time
import uuid

from ..engine.llm import SamplingParams
from . import parsers

try:  # the HTTP stack is optional for offline use
    from fastapi import Depends, FastAPI, HTTPException, Request
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse
except ImportError:  # pragma: no cover
    FastAPI = None


class ControlPlane:
    """Keeps the engines of all tensor-parallel ranks in lockstep. Rank 0 calls ``lead`` once per loop turn with the
    requests and aborts that arrived since the last one; a non-empty plan (or, while idle, an empty heartbeat every
    ``heartbeat_s`` so the followers' waits stay inside ``timeout_s``) goes to every rank (``parallel/control.py``:
    shared memory on one node, or the CPU group) and is applied on every rank in the same order. Ranks > 0 run
    ``follow`` until rank 0 sends stop. With no group (one rank) nothing is sent."""

    def __init__(self, engine, group=None, heartbeat_s: float = 1.0, timeout_s: float = 60.0,
                 transport: str = "shm"):
        self.engine = engine
        self.heartbeat_s = heartbeat_s
        self.world, self.rank, self.chan = 1, 0, None
        if group is not None:
            import torch.distributed as dist
            from ..parallel.control import GlooChannel, ShmChannel
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
            if self.world > 1:
                self.chan = ShmChannel(group, timeout_s) if transport == "shm" else GlooChannel(group)
        self._last = time.monotonic()

    def _bcast(self, plan):
        if self.chan is None:
            return plan
        if self.rank == 0:
            self.chan.publish(plan)
            return plan
        return self.chan.receive()

    def close(self) -> None:
        if self.chan is not None:
            self.chan.close()
            self.chan = None

    def _apply(self, plan) -> list[tuple[str, str]]:
        errors = []
        for rid, ids, params in plan["add"]:
            try:
                self.engine.add_request(ids, params, rid=rid)
            except ValueError as e:                  # raised alike on every rank
                errors.append((rid, str(e)))
        for rid in plan["abort"]:
            self.engine.abort(rid)
        return errors

    def lead(self, adds=(), aborts=(), stop: bool = False) -> tuple[list[tuple[str, str]], bool]:
        """Rank 0: publish and apply one plan. Returns (rejected requests with their errors, whether to step)."""
        if not adds and not aborts and not stop and not self.engine.has_work():
            if self.world == 1 or time.monotonic() - self._last < self.heartbeat_s:
                return [], False
        plan = self._bcast({"add": list(adds), "abort": list(aborts), "stop": stop})
        self._last = time.monotonic()
        errors = self._apply(plan)
        return errors, (not stop and self.engine.has_work())

    def follow(self) -> None:
        """Ranks > 0: apply rank 0's plans and step whenever there is work, until rank 0 sends stop."""
        try:
            while True:
                plan = self._bcast(None)
                if plan["stop"]:
                    return
                self._apply(plan)
                if self.engine.has_work():
                    self.engine.step()
        finally:
            self.close()


class EngineLoop:
    """Runs ``engine.step()`` on its own thread; thread-safe submission, aborts and per-request token streams."""

    def __init__(self, llm, group=None):
        self.llm = llm
        self.engine = llm.engine
        self.plane = ControlPlane(self.engine, group)
        self.inbox: queue.Queue = queue.Queue()
        self.aborts: queue.Queue = queue.Queue()
        self.streams: dict[str, tuple[asyncio.AbstractEventLoop, asyncio.Queue]] = {}
        self.alive = True
        self.error: str | None = None
        self._stop = False
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def submit(self, prompt_ids, params: SamplingParams, loop, q) -> str:
        rid = f"cmpl-{uuid.uuid4().hex[:16]}"
        self.streams[rid] = (loop, q)
        self.inbox.put((rid, prompt_ids, params))
        return rid

    def abort(self, rid: str) -> None:
        self.streams.pop(rid, None)
        self.aborts.put(rid)

    def close(self) -> None:
        """Stop the loop (and the follower ranks) after the current step."""
        self._stop = True
        self.thread.join(timeout=30)

    def _drain(self, q: queue.Queue, block: bool) -> list:
        items = []
        try:
            while True:
                items.append(q.get(block=block and not items, timeout=0.05))
        except queue.Empty:
            pass
        return items

    def _run(self):
        try:
            while self.alive and not self._stop:
                adds = self._drain(self.inbox, block=not self.engine.has_work())
                aborts = self._drain(self.aborts, block=False)
                errors, step = self.plane.lead(adds, aborts)
                for rid, msg in errors:
                    self._push(rid, {"error": msg, "finished": True})
                if not step:
                    continue
                outs = self.engine.step()
                for o in outs:
                    self._push(o.rid, {"tokens": o.new_tokens, "finished": o.finished, "reason": o.finish_reason,
                                       "logprobs": o.new_logprobs})
        except Exception as e:  # pragma: no cover - surfaced to clients and /health
            self.error = repr(e)
            for rid in list(self.streams):
                self._push(rid, {"error": self.error, "finished": True})
            raise
        finally:
            self.alive = False
            try:
                self.plane.lead(stop=True)           # release the follower ranks
            except Exception:  # pragma: no cover - a follower is gone; the others end on their timeout
                pass
            self.plane.close()

    def _push(self, rid, item):
        s = self.streams.get(rid)
        if s is None:
            return
        loop, q = s
        loop.call_soon_threadsafe(q.put_nowait, item)
        if item.get("finished"):
            self.streams.pop(rid, None)


def _params(body: dict, tok, chat: bool = False, engine=None) -> SamplingParams:
    """Sampling fields of a request. Log-probabilities: completions take ``logprobs: n`` (top-n alternatives); chat
    takes ``logprobs: true`` with ``top_logprobs: n``.  A field of the wrong type or out of range is a 400 here
    (``engine.check_params``), so it never reaches the engine thread."""
    try:
        stop_ids = tuple(int(t) for t in (body.get("stop_token_ids") or ()))
        if chat:
            lp = int(body.get("top_logprobs") or 0) if body.get("logprobs") else None
        else:
            lp = int(body["logprobs"]) if body.get("logprobs") is not None else None
        sp = SamplingParams(max_tokens=int(body.get("max_tokens") or 64),
                            temperature=float(body.get("temperature", 0.0)), top_p=float(body.get("top_p", 1.0)),
                            top_k=int(body.get("top_k", 0) or 0), seed=body.get("seed"), stop_token_ids=stop_ids,
                            ignore_eos=bool(body.get("ignore_eos", False)), logprobs=lp)
        if engine is not None:
            engine.check_params(sp)
    except (TypeError, ValueError) as e:
        raise _bad_request(str(e)) from e
    return sp


def _bad_request(detail: str):
    from fastapi import HTTPException
    return HTTPException(status_code=400, detail=detail)


def _stop_strings(body) -> list[str]:
    s = body.get("stop")
    if s is None:
        return []
    return [s] if isinstance(s, str) else list(s)


def build_app(llm, model_name: str = "glm-5.3-flash", api_key: str | None = None, reasoning: bool = True,
              group=None, max_n: int | None = None):
    """``api_key``: when set, /v1 routes need ``Authorization: Bearer <api_key>``.  ``reasoning``: split
    ``<think>`` reasoning from the answer and apply stop strings to the answer only. ``group``: the CPU process
    group of the tensor-parallel ranks (rank 0 serves; the others run ``ControlPlane.follow``).  ``max_n``: most
    choices one request may ask for (default: the engine's sequence slots), so one request cannot queue an
    unbounded number of engine requests."""
    if max_n is None:
        max_n = max(1, llm.engine.cfg.max_seqs)
    if FastAPI is None:
        raise RuntimeError("fastapi is not installed")

    async def auth(req: Request):
        if api_key and req.headers.get("authorization", "") != f"Bearer {api_key}":
            raise HTTPException(status_code=401, detail="invalid API key")

    app = FastAPI(dependencies=[Depends(auth)] if api_key else [])
    loop_holder = {"engine": EngineLoop(llm, group)}
    app.state.engine_loop = loop_holder["engine"]
    tok = llm.tokenizer

    @app.get("/health")
    async def health():
        el = loop_holder["engine"]
        if not el.alive:
            raise HTTPException(status_code=503, detail=el.error or "engine stopped")
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "glm53",
                                            "max_model_len": llm.engine.cfg.max_model_len}]}

    @app.get("/metrics")
    async def metrics():
        e = llm.engine
        m = e.metrics
        pc = e.kv.alloc.stats
        lines = [
            "# TYPE glm53_num_requests_running gauge", f"glm53_num_requests_running {len(e.running)}",
            "# TYPE glm53_num_requests_waiting gauge", f"glm53_num_requests_waiting {len(e.waiting)}",
            "# TYPE glm53_prompt_tokens_total counter", f"glm53_prompt_tokens_total {m['prompt_tokens']}",
            "# TYPE glm53_generation_tokens_total counter", f"glm53_generation_tokens_total {m['generation_tokens']}",
            "# TYPE glm53_spec_decode_num_drafts_total counter", f"glm53_spec_decode_num_drafts_total {m['spec_drafts']}",
            "# TYPE glm53_spec_decode_num_accepted_tokens_total counter",
            f"glm53_spec_decode_num_accepted_tokens_total {m['spec_accepted']}",
            "# TYPE glm53_spec_decode_num_windows_total counter",
            f"glm53_spec_decode_num_windows_total {m['spec_windows']}",
            "# TYPE glm53_spec_decode_num_accepted_tokens_per_pos counter",
            *[f'glm53_spec_decode_num_accepted_tokens_per_pos{{position="{i}"}} {c}'
              for i, c in enumerate(m["spec_accepted_per_pos"]) if i < 8],
            "# TYPE glm53_prefix_cache_hits_total counter", f"glm53_prefix_cache_hits_total {pc['hits']}",
            "# TYPE glm53_prefix_cache_queries_total counter", f"glm53_prefix_cache_queries_total {pc['queries']}",
            "# TYPE glm53_prefix_cached_tokens_total counter",
            f"glm53_prefix_cached_tokens_total {m['prefix_cached_tokens']}",
            "# TYPE glm53_request_success_total counter", f"glm53_request_success_total {m['requests_finished']}",
        ]
        return PlainTextResponse("\n".join(lines) + "\n")

    async def _run(prompt_ids, params, stops, chat: bool, stream: bool, body: dict, raw: bool = False):
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        rid = loop_holder["engine"].submit(prompt_ids, params, loop, q)
        created = int(time.time())
        obj = "chat.completion" if chat else "text_completion"

        async def events():
            engine_done = False
            try:
                async for ev in _events():
                    engine_done = ev.pop("engine_done")
                    yield ev
            finally:
                if not engine_done:
                    # a stop string ended the answer or the client went away: free the request's slot and pages
                    loop_holder["engine"].abort(rid)

        async def _events():
            text_so_far = ""
            toks, lps = [], []
            while True:
                item = await q.get()
                if "error" in item:
                    yield {"error": item["error"], "engine_done": True}
                    return
                engine_finished = bool(item["finished"])
                toks += item["tokens"]
                lps += item.get("logprobs") or []
                text = tok.decode(toks)
                delta = text[len(text_so_far):]
                reason = item.get("reason")
                k = parsers.stop_index(text, stops, reasoning)
                if k >= 0:
                    delta = text[len(text_so_far):k]
                    text = text[:k]
                    reason = "stop"
                    item["finished"] = True
                text_so_far = text
                yield {"delta": delta, "tokens": item["tokens"], "finished": item["finished"], "reason": reason,
                       "all": toks, "text": text, "engine_done": engine_finished,
                       "new_lps": item.get("logprobs"), "lps": lps}
                if item["finished"]:
                    return

        def fmt_lps(toks, lps):
            if params.logprobs is None or lps is None:
                return None
            if chat:
                def entry(t, lp):
                    s_ = tok.decode([t])
                    return {"token": s_, "logprob": lp, "bytes": list(s_.encode())}
                return {"content": [{**entry(t, lp), "top_logprobs": [entry(k, v) for k, v in top.items()]}
                                    for t, (lp, top) in zip(toks, lps)]}
            return {"tokens": [tok.decode([t]) for t in toks], "token_logprobs": [lp for lp, _ in lps],
                    "top_logprobs": [{tok.decode([k]): v for k, v in top.items()} for _, top in lps]}

        def choice(delta=None, text=None, reason=None, toks=None, lps=None):
            out = _choice(delta, text, reason, toks)
            lp = fmt_lps(toks or [], lps)
            if lp is not None:
                out["logprobs"] = lp
            return out

        def _choice(delta=None, text=None, reason=None, toks=None):
            if chat:
                if delta is not None:
                    return {"index": 0, "delta": {"role": "assistant", "content": delta}, "finish_reason": reason}
                msg = {"role": "assistant", "content": text}
                if reasoning:
                    r_text, text = parsers.split_reasoning(text)
                    msg["content"] = text
                    if r_text:
                        msg["reasoning_content"] = r_text
                if body.get("tools"):
                    content, calls = parsers.parse_tool_calls(msg["content"])
                    if calls:
                        msg["content"] = content or None
                        msg["tool_calls"] = calls
                        reason = "tool_calls"
                return {"index": 0, "message": msg, "finish_reason": reason}
            return {"index": 0, "text": delta if delta is not None else text, "finish_reason": reason,
                    "token_ids": toks}

        if stream:
            async def sse():
                async for ev in events():
                    if "error" in ev:
                        yield f"data: {json.dumps({'error': ev['error']})}\n\n"
                        break
                    chunk = {"id": rid, "object": obj + (".chunk" if chat else ""), "created": created,
                             "model": model_name,
                             "choices": [choice(delta=ev["delta"], reason=ev["reason"] if ev["finished"] else None,
                                                toks=ev["tokens"], lps=ev["new_lps"])]}
                    yield f"data: {json.dumps(chunk)}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(sse(), media_type="text/event-stream")
        last = None
        async for ev in events():
            if "error" in ev:
                raise HTTPException(status_code=400, detail=ev["error"])
            last = ev
        usage = {"prompt_tokens": len(prompt_ids), "completion_tokens": len(last["all"]) if last else 0}
        usage["total_tokens"] = usage["prompt_tokens"] + usage["completion_tokens"]
        res = {"id": rid, "object": obj, "created": created, "model": model_name,
               "choices": [choice(text=last["text"] if last else "", reason=last["reason"] if last else "stop",
                                  toks=last["all"] if last else [], lps=last["lps"] if last else [])],
               "usage": usage}
        return res if raw else JSONResponse(res)

    async def _run_n(prompt_ids, params, stops, chat: bool, body: dict, n: int):
        """n completions of one prompt (non-streaming): request i samples with seed + i when a seed is given."""
        from dataclasses import replace
        outs = await asyncio.gather(*[
            _run(prompt_ids, replace(params, seed=None if params.seed is None else params.seed + i), stops, chat,
                 False, body, raw=True) for i in range(n)])
        choices = []
        for i, o in enumerate(outs):
            c = o["choices"][0]
            c["index"] = i
            choices.append(c)
        comp = sum(o["usage"]["completion_tokens"] for o in outs)
        return JSONResponse({**outs[0], "choices": choices,
                             "usage": {"prompt_tokens": len(prompt_ids), "completion_tokens": comp,
                                       "total_tokens": len(prompt_ids) + comp}})

    async def _dispatch(prompt_ids, params, stops, chat: bool, body: dict):
        n = int(body.get("n") or 1)
        stream = bool(body.get("stream"))
        if not 1 <= n <= max_n:
            raise HTTPException(status_code=400, detail=f"n must be in [1, {max_n}]")
        if n > 1:
            if stream:
                raise HTTPException(status_code=400, detail="n > 1 is not supported with stream")
            return await _run_n(prompt_ids, params, stops, chat, body, n)
        return await _run(prompt_ids, params, stops, chat, stream, body)

    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        prompt = body.get("prompt", "")
        if isinstance(prompt, list) and prompt and isinstance(prompt[0], int):
            ids = list(prompt)
        elif isinstance(prompt, list):
            ids = tok.encode("".join(str(p) for p in prompt))
        else:
            ids = tok.encode(str(prompt))
        return await _dispatch(ids, _params(body, tok, engine=llm.engine), _stop_strings(body), False, body)

    @app.post("/tokenize")
    async def tokenize(req: Request):
        """Token ids of a prompt, or of chat messages after the chat template (``messages``)."""
        body = await req.json()
        if "messages" in body:
            msgs = [m for m in body.get("messages") or [] if isinstance(m, dict)]
            ids = tok.encode(tok.apply_chat_template(msgs, reasoning_effort=body.get("reasoning_effort"),
                                                     tools=body.get("tools")))
        else:
            ids = tok.encode(str(body.get("prompt", "")))
        return {"tokens": ids, "count": len(ids), "max_model_len": llm.engine.cfg.max_model_len}

    @app.post("/detokenize")
    async def detokenize(req: Request):
        body = await req.json()
        return {"prompt": tok.decode([int(t) for t in body.get("tokens") or []])}

    @app.post("/v1/chat/completions")
    async def chat(req: Request):
        body = await req.json()
        msgs = [m for m in body.get("messages", []) if isinstance(m, dict)]     # skip unknown input items
        ids = tok.encode(tok.apply_chat_template(msgs, reasoning_effort=body.get("reasoning_effort"),
                                                 tools=body.get("tools")))
        return await _dispatch(ids, _params(body, tok, chat=True, engine=llm.engine), _stop_strings(body), True, body)

    @app.post("/v1/responses")
    async def responses(req: Request):
        body = await req.json()
        msgs = parsers.responses_input_to_messages(body.get("input"), body.get("instructions"))
        ids = tok.encode(tok.apply_chat_template(msgs, reasoning_effort=(body.get("reasoning") or {}).get("effort"),
                                                 tools=body.get("tools")))
        cbody = dict(body, max_tokens=body.get("max_output_tokens") or body.get("max_tokens") or 64)
        res = await _run(ids, _params(cbody, tok, engine=llm.engine), _stop_strings(body), True, False, cbody)
        data = json.loads(res.body)
        msg = data["choices"][0]["message"]
        output = []
        if msg.get("reasoning_content"):
            output.append({"type": "reasoning", "id": f"rs_{uuid.uuid4().hex[:16]}",
                           "summary": [{"type": "summary_text", "text": msg["reasoning_content"]}]})
        for call in msg.get("tool_calls") or []:
            output.append({"type": "function_call", "id": f"fc_{uuid.uuid4().hex[:16]}", "call_id": call["id"],
                           "name": call["function"]["name"], "arguments": call["function"]["arguments"]})
        if msg.get("content"):
            output.append({"type": "message", "id": f"msg_{uuid.uuid4().hex[:16]}", "role": "assistant",
                           "status": "completed",
                           "content": [{"type": "output_text", "text": msg["content"], "annotations": []}]})
        u = data["usage"]
        return JSONResponse({"id": "resp_" + data["id"], "object": "response", "created_at": data["created"],
                             "model": model_name, "status": "completed", "output": output,
                             "output_text": msg.get("content") or "",
                             "usage": {"input_tokens": u["prompt_tokens"], "output_tokens": u["completion_tokens"],
                                       "total_tokens": u["total_tokens"]}})

    return app


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description="OpenAI-compatible GLM-5.3-Flash server on B200")
    ap.add_argument("--model", default="tiny")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-seqs", type=int, default=4)
    ap.add_argument("--max-model-len", type=int, default=8192)
    ap.add_argument("--prefill-chunk", type=int, default=2048)
    ap.add_argument("--mixed-prefill-chunk", type=int, default=0,
                    help="prefill tokens per step while requests decode (0: the whole prefill chunk)")
    ap.add_argument("--page-size", type=int, default=64)
    ap.add_argument("--kv-cache-bytes", type=int, default=None,
                    help="KV cache budget per GPU in bytes (default: enough for max-seqs x max-model-len)")
    ap.add_argument("--checkpoints", type=int, default=4, help="KDA state checkpoint slots for prefix caching")
    ap.add_argument("--no-spec", action="store_true")
    ap.add_argument("--num-speculative-tokens", type=int, default=None,
                    help="fixed draft length (default: adaptive over --k-set)")
    ap.add_argument("--k-set", default="4,5,7", help="draft lengths of the adaptive K")
    ap.add_argument("--block-verify", action="store_true", help="block verification for sampled requests")
    ap.add_argument("--vtrim-tau", type=float, default=0.0, help="verify trimming by drafter confidence (0: off)")
    ap.add_argument("--no-cuda-graphs", action="store_true")
    ap.add_argument("--served-model-name", default="glm-5.3-flash")
    ap.add_argument("--api-key", default=None, help="require Authorization: Bearer <key> on /v1 routes")
    ap.add_argument("--no-reasoning-parser", action="store_true")
    return ap


def options_from_args(args):
    """The engine options of a parsed command line."""
    from .offline import LLMOptions
    return LLMOptions(model=args.model, max_seqs=args.max_seqs, max_model_len=args.max_model_len,
                      prefill_chunk=args.prefill_chunk, mixed_prefill_chunk=args.mixed_prefill_chunk,
                      page_size=args.page_size, kv_cache_bytes=args.kv_cache_bytes, checkpoints=args.checkpoints,
                      speculative=not args.no_spec, k_set=tuple(int(k) for k in args.k_set.split(",")),
                      k_fixed=args.num_speculative_tokens, block_verify=args.block_verify,
                      vtrim_tau=args.vtrim_tau, cuda_graphs=not args.no_cuda_graphs)


def serve(argv=None):
    args = build_parser().parse_args(argv)
    from ..parallel import dist as D
    from .offline import LLM
    rank, _, world = D.init()
    comm, group = None, None
    if world > 1:
        import datetime

        import torch.distributed as dist
        comm = D.NcclComm()
        group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=60))
    llm = LLM(options_from_args(args), comm=comm, rank=rank, world=world)
    try:
        if rank != 0:
            ControlPlane(llm.engine, group).follow()
        else:
            import uvicorn
            app = build_app(llm, args.served_model_name, api_key=args.api_key,
                            reasoning=not args.no_reasoning_parser, group=group)
            try:
                uvicorn.run(app, host=args.host, port=args.port, log_level="info")
            finally:
                app.state.engine_loop.close()
    finally:
        # graphs that hold collectives are released before the process group, or the exit waits on them
        llm.backend._graphs.clear()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    serve()
