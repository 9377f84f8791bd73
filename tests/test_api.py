"""OpenAI-compatible server on CPU (fake backend): completions, chat, streaming, stop strings, metrics, health."""

import json

import pytest

from glm53.engine.llm import EngineConfig, LLMEngine
from glm53.engine.tokenizer import ByteTokenizer
from tests.fake_backend import FakeBackend, reference_greedy


class FakeLLM:
    def __init__(self):
        self.engine = LLMEngine(FakeBackend(), EngineConfig(max_seqs=4, page_size=16, num_pages=256,
                                                             max_model_len=2048, prefill_chunk=64,
                                                             cuda_graphs=False))
        self.tokenizer = ByteTokenizer(512)


@pytest.fixture(scope="module")
def client():
    from fastapi.testclient import TestClient
    from glm53.api.server import build_app
    app = build_app(FakeLLM(), "glm-test")
    with TestClient(app) as c:
        yield c


def test_health_models(client):
    assert client.get("/health").json()["status"] == "ok"
    assert client.get("/v1/models").json()["data"][0]["id"] == "glm-test"


def test_completion_token_ids(client):
    prompt = list(range(20, 60))
    r = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 12})
    body = r.json()
    assert r.status_code == 200
    assert body["choices"][0]["token_ids"] == reference_greedy(prompt, 12)
    assert body["usage"]["completion_tokens"] == 12 and body["usage"]["prompt_tokens"] == 40


def test_completion_stream_and_chat(client):
    r = client.post("/v1/completions", json={"prompt": "hello", "max_tokens": 9, "stream": True})
    events = [l[6:] for l in r.text.splitlines() if l.startswith("data: ")]
    assert events[-1] == "[DONE]"
    toks = []
    for ev in events[:-1]:
        toks += json.loads(ev)["choices"][0]["token_ids"]
    tok = ByteTokenizer(512)
    assert toks == reference_greedy(tok.encode("hello"), 9)
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}, "junk item"],
                                                  "max_tokens": 5})
    body = r.json()
    assert body["object"] == "chat.completion" and body["choices"][0]["message"]["role"] == "assistant"


def test_metrics(client):
    client.post("/v1/completions", json={"prompt": list(range(20, 60)), "max_tokens": 24})
    txt = client.get("/metrics").text
    assert "glm53_generation_tokens_total" in txt and "glm53_spec_decode_num_drafts_total" in txt
    vals = {l.split(" ")[0]: float(l.split(" ")[1]) for l in txt.splitlines() if l and not l.startswith("#")}
    windows = vals["glm53_spec_decode_num_windows_total"]
    per_pos = [vals[f'glm53_spec_decode_num_accepted_tokens_per_pos{{position="{i}"}}'] for i in range(8)]
    assert windows > 0 and per_pos[0] <= windows
    assert all(a >= b for a, b in zip(per_pos, per_pos[1:]))     # position i is accepted only after 0 .. i-1


def test_too_long_is_400(client):
    r = client.post("/v1/completions", json={"prompt": list(range(3000)), "max_tokens": 10})
    assert r.status_code == 400


def test_parsers_reasoning_tools_stops():
    from glm53.api import parsers
    r, a = parsers.split_reasoning("<think>plan it</think>\nThe answer")
    assert (r, a) == ("plan it", "The answer")
    assert parsers.split_reasoning("plain")[1] == "plain"
    text = "pre <tool_call>get_weather\n<arg_key>city</arg_key>\n<arg_value>Paris</arg_value>\n" \
           "<arg_key>days</arg_key>\n<arg_value>3</arg_value>\n</tool_call>"
    content, calls = parsers.parse_tool_calls(text)
    assert content == "pre" and calls[0]["function"]["name"] == "get_weather"
    assert json.loads(calls[0]["function"]["arguments"]) == {"city": "Paris", "days": 3}
    _, calls = parsers.parse_tool_calls('<tool_call>{"name": "f", "arguments": {"x": 1}}</tool_call>')
    assert calls[0]["function"]["name"] == "f"
    # stops inside the reasoning are ignored
    t = "<think>STOP here</think>answer STOP"
    assert parsers.stop_index(t, ["STOP"], True) == t.rfind("STOP")
    assert parsers.stop_index(t, ["STOP"], False) == t.find("STOP")
    msgs = parsers.responses_input_to_messages(
        [{"type": "message", "role": "user", "content": [{"type": "input_text", "text": "hi"}]},
         {"type": "reasoning", "summary": []}, {"type": "unknown_thing"}], "be brief")
    assert msgs == [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"}]


def test_chat_template_effort_placement():
    tok = ByteTokenizer(512)
    sys_msg = {"role": "system", "content": "S"}
    a = tok.apply_chat_template([sys_msg, {"role": "user", "content": "u"}], reasoning_effort="high")
    b = tok.apply_chat_template([sys_msg, {"role": "user", "content": "u"}], reasoning_effort="low")
    head = tok.apply_chat_template([sys_msg], add_generation_prompt=False)
    assert a.startswith(head) and b.startswith(head) and "Reasoning effort: high" in a


def test_responses_endpoint(client):
    r = client.post("/v1/responses", json={"input": [{"role": "user", "content": "hi"}, {"type": "bogus"}],
                                           "max_output_tokens": 6})
    body = r.json()
    assert r.status_code == 200 and body["object"] == "response" and body["usage"]["output_tokens"] == 6


def test_api_key():
    from fastapi.testclient import TestClient
    from glm53.api.server import build_app
    app = build_app(FakeLLM(), "glm-test", api_key="sekret")
    with TestClient(app) as c:
        assert c.get("/v1/models").status_code == 401
        assert c.get("/v1/models", headers={"Authorization": "Bearer sekret"}).status_code == 200


def test_server_flags_map_to_engine_options():
    from glm53.api.server import build_parser, options_from_args
    args = build_parser().parse_args(["--model", "full", "--num-speculative-tokens", "7", "--block-verify",
                                      "--kv-cache-bytes", "16106127360", "--k-set", "3,5", "--checkpoints", "2",
                                      "--mixed-prefill-chunk", "1024", "--no-cuda-graphs", "--vtrim-tau", "0.2"])
    o = options_from_args(args)
    assert (o.model, o.k_fixed, o.block_verify, o.kv_cache_bytes, o.k_set, o.checkpoints) == (
        "full", 7, True, 16106127360, (3, 5), 2)
    assert o.mixed_prefill_chunk == 1024 and not o.cuda_graphs and o.vtrim_tau == 0.2 and o.speculative
    d = options_from_args(build_parser().parse_args([]))
    assert d.k_fixed is None and d.k_set == (4, 5, 7) and not d.block_verify and d.cuda_graphs


def test_logprobs_and_n(client):
    """Completions: logprobs=n gives per-token log-probabilities and top-n alternatives; chat: logprobs with
    top_logprobs; n > 1 returns n choices (seed + i each), refused with stream."""
    prompt = list(range(20, 60))
    body = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 6, "logprobs": 2}).json()
    lp = body["choices"][0]["logprobs"]
    assert len(lp["token_logprobs"]) == 6 and all(v <= 0 for v in lp["token_logprobs"])
    assert all(len(t) <= 2 for t in lp["top_logprobs"]) and len(lp["tokens"]) == 6
    body = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                     "max_tokens": 4, "logprobs": True, "top_logprobs": 3}).json()
    content = body["choices"][0]["logprobs"]["content"]
    assert len(content) == 4 and all(len(c["top_logprobs"]) == 3 for c in content)
    assert "logprobs" not in client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 3}).json()[
        "choices"][0]
    body = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 5, "n": 3, "temperature": 1.0,
                                                "seed": 4}).json()
    assert [c["index"] for c in body["choices"]] == [0, 1, 2] and body["usage"]["completion_tokens"] == 15
    greedy = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 5, "n": 2}).json()
    assert greedy["choices"][0]["token_ids"] == greedy["choices"][1]["token_ids"] == reference_greedy(prompt, 5)
    r = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 5, "n": 2, "stream": True})
    assert r.status_code == 400


def test_tokenize_detokenize(client):
    r = client.post("/tokenize", json={"prompt": "hello B200"}).json()
    assert r["count"] == len(r["tokens"]) > 0 and r["max_model_len"] == 2048
    assert client.post("/detokenize", json={"tokens": r["tokens"]}).json()["prompt"] == "hello B200"
    chat = client.post("/tokenize", json={"messages": [{"role": "user", "content": "hi"}]}).json()
    assert chat["count"] > 2


def test_bad_sampling_fields_are_400_and_server_keeps_serving(client):
    """A request whose sampling fields the engine could not serve (top_logprobs beyond the cap, a negative
    temperature, n beyond the slot count, a non-numeric field) is refused with 400 before it reaches the engine
    thread; requests after it are served normally."""
    prompt = list(range(20, 60))
    bad = [
        ("/v1/chat/completions", {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 2,
                                  "logprobs": True, "top_logprobs": 10 ** 6}),
        ("/v1/completions", {"prompt": prompt, "max_tokens": 2, "logprobs": 10 ** 6}),
        ("/v1/completions", {"prompt": prompt, "max_tokens": 2, "logprobs": -1}),
        ("/v1/completions", {"prompt": prompt, "max_tokens": 2, "temperature": -0.5}),
        ("/v1/completions", {"prompt": prompt, "max_tokens": 2, "top_p": 0.0}),
        ("/v1/completions", {"prompt": prompt, "max_tokens": 2, "top_k": "many"}),
        ("/v1/completions", {"prompt": prompt, "max_tokens": 2, "n": 10 ** 6}),
    ]
    for route, body in bad:
        r = client.post(route, json=body)
        assert r.status_code == 400, (route, body, r.status_code)
    assert client.get("/health").json()["status"] == "ok"
    body = client.post("/v1/completions", json={"prompt": prompt, "max_tokens": 6}).json()
    assert body["choices"][0]["token_ids"] == reference_greedy(prompt, 6)


def test_engine_rejects_bad_sampling_fields_per_request():
    """add_request raises ValueError (reported for that request alone) for logprobs beyond the cap."""
    from glm53.engine.llm import MAX_LOGPROBS, SamplingParams
    eng = FakeLLM().engine
    with pytest.raises(ValueError):
        eng.add_request([1, 2, 3], SamplingParams(max_tokens=2, logprobs=MAX_LOGPROBS + 1))
    eng.add_request([1, 2, 3], SamplingParams(max_tokens=2, logprobs=MAX_LOGPROBS))
