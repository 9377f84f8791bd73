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
    txt = client.get("/metrics").text
    assert "glm53_generation_tokens_total" in txt and "glm53_spec_decode_num_drafts_total" in txt


def test_too_long_is_400(client):
    r = client.post("/v1/completions", json={"prompt": list(range(3000)), "max_tokens": 10})
    assert r.status_code == 400
