"""OpenAI-compatible server on the CPU tiny model (FastAPI TestClient), parsers, detokenizer."""
import json

import pytest
from fastapi.testclient import TestClient

from vllm_sly_radiance_b200.config import EngineConfig
from vllm_sly_radiance_b200.engine.llm_engine import LLMEngine
from vllm_sly_radiance_b200.engine.tokenizer import ByteTokenizer, IncrementalDetokenizer
from vllm_sly_radiance_b200.entrypoints.openai_server import build_app
from vllm_sly_radiance_b200.entrypoints.parsers import ReasoningParser, ToolParser


@pytest.fixture(scope="module")
def client():
    eng = LLMEngine(EngineConfig(model="tiny_hybrid", device="cpu", max_model_len=512,
                                 max_num_seqs=4, max_num_batched_tokens=128, num_kv_blocks=64))
    app = build_app(eng, "tiny,alias", reasoning_parser="qwen3", tool_parser="qwen3_xml")
    with TestClient(app) as c:
        yield c


def test_health_models_metrics(client):
    assert client.get("/health").status_code == 200
    ids = [m["id"] for m in client.get("/v1/models").json()["data"]]
    assert ids == ["tiny", "alias"]
    assert "vllm:num_requests_running" in client.get("/metrics").text


def test_completion(client):
    r = client.post("/v1/completions", json={"model": "tiny", "prompt": "hello world",
                                             "max_tokens": 5, "temperature": 0})
    j = r.json()
    assert r.status_code == 200, j
    assert j["usage"]["completion_tokens"] == 5
    assert j["choices"][0]["finish_reason"] == "length"


def test_completion_stream_and_chat(client):
    with client.stream("POST", "/v1/completions",
                       json={"prompt": "abc", "max_tokens": 4, "stream": True, "temperature": 0}) as r:
        lines = [l for l in r.iter_lines() if l.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    assert json.loads(lines[-2][6:])["choices"][0]["finish_reason"] == "length"
    r = client.post("/v1/chat/completions", json={
        "messages": [{"role": "user", "content": "hi"}], "max_tokens": 3, "temperature": 0.7,
        "top_p": 0.95, "top_k": 20, "seed": 3})
    j = r.json()
    assert j["object"] == "chat.completion" and j["usage"]["completion_tokens"] == 3


def test_bad_requests(client):
    assert client.post("/v1/completions", json={"model": "nope", "prompt": "x"}).status_code == 404
    assert client.post("/v1/completions", json={"prompt": "x", "top_p": 0}).status_code == 400


def test_reasoning_and_tool_parsers():
    rp = ReasoningParser("qwen3")
    assert rp.split("<think>plan</think>\n\nanswer") == ("plan", "answer")
    rp2 = ReasoningParser("qwen3")
    got_r, got_c = "", ""
    for piece in ["<think>pl", "an</thi", "nk>\nans", "wer"]:
        r, c = rp2.stream(piece)
        got_r += r
        got_c += c
    assert got_r == "plan" and got_c == "answer"
    tp = ToolParser("qwen3_xml")
    calls, rest = tp.parse("ok <tool_call>\n<function=get_weather>\n<parameter=city>\nParis\n"
                           "</parameter>\n<parameter=days>\n3\n</parameter>\n</function>\n</tool_call>")
    assert calls[0]["function"]["name"] == "get_weather"
    assert json.loads(calls[0]["function"]["arguments"]) == {"city": "Paris", "days": 3}
    assert rest == "ok"
    calls, _ = ToolParser("hermes").parse('<tool_call>{"name": "f", "arguments": {"a": 1}}</tool_call>')
    assert calls[0]["function"]["name"] == "f"


def test_detokenizer_stop_strings():
    tok = ByteTokenizer()
    d = IncrementalDetokenizer(tok, stop=["END"])
    ids = tok.encode("hello EN")
    assert d.update(ids) == "hello "          # "EN" held back as a possible stop prefix
    ids = tok.encode("hello END more")
    d.update(ids)
    assert d.stopped and d.text == "hello "
