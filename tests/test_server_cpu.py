"""OpenAI HTTP contract against the engine with a fake model runner (no GPU)."""
import asyncio
import json

import pytest
from aiohttp.test_utils import TestClient, TestServer

from vm_c_b200.config import ServerConfig
from vm_c_b200.server.http import OpenAIServer

from test_engine_cpu import make
from test_tokenizer import gpt2_tok


def run(coro):
    return asyncio.new_event_loop().run_until_complete(coro)


async def with_client(fn):
    eng = make()
    eng.cfg.model.vocab = 100000
    tok = gpt2_tok()
    srv = OpenAIServer(eng, tok, "test-model", ServerConfig())
    client = TestClient(TestServer(srv.app))
    await client.start_server()
    try:
        return await fn(client, tok)
    finally:
        await client.close()
        srv.loop_thread.shutdown()


def test_models_health_version_tokenize():
    async def body(c, tok):
        r = await c.get("/v1/models")
        assert (await r.json())["data"][0]["id"] == "test-model"
        assert (await (await c.get("/health")).json())["status"] == "ok"
        assert "version" in await (await c.get("/version")).json()
        ids = (await (await c.post("/tokenize", json={"content": "hello"})).json())["tokens"]
        assert tok.decode(ids) == "hello"
        txt = (await (await c.post("/detokenize", json={"tokens": ids})).json())["content"]
        assert txt == "hello"
        m = await (await c.get("/metrics")).text()
        assert "vmc_num_running" in m
    run(with_client(body))


def test_completion_non_stream_and_usage():
    async def body(c, tok):
        r = await c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 4, "temperature": 0})
        j = await r.json()
        assert j["object"] == "text_completion"
        assert j["usage"] == {"prompt_tokens": 3, "completion_tokens": 4, "total_tokens": 7}
        assert j["choices"][0]["finish_reason"] == "length"
        assert j["choices"][0]["text"] == tok.decode([8, 9, 10, 11])
    run(with_client(body))


def test_chat_stream_done_and_include_usage():
    async def body(c, tok):
        r = await c.post("/v1/chat/completions", json={
            "messages": [{"role": "user", "content": "hi"}], "max_tokens": 3, "stream": True,
            "stream_options": {"include_usage": True}, "chat_template_kwargs": {"enable_thinking": False}})
        raw = (await r.read()).decode()
        events = [l[6:] for l in raw.split("\n") if l.startswith("data: ")]
        assert events[-1] == "[DONE]"
        chunks = [json.loads(e) for e in events[:-1]]
        assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
        assert chunks[-1]["choices"] == [] and chunks[-1]["usage"]["completion_tokens"] == 3
        assert chunks[-2]["choices"][0]["finish_reason"] == "length"
    run(with_client(body))


def test_bad_requests():
    async def body(c, tok):
        assert (await c.post("/v1/chat/completions", data=b"{not json")).status == 400
        assert (await c.post("/v1/chat/completions", json={"messages": []})).status == 400
    run(with_client(body))


def test_echo_joined_prompts_and_running_usage():
    async def body(c, tok):
        r = await c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 2, "temperature": 0, "echo": True})
        j = await r.json()
        assert j["choices"][0]["text"] == tok.decode([5, 6, 7], skip_special=False) + tok.decode([8, 9])
        r = await c.post("/v1/completions", json={"prompt": ["he", "llo"], "max_tokens": 1, "temperature": 0})
        assert (await r.json())["usage"]["prompt_tokens"] == len(tok.encode("he\nllo"))
        r = await c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 4, "temperature": 0, "stream": True,
                                                  "stream_options": {"continuous_usage_stats": True}})
        evs = [json.loads(x[6:]) for x in (await r.text()).split("\n\n") if x.startswith("data: {")]
        counts = [e["usage"]["completion_tokens"] for e in evs if e.get("usage")]
        assert counts and counts == sorted(counts) and counts[-1] <= 4
    run(with_client(body))
