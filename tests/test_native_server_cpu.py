"""Native OpenAI server (csrc/server/) on the CPU: vmc_serve_cpu serves GGUF vocabularies through the
same HTTP routes, tokenizer, chat prompts, serving loop and scheduler as vmc_run --serve, with a
deterministic rule in place of the model (token after t at position p = (31 t + 7 p + 11) mod V), so
every completion can be predicted here. The text pipeline is compared with the Python server's
(vm_c_b200/server/tokenizer.py, chat.py) and, for the pre-tokenisers, with the published regular
expressions themselves."""
import http.client
import json
import os
import random
import socket
import subprocess
import threading
import time

import pytest
import regex

from vm_c_b200 import _build
from vm_c_b200.gguf.constants import VType
from vm_c_b200.gguf.random_init import synthetic_vocab
from vm_c_b200.server.chat import ChatTemplate, chatml, split_reasoning
from vm_c_b200.server.tokenizer import _PRE, IncrementalDetokenizer, Tokenizer, _byte_unicode

MAX_LEN = 512


@pytest.fixture(scope="module")
def exe():
    return str(_build.build_serve_cpu())


def write_vocab_gguf(path, toks, scores, types, merges, model, pre, bos, eos, template=None, add_bos=True):
    from vm_c_b200 import _native
    w = _native.host().GgufWriter(32)
    md = [("general.architecture", VType.STRING, "llama", 0),
          ("tokenizer.ggml.model", VType.STRING, model, 0),
          ("tokenizer.ggml.pre", VType.STRING, pre, 0),
          ("tokenizer.ggml.tokens", VType.ARRAY, toks, int(VType.STRING)),
          ("tokenizer.ggml.token_type", VType.ARRAY, types, int(VType.INT32)),
          ("tokenizer.ggml.bos_token_id", VType.UINT32, bos, 0),
          ("tokenizer.ggml.eos_token_id", VType.UINT32, eos, 0),
          ("tokenizer.ggml.add_bos_token", VType.BOOL, add_bos, 0)]
    if scores:
        md.append(("tokenizer.ggml.scores", VType.ARRAY, scores, int(VType.FLOAT32)))
    if merges:
        md.append(("tokenizer.ggml.merges", VType.ARRAY, merges, int(VType.STRING)))
    if template:
        md.append(("tokenizer.chat_template", VType.STRING, template, 0))
    for key, vt, val, et in md:
        w.set(key, int(vt), val, int(et))
    w.write(path, lambda i: None)


def spm_vocab():
    toks, scores, types = synthetic_vocab(600)
    scores = [float(len(t)) if ty == 1 else 0.0 for t, ty in zip(toks, types)]
    return toks, scores, types


CORPUS = ("the quick brown fox jumps over the lazy dog. It's 2024 and we'll see 12345 tokens!\n"
          "naïve café déjà vu, 漢字 かな and emoji 😀 in text; don't stop believing\n\tindented  spaces") * 3


def gpt2_vocab(n_merges=300):
    """Byte-level vocabulary with merges learned on CORPUS (a few steps of BPE), plus specials."""
    b2u, _ = _byte_unicode()
    toks = [b2u[b] for b in range(256)]
    words = [[b2u[b] for b in w.encode()] for w in regex.findall(_PRE["llama-bpe"], CORPUS)]
    merges = []
    for _ in range(n_merges):
        counts = {}
        for w in words:
            for a, b in zip(w, w[1:]):
                counts[(a, b)] = counts.get((a, b), 0) + 1
        if not counts:
            break
        (a, b), _c = max(counts.items(), key=lambda kv: (kv[1], kv[0]))
        merges.append(f"{a} {b}")
        toks.append(a + b)
        nw = []
        for w in words:
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and w[i] == a and w[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            nw.append(out)
        words = nw
    specials = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]
    types = [1] * len(toks) + [3] * len(specials)
    toks += specials
    return toks, types, merges


class Server:
    def __init__(self, exe, gguf, tmp, *extra):
        pf = os.path.join(tmp, f"port{random.randrange(1 << 30)}")
        self.proc = subprocess.Popen([exe, gguf, "--port", "0", "--port-file", pf, "--max-model-len", str(MAX_LEN),
                                      *extra], stdout=subprocess.DEVNULL, stderr=subprocess.PIPE)
        t0 = time.time()
        while not os.path.exists(pf) or not open(pf).read().strip():
            if self.proc.poll() is not None:
                raise RuntimeError("server exited: " + self.proc.stderr.read().decode())
            if time.time() - t0 > 30:
                raise RuntimeError("server did not start")
            time.sleep(0.02)
        self.port = int(open(pf).read())

    def request(self, method, path, body=None, raw=None, headers=None):
        c = http.client.HTTPConnection("127.0.0.1", self.port, timeout=30)
        data = raw if raw is not None else (json.dumps(body).encode() if body is not None else None)
        c.request(method, path, body=data, headers=headers or ({"Content-Type": "application/json"} if data else {}))
        r = c.getresponse()
        out = r.status, dict(r.getheaders()), r.read()
        c.close()
        return out

    def post(self, path, body):
        st, _, data = self.request("POST", path, body)
        return st, json.loads(data)

    def stream(self, path, body):
        c = http.client.HTTPConnection("127.0.0.1", self.port, timeout=30)
        c.request("POST", path, body=json.dumps(body).encode(), headers={"Content-Type": "application/json"})
        r = c.getresponse()
        assert r.status == 200 and r.getheader("Content-Type") == "text/event-stream"
        events = [e for e in r.read().decode().split("\n\n") if e]
        c.close()
        assert events[-1] == "data: [DONE]"
        return [json.loads(e[len("data: "):]) for e in events[:-1]]

    def close(self):
        self.proc.terminate()
        try:
            self.proc.wait(10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()


def predict(prompt, V, max_tokens, eos, ignore_eos=False, min_tokens=0, stop_ids=()):
    """Tokens the rule backend produces for `prompt` and the finish reason (the scheduler's rules)."""
    out, t, p = [], prompt[-1], len(prompt) - 1
    while True:
        t = (31 * t + 7 * p + 11) % V
        p += 1
        out.append(t)
        n = len(out)
        is_eos = t in eos and not ignore_eos and n > min_tokens
        is_stop = t in stop_ids and n > min_tokens
        if is_eos or is_stop:
            return out, "stop"
        if n >= max_tokens or len(prompt) + n >= MAX_LEN:
            return out, "length"


def detok(tok, ids, stop=None):
    d = IncrementalDetokenizer(tok, stop)
    text = "".join(d.push([i]) for i in ids)
    return text + d.push([], final=True), d.stopped


@pytest.fixture(scope="module")
def spm(exe, tmp_path_factory):
    tmp = str(tmp_path_factory.mktemp("spm"))
    toks, scores, types = spm_vocab()
    path = os.path.join(tmp, "spm.gguf")
    write_vocab_gguf(path, toks, scores, types, [], "llama", "default", 1, 2)
    tok = Tokenizer(toks, scores, types, [], "llama", "default", 1, [2], True)
    srv = Server(exe, path, tmp, "--max-num-batched-tokens", "64", "--max-num-seqs", "8")
    yield srv, tok
    srv.close()


@pytest.fixture(scope="module", params=["llama-bpe", "qwen2", "gpt2", "qwen35", "llama3"])
def bpe(exe, tmp_path_factory, request):
    tmp = str(tmp_path_factory.mktemp("bpe"))
    toks, types, merges = gpt2_vocab()
    path = os.path.join(tmp, "bpe.gguf")
    eos = toks.index("<|im_end|>")
    write_vocab_gguf(path, toks, [], types, merges, "gpt2", request.param, toks.index("<|endoftext|>"), eos,
                     add_bos=False)
    tok = Tokenizer(toks, [], types, merges, "gpt2", request.param, toks.index("<|endoftext|>"), [eos], False)
    srv = Server(exe, path, tmp)
    yield srv, tok
    srv.close()


TEXTS = ["hello world", "I'm here, it's fine; they'll go", "  two  spaces\n\nand lines\r\n", "digits 1234567 x",
         "naïve café 漢字 😀", "<|im_start|>user\nhi<|im_end|>", "", "tab\tsep", "UPPER 'S 'LL", CORPUS[:200],
         "cafe\u0301 ke\u0300 नि क\u093fत \u20d7x"]


def test_pre_tokenizers_match_regex(exe):
    alphabet = list("abcXYZ'sStTrReEvVmMlLdD019 \t\n\r.,!?-_()\"") + \
        ["é", "ü", "漢", "٣", "½", "Ⅻ", "😀", " ", "　", "​", "́", "ſ", "ǅ", "\x0b", "\x85", "ß",
         "\u0300", "\u093f", "\u20d7", "क"]  # combining marks (Mn, Mc) and a letter they follow
    rng = random.Random(0)
    texts = TEXTS + ["".join(rng.choice(alphabet) for _ in range(rng.randint(0, 24))) for _ in range(1500)]
    for fam in ("gpt2", "llama-bpe", "qwen2", "qwen35"):
        inp = "".join(json.dumps(t) + "\n" for t in texts).encode()
        out = subprocess.run([exe, "--tool", "pre-split", fam], input=inp, capture_output=True, check=True).stdout
        got = [json.loads(x) for x in out.decode().split("\n") if x]
        rx = regex.compile(_PRE[fam])
        bad = [(t, rx.findall(t), g) for t, g in zip(texts, got) if rx.findall(t) != g]
        assert len(got) == len(texts) and not bad, (fam, bad[:3])


def test_tokenize_matches_python_spm(spm):
    srv, tok = spm
    for text in TEXTS:
        for add in (False, True):
            st, r = srv.post("/tokenize", {"content": text, "add_special": add})
            assert st == 200 and r["tokens"] == tok.encode(text, add_bos=add), text
        st, r = srv.post("/detokenize", {"tokens": tok.encode(text, add_bos=True)})
        assert r["content"] == r["text"] == tok.decode(tok.encode(text, add_bos=True), skip_special=False)
        st, r = srv.post("/tokenize", {"text": text})  # the reference's field name
        assert r["tokens"] == tok.encode(text, add_bos=False)


def test_tokenize_matches_python_bpe(bpe):
    srv, tok = bpe
    rng = random.Random(1)
    words = CORPUS.split(" ")
    texts = TEXTS + [" ".join(rng.choice(words) for _ in range(rng.randint(1, 12))) for _ in range(60)]
    for text in texts:
        st, r = srv.post("/tokenize", {"content": text})
        assert st == 200 and r["tokens"] == tok.encode(text, add_bos=False), text
        ids = r["tokens"]
        st, r = srv.post("/detokenize", {"tokens": ids})
        assert r["content"] == tok.decode(ids, skip_special=False) == text


def test_completion_matches_prediction(spm):
    srv, tok = spm
    V = len(tok.tokens)
    for i, prompt in enumerate(["the rain in spain", "once upon a time there was a " * 5, "x"]):
        body = {"prompt": prompt, "max_tokens": 20 + i, "temperature": 0}
        st, r = srv.post("/v1/completions", body)
        ids = tok.encode(prompt)
        want, reason = predict(ids, V, 20 + i, [2])
        text, _ = detok(tok, want)
        assert st == 200 and r["object"] == "text_completion"
        assert r["choices"][0]["text"] == text and r["choices"][0]["finish_reason"] == reason
        assert r["usage"] == {"prompt_tokens": len(ids), "completion_tokens": len(want),
                              "total_tokens": len(ids) + len(want)}
        # the same request streamed: the deltas add up to the same text
        ev = srv.stream("/v1/completions", {**body, "stream": True, "stream_options": {"include_usage": True}})
        assert "".join(e["choices"][0]["text"] for e in ev if e["choices"]) == text
        assert ev[-2]["choices"][0]["finish_reason"] == reason
        assert ev[-1]["choices"] == [] and ev[-1]["usage"]["completion_tokens"] == len(want)


def test_token_id_prompt_stop_ids_min_tokens_ignore_eos(spm):
    srv, tok = spm
    V = len(tok.tokens)
    ids = tok.encode("ids given directly", add_bos=True)
    want, _ = predict(ids, V, 40, [2], ignore_eos=True)
    stop_id = want[5]
    st, r = srv.post("/v1/completions", {"prompt": ids, "max_tokens": 40, "ignore_eos": True,
                                         "stop_token_ids": [stop_id], "min_tokens": 3})
    exp, reason = predict(ids, V, 40, [2], ignore_eos=True, min_tokens=3, stop_ids=[stop_id])
    assert st == 200 and r["choices"][0]["finish_reason"] == reason == "stop"
    assert r["usage"]["completion_tokens"] == len(exp) and r["choices"][0]["text"] == detok(tok, exp)[0]


def test_stop_string_truncates(spm):
    srv, tok = spm
    V = len(tok.tokens)
    ids = tok.encode("stop strings")
    want, _ = predict(ids, V, 60, [2], ignore_eos=True)
    full, _ = detok(tok, want)
    stop = full[len(full) // 2: len(full) // 2 + 2]
    expect, stopped = detok(tok, want, [stop])
    assert stopped
    for stream in (False, True):
        body = {"prompt": "stop strings", "max_tokens": 60, "ignore_eos": True, "stop": stop}
        if stream:
            ev = srv.stream("/v1/completions", {**body, "stream": True})
            text = "".join(e["choices"][0]["text"] for e in ev)
            reason = ev[-1]["choices"][0]["finish_reason"]
        else:
            st, r = srv.post("/v1/completions", body)
            text, reason = r["choices"][0]["text"], r["choices"][0]["finish_reason"]
        assert text == expect and reason == "stop"


def test_chat_chatml_prompt_and_reasoning(spm):
    srv, tok = spm
    V = len(tok.tokens)
    msgs = [{"role": "system", "content": "be brief"}, {"role": "user", "content": [{"type": "text", "text": "hi"}]}]
    for thinking in (True, False):
        prompt = chatml([{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"}], True, thinking)
        ids = tok.encode(prompt, add_bos=not prompt.startswith(tok.tokens[tok.bos_id]))
        want, reason = predict(ids, V, 30, [2])
        text, _ = detok(tok, want)
        reasoning, content = split_reasoning(text, thinking)
        st, r = srv.post("/v1/chat/completions", {"messages": msgs, "max_tokens": 30,
                                                  "chat_template_kwargs": {"enable_thinking": thinking}})
        assert st == 200 and r["object"] == "chat.completion"
        assert r["usage"]["prompt_tokens"] == len(ids)
        m = r["choices"][0]["message"]
        assert m["role"] == "assistant" and m["content"] == content and m.get("reasoning_content", "") == reasoning
        ev = srv.stream("/v1/chat/completions", {"messages": msgs, "max_tokens": 30, "stream": True,
                                                 "enable_thinking": thinking})
        assert ev[0]["choices"][0]["delta"] == {"role": "assistant", "content": ""}
        # streamed, everything before "</think>" is reasoning (all of it when the tag never comes)
        s_reason, s_content = (text, "") if thinking and "</think>" not in text else (reasoning, content)
        assert "".join(e["choices"][0]["delta"].get("reasoning_content", "") for e in ev) == s_reason
        assert "".join(e["choices"][0]["delta"].get("content", "") for e in ev) == s_content
        assert ev[-1]["choices"][0]["finish_reason"] == reason


def test_concurrent_requests_continuous_batching(spm):
    """Many clients at once: prompts of different lengths span several 64-token prefill chunks and the
    decode batch changes every step; every answer must equal its own prediction."""
    srv, tok = spm
    V = len(tok.tokens)
    rng = random.Random(3)
    prompts = [" ".join(rng.choice(["alpha", "beta", "gamma", "delta"]) for _ in range(rng.randint(1, 40)))
               for _ in range(24)]
    results = [None] * len(prompts)

    def run(i):
        results[i] = srv.post("/v1/completions", {"prompt": prompts[i], "max_tokens": 5 + i, "temperature": 0,
                                                  "ignore_eos": True})
    th = [threading.Thread(target=run, args=(i,)) for i in range(len(prompts))]
    for t in th:
        t.start()
    for t in th:
        t.join(60)
    for i, (st, r) in enumerate(results):
        want, reason = predict(tok.encode(prompts[i]), V, 5 + i, [2], ignore_eos=True)
        assert st == 200 and r["choices"][0]["text"] == detok(tok, want)[0] and r["usage"]["completion_tokens"] == len(want)
    _, _, m = srv.request("GET", "/metrics")
    m = dict(line.split(" ", 1) for line in m.decode().splitlines() if line and not line.startswith("#"))
    assert float(m["vmc_num_running"]) == 0 and float(m["vmc_finished"]) >= len(prompts)


def test_client_disconnect_aborts(exe, tmp_path):
    toks, scores, types = spm_vocab()
    path = str(tmp_path / "v.gguf")
    write_vocab_gguf(path, toks, scores, types, [], "llama", "default", 1, 2)
    srv = Server(exe, path, str(tmp_path), "--step-delay-ms", "20")
    try:
        s = socket.create_connection(("127.0.0.1", srv.port), timeout=10)
        body = json.dumps({"prompt": "never ending", "max_tokens": 400, "ignore_eos": True, "stream": True}).encode()
        s.sendall(b"POST /v1/completions HTTP/1.1\r\nHost: x\r\nContent-Type: application/json\r\n"
                  b"Content-Length: " + str(len(body)).encode() + b"\r\n\r\n" + body)
        got = b""
        while got.count(b"data: ") < 3:
            got += s.recv(4096)
        s.close()
        t0 = time.time()
        while True:
            _, _, m = srv.request("GET", "/metrics")
            m = dict(line.split(" ", 1) for line in m.decode().splitlines() if line and not line.startswith("#"))
            if float(m["vmc_aborted"]) == 1 and float(m["vmc_num_running"]) == 0:
                break
            assert time.time() - t0 < 10, m
            time.sleep(0.05)
        assert float(m["vmc_tokens_generated"]) < 400
    finally:
        srv.close()


def test_routes_and_errors(spm):
    srv, tok = spm
    st, h, data = srv.request("GET", "/v1/models")
    assert st == 200 and json.loads(data)["data"][0]["id"] == "vm_c" and h["Access-Control-Allow-Origin"] == "*"
    assert json.loads(data)["data"][0]["permission"][0]["object"] == "model_permission"
    assert json.loads(srv.request("GET", "/health")[2]) == {"status": "ok"}
    assert "version" in json.loads(srv.request("GET", "/version")[2])
    assert srv.request("OPTIONS", "/v1/completions")[0] == 204
    assert srv.request("GET", "/nope")[0] == 404
    assert srv.request("GET", "/v1/completions")[0] == 405
    st, _, data = srv.request("POST", "/v1/completions", raw=b"{not json")
    assert st == 400 and json.loads(data)["error"]["code"] == 400
    assert srv.post("/v1/chat/completions", {"messages": []})[0] == 400
    st, r = srv.post("/v1/completions", {"prompt": [len(tok.tokens) + 5]})
    assert st == 400 and "vocabulary" in r["error"]["message"]
    assert srv.post("/v1/completions", {"prompt": "x", "max_tokens": "many"})[0] == 400
    # keep-alive: two requests over one connection
    c = http.client.HTTPConnection("127.0.0.1", srv.port, timeout=10)
    for _ in range(2):
        c.request("GET", "/health")
        assert c.getresponse().read() == b'{"status": "ok"}'
    c.close()


LLAMA3 = ("{% set loop_messages = messages %}{% for message in loop_messages %}{% set content = "
          "'<|start_header_id|>' + message['role'] + '<|end_header_id|>\n\n'+ message['content'] | trim + "
          "'<|eot_id|>' %}{% if loop.index0 == 0 %}{% set content = bos_token + content %}{% endif %}"
          "{{ content }}{% endfor %}{% if add_generation_prompt %}"
          "{{ '<|start_header_id|>assistant<|end_header_id|>\n\n' }}{% endif %}")
MISTRAL = ("{{ bos_token }}{% for message in messages %}{% if (message['role'] == 'user') != "
           "(loop.index0 % 2 == 0) %}{{ raise_exception('Conversation roles must alternate "
           "user/assistant/user/assistant/...') }}{% endif %}{% if message['role'] == 'user' %}"
           "{{ '[INST] ' + message['content'] + ' [/INST]' }}{% elif message['role'] == 'assistant' %}"
           "{{ message['content'] + eos_token}}{% else %}{{ raise_exception('Only user and assistant roles "
           "are supported!') }}{% endif %}{% endfor %}")
GEMMA = ("{{ bos_token }}{% if messages[0]['role'] == 'system' %}{{ raise_exception('System role not supported') }}"
         "{% endif %}{% for message in messages %}{% if (message['role'] == 'user') != (loop.index0 % 2 == 0) %}"
         "{{ raise_exception('Conversation roles must alternate user/assistant/user/assistant/...') }}{% endif %}"
         "{% if (message['role'] == 'assistant') %}{% set role = 'model' %}{% else %}{% set role = message['role'] %}"
         "{% endif %}{{ '<start_of_turn>' + role + '\n' + message['content'] | trim + '<end_of_turn>\n' }}"
         "{% endfor %}{% if add_generation_prompt %}{{'<start_of_turn>model\n'}}{% endif %}")
PHI3 = ("{% for message in messages %}{% if message['role'] == 'system' %}{{'<|system|>\n' + message['content'] + "
        "'<|end|>\n'}}{% elif message['role'] == 'user' %}{{'<|user|>\n' + message['content'] + '<|end|>\n'}}"
        "{% elif message['role'] == 'assistant' %}{{'<|assistant|>\n' + message['content'] + '<|end|>\n'}}{% endif %}"
        "{% endfor %}{% if add_generation_prompt %}{{ '<|assistant|>\n' }}{% else %}{{ eos_token }}{% endif %}")
ZEPHYR = """{% for message in messages %}
{% if message['role'] == 'user' %}
{{ '<|user|>\n' + message['content'] + eos_token }}
{% elif message['role'] == 'system' %}
{{ '<|system|>\n' + message['content'] + eos_token }}
{% elif message['role'] == 'assistant' %}
{{ '<|assistant|>\n'  + message['content'] + eos_token }}
{% endif %}
{% if loop.last and add_generation_prompt %}
{{ '<|assistant|>' }}
{% endif %}
{% endfor %}"""
QWEN25 = """{%- if tools %}
    {{- '<|im_start|>system\n' }}
    {%- if messages[0]['role'] == 'system' %}
        {{- messages[0]['content'] }}
    {%- else %}
        {{- 'You are Qwen, created by Alibaba Cloud. You are a helpful assistant.' }}
    {%- endif %}
    {{- "\n\n# Tools\n\n<tools>" }}
    {%- for tool in tools %}
        {{- "\n" }}
        {{- tool | tojson }}
    {%- endfor %}
    {{- "\n</tools><|im_end|>\n" }}
{%- else %}
    {%- if messages[0]['role'] == 'system' %}
        {{- '<|im_start|>system\n' + messages[0]['content'] + '<|im_end|>\n' }}
    {%- else %}
        {{- '<|im_start|>system\nYou are Qwen, created by Alibaba Cloud. You are a helpful assistant.<|im_end|>\n' }}
    {%- endif %}
{%- endif %}
{%- for message in messages %}
    {%- if (message.role == "user") or (message.role == "system" and not loop.first) or (message.role == "assistant" and not message.tool_calls) %}
        {{- '<|im_start|>' + message.role + '\n' + message.content + '<|im_end|>' + '\n' }}
    {%- elif message.role == "tool" %}
        {%- if (loop.index0 == 0) or (messages[loop.index0 - 1].role != "tool") %}
            {{- '<|im_start|>user' }}
        {%- endif %}
        {{- '\n<tool_response>\n' }}
        {{- message.content }}
        {{- '\n</tool_response>' }}
        {%- if loop.last or (messages[loop.index0 + 1].role != "tool") %}
            {{- '<|im_end|>\n' }}
        {%- endif %}
    {%- endif %}
{%- endfor %}
{%- if add_generation_prompt %}
    {{- '<|im_start|>assistant\n' }}
{%- endif %}
"""
QWEN3 = """{%- if messages[0].role == 'system' %}
    {{- '<|im_start|>system\n' + messages[0].content + '<|im_end|>\n' }}
{%- endif %}
{%- set ns = namespace(multi_step_tool=true, last_query_index=messages|length - 1) %}
{%- for message in messages[::-1] %}
    {%- set index = (messages|length - 1) - loop.index0 %}
    {%- if ns.multi_step_tool and message.role == "user" and message.content is string and not(message.content.startswith('<tool_response>') and message.content.endswith('</tool_response>')) %}
        {%- set ns.multi_step_tool = false %}
        {%- set ns.last_query_index = index %}
    {%- endif %}
{%- endfor %}
{%- for message in messages %}
    {%- if message.content is string %}
        {%- set content = message.content %}
    {%- else %}
        {%- set content = '' %}
    {%- endif %}
    {%- if (message.role == "user") or (message.role == "system" and not loop.first) %}
        {{- '<|im_start|>' + message.role + '\n' + content + '<|im_end|>' + '\n' }}
    {%- elif message.role == "assistant" %}
        {%- set reasoning_content = '' %}
        {%- if message.reasoning_content is string %}
            {%- set reasoning_content = message.reasoning_content %}
        {%- else %}
            {%- if '</think>' in content %}
                {%- set reasoning_content = content.split('</think>')[0].rstrip('\n').split('<think>')[-1].lstrip('\n') %}
                {%- set content = content.split('</think>')[-1].lstrip('\n') %}
            {%- endif %}
        {%- endif %}
        {%- if loop.index0 > ns.last_query_index %}
            {%- if loop.last or (not loop.last and reasoning_content) %}
                {{- '<|im_start|>' + message.role + '\n<think>\n' + reasoning_content.strip('\n') + '\n</think>\n\n' + content.lstrip('\n') }}
            {%- else %}
                {{- '<|im_start|>' + message.role + '\n' + content }}
            {%- endif %}
        {%- else %}
            {{- '<|im_start|>' + message.role + '\n' + content }}
        {%- endif %}
        {{- '<|im_end|>\n' }}
    {%- endif %}
{%- endfor %}
{%- if add_generation_prompt %}
    {{- '<|im_start|>assistant\n' }}
    {%- if enable_thinking is defined and enable_thinking is false %}
        {{- '<think>\n\n</think>\n\n' }}
    {%- endif %}
{%- endif %}"""
# every construct the interpreter supports, in one template
KITCHEN = """{%- macro fmt(m, prefix='> ') -%}{{ prefix }}{{ m.role | upper }}: {{ m.content | trim }}{%- endmacro -%}
{%- set ns = namespace(n=0) -%}
{%- for m in messages if m.role != 'tool' -%}
  {%- set ns.n = ns.n + 1 -%}
  {{ fmt(m) }}{{ loop.cycle('|', '/') }}{% if not loop.last %}
{% endif %}
{%- else -%}
  no messages
{%- endfor %}
count={{ ns.n }} roles={{ messages | map(attribute='role') | join(',') }}
users={{ messages | selectattr('role', 'equalto', 'user') | list | length }} others={{ messages | rejectattr('role', 'eq', 'user') | list | length }}
{% set block %}{{ bos_token ~ 'x' }}{% endset %}{{ block | replace('x', 'y') }}
{{ {'b': 1, 'a': [1, 2.5, none, true, "q<'&>"]} | tojson }} {{ [3, 'é'] | tojson(indent=2) }}
{{ (messages | first).content[:3] }}|{{ messages[-1]['content'][::-1] }}|{{ messages[1:] | length }}
{{ 'A' if enable_thinking else 'B' }} {{ 7 // 2 }} {{ -7 // 2 }} {{ 7 % 3 }} {{ -7 % 3 }} {{ 2 ** 10 }} {{ 1 / 4 }} {{ 'ab' * 2 }} {{ 3 - 5 }} {{ 1.5 + 1 }}
{%- for i in range(6) %}{% if i == 4 %}{% break %}{% endif %}{% if i is odd %}{% continue %}{% endif %}{{ i }}{% endfor %}
{{ undefined_var | default('dflt') }} {{ undefined_var is defined }} {{ none is none }} {{ '' | default('e', true) }} {{ 3 is divisibleby 3 }}
{{ "  padded  " | trim }}|{{ "a-b-c".split("-") | join("+") }}|{{ "Hello World".lower().title() }}|{{ "x y  z".split() }}|{{ "a,b,c".rsplit(",", 1) }}
{{ "line1\nline2\n\nline4" | indent(2) }}
{% for k, v in {'x': 1, 'y': 2}.items() %}{{ k }}={{ v }};{% endfor %} {{ {'k': 'v'}.get('k') }} {{ {'k': 'v'}.get('z', 'dz') }}
{{ [1, 2] + [3] }} {{ 'b' in ['a', 'b'] }} {{ 'z' not in 'abc' }} {{ [1, 2] == [1, 2] }} {{ 2 < 3 < 4 }} {{ 3 > 2 > 1 }} {{ 1 < 2 > 3 }} {{ not true or false and true }}
{{ messages | length > 1 and messages[0].role }} {{ 1 if 0 else (2 if 1 else 3) }} {{ [3, 1, 2] | reverse | list }} {{ 'abc' | reverse }}
{{ 42 | string ~ '!' }} {{ '12' | int + 1 }} {{ 'x' | int }} {{ 2.0 }} {{ 1e20 }} {{ 0.1 + 0.2 }} {{ [1, 'a', none, true] }} {{ {'a': [1]} }}
{{ "It's" }} {{ 'say "hi"' | e }} {{ messages | map('upper') | list if false else 'mapped' }} {{ [1, 1, 2] | unique | list }}
{{ fmt(messages[0]) + '<&>' }} {{ 'x' ~ ('<'|safe) }} {{ ['a'|safe, 'b'|e, 'c'] }} {{ ('q'|tojson) + '"' }}
{#- a comment -#}
{%+ if true %}kept{% endif %}
  {% if true %}lstripped{% endif %}
end"""
TEMPLATES = [("llama3", LLAMA3), ("mistral", MISTRAL), ("gemma", GEMMA), ("phi3", PHI3), ("zephyr", ZEPHYR),
             ("qwen25", QWEN25), ("qwen3", QWEN3), ("kitchen", KITCHEN), ("none", "")]
CONVS = [
    [{"role": "user", "content": " hello "}],
    [{"role": "user", "content": "a"}, {"role": "assistant", "content": "b"}, {"role": "user", "content": "c"}],
    [{"role": "system", "content": "sys"}, {"role": "user", "content": "q"}],
    [{"role": "user", "content": "q1"}, {"role": "assistant", "content": "<think>\nr1\n</think>\n\na1"},
     {"role": "user", "content": "q2"}, {"role": "assistant", "content": "<think>r2</think>a2"}],
    [{"role": "system", "content": "s"}, {"role": "user", "content": "u"}, {"role": "tool", "content": "t1"},
     {"role": "tool", "content": "t2"}, {"role": "assistant", "content": "x"}],
    [{"role": "user", "content": "naïve ✓ 漢字\nline\ttab"}],
]


@pytest.mark.parametrize("name,template", TEMPLATES)
def test_chat_templates_match_jinja2(exe, tmp_path, name, template):
    """The server's Jinja interpreter renders what the Python server's jinja2 renders (raise_exception
    and unsupported templates fall back to ChatML in both)."""
    tf = tmp_path / "t.jinja"
    tf.write_text(template)
    lines, want = [], []
    for conv in CONVS:
        for gen in (True, False):
            for think in (True, False):
                lines.append(json.dumps({"messages": conv, "add_generation_prompt": gen, "enable_thinking": think,
                                         "bos": "<s>", "eos": "</s>"}))
                want.append(ChatTemplate(template or None, "<s>", "</s>").render(conv, gen, think))
    out = subprocess.run([exe, "--tool", "render-chat", str(tf)], input="\n".join(lines).encode() + b"\n",
                         capture_output=True, check=True).stdout.decode()
    got = [json.loads(x) for x in out.split("\n") if x]
    assert len(got) == len(want)
    for k, (g, w) in enumerate(zip(got, want)):
        assert g == w, (name, k, lines[k], g, w)


def test_server_threads_race_free_under_tsan(tmp_path):
    """The server built with ThreadSanitizer: concurrent plain, streamed, stop-string and abandoned
    requests plus metrics reads while the loop steps; no race may be reported and the process must exit
    cleanly on SIGTERM."""
    exe = str(_build.build_serve_cpu(tsan=True))
    toks, scores, types = spm_vocab()
    path = str(tmp_path / "v.gguf")
    write_vocab_gguf(path, toks, scores, types, [], "llama", "default", 1, 2)
    srv = Server(exe, path, str(tmp_path), "--step-delay-ms", "2", "--max-num-batched-tokens", "64",
                 "--max-num-seqs", "6")
    errors = []

    def client(i):
        try:
            body = {"prompt": "tsan " * (1 + i % 7), "max_tokens": 10 + i, "ignore_eos": True}
            if i % 4 == 0:
                srv.stream("/v1/completions", {**body, "stream": True})
            elif i % 4 == 1:
                srv.post("/v1/chat/completions", {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 8})
            elif i % 4 == 2:
                s = socket.create_connection(("127.0.0.1", srv.port), timeout=10)
                b = json.dumps({**body, "stream": True, "max_tokens": 200}).encode()
                s.sendall(b"POST /v1/completions HTTP/1.1\r\nHost: x\r\nContent-Length: " + str(len(b)).encode() +
                          b"\r\n\r\n" + b)
                s.recv(100)
                s.close()
            else:
                srv.request("GET", "/metrics")
                srv.post("/v1/completions", {**body, "stop": "e"})
        except Exception as e:  # noqa: BLE001
            errors.append(repr(e))
    th = [threading.Thread(target=client, args=(i,)) for i in range(16)]
    for t in th:
        t.start()
    for t in th:
        t.join(120)
    srv.proc.send_signal(2)
    rc = srv.proc.wait(60)
    err = srv.proc.stderr.read().decode()
    assert not errors, errors
    assert "ThreadSanitizer" not in err and rc == 0, err[-4000:]


def test_chat_template_mutations_match_jinja2(exe):
    """Random edits of the template bank (deleted spans, inserted delimiters, operators and keywords):
    whatever jinja2 makes of each broken or altered template (a render, or an error and the ChatML
    fallback), the native interpreter must produce the same prompt."""
    rng = random.Random(2024)
    base = [tm for _, tm in TEMPLATES if tm]
    pieces = ["{%", "%}", "{{", "}}", "-", "+", "(", ")", "[", "]", "'", '"', "|", ".", ":", ",", "~", "*", "\n",
              " ", " if ", " else ", " for ", " in ", " not ", " is ", "endfor", "endif", "loop.", "ns.", "none"]
    lines, want = [], []
    for _ in range(1500):
        s = rng.choice(base)
        for _ in range(rng.randint(1, 4)):
            k = rng.randrange(len(s) + 1)
            if rng.random() < 0.5 and len(s) > 2:
                s = s[:k] + s[k + rng.randint(1, 5):]
            else:
                s = s[:k] + rng.choice(pieces) + s[k:]
        conv = rng.choice(CONVS)
        gen, think = rng.random() < 0.8, rng.random() < 0.5
        lines.append(json.dumps({"template": s, "messages": conv, "add_generation_prompt": gen,
                                 "enable_thinking": think, "bos": "<s>", "eos": "</s>"}))
        want.append(ChatTemplate(s, "<s>", "</s>").render(conv, gen, think))
    out = subprocess.run([exe, "--tool", "render-chat", "-"], input="\n".join(lines).encode() + b"\n",
                         capture_output=True, check=True, timeout=300).stdout.decode()
    got = [json.loads(x) for x in out.split("\n") if x]
    assert len(got) == len(want)
    bad = [k for k in range(len(want)) if got[k] != want[k]]
    assert not bad, [(json.loads(lines[k])["template"][:300], got[k][:200], want[k][:200]) for k in bad[:3]]


@pytest.mark.parametrize("impl", ["native", "python"])
def test_host_bench_runs(impl):
    """The host-path load test (vm_c_b200/server/host_bench.py) drives both servers to completion."""
    import sys
    r = subprocess.run([sys.executable, "-m", "vm_c_b200.server.host_bench", "--impl", impl, "--clients", "4",
                        "--requests", "16", "--max-tokens", "8"], capture_output=True, text=True, timeout=300,
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["errors"] == 0 and out["completion_tokens"] == 16 * 8


def test_host_bench_engine_mode():
    """`host_bench --engine` runs the engine's pipelined path to completion and reports its host cost."""
    from vm_c_b200.server.host_bench import engine_host_cost
    out = engine_host_cost(8, 32, 16, vocab=1000)
    assert out["steps"] >= 16 and out["host_us_per_step"] > 0
    assert 0 < out["gap_wait_to_launch_us_p50"] <= out["gap_wait_to_launch_us_p90"]


def test_streaming_utf8_decoder_matches_python(exe):
    """The native detokenizer's streaming UTF-8 decoder releases, chunk by chunk, what Python's
    incremental decoder (errors="replace") releases: incomplete trailing sequences wait for their next
    byte, ill-formed bytes become U+FFFD at once."""
    import codecs
    rng = random.Random(7)
    pool = [b for ch in "aé✓😀漢" for b in ch.encode()] + [0x80, 0xBF, 0xC0, 0xC2, 0xE0, 0xED, 0xF0, 0xF4, 0xF5, 0xFF]
    cases = []
    for _ in range(400):
        data = [rng.choice(pool) for _ in range(rng.randint(0, 24))]
        cuts = sorted(rng.sample(range(len(data) + 1), min(len(data) + 1, rng.randint(1, 6))))
        chunks, prev = [], 0
        for c in cuts + [len(data)]:
            chunks.append(data[prev:c])
            prev = c
        cases.append(chunks)
    inp = "".join(json.dumps(c) + "\n" for c in cases).encode()
    out = subprocess.run([exe, "--tool", "utf8-stream", "-"], input=inp, capture_output=True, check=True).stdout
    got = [json.loads(x) for x in out.decode().split("\n") if x]
    for chunks, g in zip(cases, got):
        dec = codecs.getincrementaldecoder("utf-8")(errors="replace")
        want = [dec.decode(bytes(c), final=(k + 1 == len(chunks))) for k, c in enumerate(chunks)]
        assert g == want, (chunks, g, want)


def test_cli_native_flag_builds_runtime_command():
    """`vm_c_server --native` hands the options over to `vmc_run --serve` and refuses the ones that
    runtime does not have."""
    from vm_c_b200.cli import build_parser, native_argv
    a = build_parser().parse_args(["m.gguf", "--native", "--port", "9001", "--served-model-name", "x",
                                   "--max-num-seqs", "32", "--max-model-len", "4096"])
    argv = native_argv(a)
    assert argv[0].endswith("vmc_run") and argv[1:3] == ["m.gguf", "--serve"]
    assert argv[argv.index("--port") + 1] == "9001" and argv[argv.index("--model-name") + 1] == "x"
    assert argv[argv.index("--max-num-seqs") + 1] == "32" and argv[argv.index("--max-model-len") + 1] == "4096"
    for extra in (["-tp", "2"], ["--kv-cache-dtype", "turboquant_4bit_nc"], ["--draft-model", "d.gguf"]):
        with pytest.raises(ValueError):
            native_argv(build_parser().parse_args(["m.gguf", "--native"] + extra))


def test_echo_joined_prompts_running_usage_and_no_generation_prompt(spm):
    """Request options of the reference's API: `echo`, a list of prompt strings (one per line),
    `stream_options.continuous_usage_stats` and `add_generation_prompt`."""
    srv, tok = spm
    V = len(tok.tokens)
    st, r = srv.post("/v1/completions", {"prompt": "echo me", "max_tokens": 6, "echo": True, "temperature": 0})
    want, _ = predict(tok.encode("echo me"), V, 6, [2])
    assert st == 200 and r["choices"][0]["text"] == "echo me" + detok(tok, want)[0]
    st, r = srv.post("/v1/completions", {"prompt": ["first", "second"], "max_tokens": 2})
    assert st == 200 and r["usage"]["prompt_tokens"] == len(tok.encode("first\nsecond"))
    ev = srv.stream("/v1/completions", {"prompt": "count", "max_tokens": 9, "ignore_eos": True, "stream": True,
                                        "stream_options": {"continuous_usage_stats": True, "include_usage": True}})
    counts = [e["usage"]["completion_tokens"] for e in ev[:-2] if e.get("usage")]
    assert counts and counts == sorted(counts) and counts[-1] <= 9 and ev[-1]["usage"]["completion_tokens"] == 9
    msgs = [{"role": "user", "content": "hi"}]
    st, r = srv.post("/v1/chat/completions", {"messages": msgs, "max_tokens": 2, "add_generation_prompt": False})
    prompt = chatml(msgs, False, True)
    assert r["usage"]["prompt_tokens"] == len(tok.encode(prompt, add_bos=not prompt.startswith(tok.tokens[1])))


def test_prompt_and_detok_diagnostics(exe, tmp_path):
    """VMC_LOG_PROMPT_VERBOSE / VMC_LOG_DETOK (the reference's request diagnostics) log the prompt with
    its round-trip check and every generated token."""
    toks, scores, types = spm_vocab()
    path = str(tmp_path / "v.gguf")
    write_vocab_gguf(path, toks, scores, types, [], "llama", "default", 1, 2)
    pf = str(tmp_path / "port")
    env = dict(os.environ, VMC_LOG_PROMPT_VERBOSE="1", VMC_LOG_DETOK="1")
    proc = subprocess.Popen([exe, path, "--port", "0", "--port-file", pf], stderr=subprocess.PIPE, env=env)
    try:
        t0 = time.time()
        while not os.path.exists(pf) or not open(pf).read().strip():
            assert proc.poll() is None and time.time() - t0 < 30
            time.sleep(0.02)
        c = http.client.HTTPConnection("127.0.0.1", int(open(pf).read()), timeout=30)
        c.request("POST", "/v1/completions", body=json.dumps({"prompt": "the rain", "max_tokens": 3}))
        assert c.getresponse().status == 200
        c.close()
    finally:
        proc.terminate()
        err = proc.communicate(timeout=30)[1].decode()
    assert "[PROMPT]" in err and "round-trip=Y" in err and "[DETOK]" in err, err


def test_json_parser_matches_python(exe):
    """The native JSON parser and writer against Python's json module: random documents survive the
    round trip unchanged (integers stay exact), and random edits of them are accepted or rejected as
    Python accepts or rejects them (Python's NaN / Infinity extension excluded)."""
    rng = random.Random(11)

    def value(depth):
        k = rng.randrange(8 if depth < 4 else 5)
        if k == 0:
            return None
        if k == 1:
            return rng.random() < 0.5
        if k == 2:
            return rng.randrange(-2 ** 62, 2 ** 62)
        if k == 3:
            return rng.choice([0.5, -1e-300, 1.5e300, 3.141592653589793, -0.0, 2.5e-8])
        if k == 4:
            return "".join(rng.choice(["a", "é", "\\", '"', "\n", "\t", "\x01", "😀", "漢", "/", " "])
                           for _ in range(rng.randrange(8)))
        if k in (5, 6):
            return [value(depth + 1) for _ in range(rng.randrange(4))]
        return {f"k{rng.randrange(5)}{i}": value(depth + 1) for i in range(rng.randrange(4))}

    docs = [json.dumps(value(0), ensure_ascii=rng.random() < 0.5) for _ in range(600)]
    edits = []
    for d in docs[:400]:
        for _ in range(2):
            k = rng.randrange(len(d) + 1)
            e = d[:k] + rng.choice([",", "]", "}", '"', "\\", "{", "[", "1", "e", ".", "-", " ", ":", "tru"]) + d[k + rng.randrange(2):]
            if "\n" not in e:
                edits.append(e)
    lines = docs + edits
    out = subprocess.run([exe, "--tool", "json", "-"], input=("\n".join(lines) + "\n").encode(), capture_output=True,
                         check=True, timeout=120).stdout.decode().split("\n")

    def py(doc):
        try:
            return True, json.loads(doc, parse_constant=lambda c: (_ for _ in ()).throw(ValueError(c)))
        except ValueError:
            return False, None

    def wide(v):  # integers beyond int64 are doubles, lone surrogates U+FFFD in the native model
        if isinstance(v, int) and not isinstance(v, bool) and not -2 ** 63 <= v < 2 ** 63:
            return float(v)
        if isinstance(v, str):
            return v.encode("utf-16-le", "surrogatepass").decode("utf-16-le", "replace")
        if isinstance(v, list):
            return [wide(x) for x in v]
        if isinstance(v, dict):
            return {wide(k): wide(x) for k, x in v.items()}
        return v

    def finite(v):
        if isinstance(v, float):
            return v == v and abs(v) != float("inf")
        if isinstance(v, list):
            return all(finite(x) for x in v)
        if isinstance(v, dict):
            return all(finite(x) for x in v.values())
        return True

    for doc, got in zip(lines, out):
        ok, want = py(doc)
        if not ok:
            assert got.startswith('{"error": '), (doc, got)
        elif finite(want):  # a literal beyond double range: Python keeps infinity, the writer emits null
            assert json.loads(got) == wide(want), (doc, got)
