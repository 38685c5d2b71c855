"""Host-path load test of an OpenAI server: requests/s, streamed completion tokens/s, time to first
token and the gap between streamed chunks, measured at the client.

    # any running server (the native `vmc_run --serve` on a GPU, or the Python server)
    python -m vm_c_b200.server.host_bench --url http://127.0.0.1:8000 --clients 64 --requests 512

    # the two servers' host paths on the CPU, with the same rule instead of a model
    python -m vm_c_b200.server.host_bench --impl native --clients 64 --requests 512
    python -m vm_c_b200.server.host_bench --impl python --clients 64 --requests 512

    # the engine alone (core/engine.py, no HTTP): host time per step and the gap between one step's
    # wait and the next step's launch, where the GPU idles
    python -m vm_c_b200.server.host_bench --engine --clients 64 --prompt-tokens 1024 --max-tokens 256

With --impl, a tokenizer-only GGUF is written and the server is started with a deterministic rule in
place of the model (token after t at position p = (31 t + 7 p + 11) mod V): `vmc_serve_cpu` for the
native server (csrc/server/), and for the Python server (server/http.py) the same engine
(core/engine.py) the GPU path uses, over a runner that applies the rule. What remains is each server's
own per-request and per-token cost: HTTP, JSON, detokenisation, streaming, the serving loop and the
scheduler. Prompts are token ids; every request generates exactly --max-tokens tokens (ignore_eos).
One JSON line on stdout.
"""
from __future__ import annotations

import argparse
import http.client
import json
import os
import subprocess
import sys
import tempfile
import threading
import time
from urllib.parse import urlparse

import numpy as np

RULE = (31, 7, 11)


def write_vocab_gguf(path: str, vocab: int = 32000) -> None:
    """A GGUF holding only a SentencePiece-style vocabulary (no tensors)."""
    from .. import _native
    from ..gguf.constants import VType
    from ..gguf.random_init import synthetic_vocab
    toks, scores, types = synthetic_vocab(vocab)
    w = _native.host().GgufWriter(32)
    for key, vt, val, et in [("general.architecture", VType.STRING, "llama", 0),
                             ("tokenizer.ggml.model", VType.STRING, "llama", 0),
                             ("tokenizer.ggml.tokens", VType.ARRAY, toks, int(VType.STRING)),
                             ("tokenizer.ggml.scores", VType.ARRAY, scores, int(VType.FLOAT32)),
                             ("tokenizer.ggml.token_type", VType.ARRAY, types, int(VType.INT32)),
                             ("tokenizer.ggml.bos_token_id", VType.UINT32, 1, 0),
                             ("tokenizer.ggml.eos_token_id", VType.UINT32, 2, 0)]:
        w.set(key, int(vt), val, int(et))
    w.write(path, lambda i: None)


def serve_python_rule(gguf: str, port: int, max_seqs: int, max_batched: int, max_len: int) -> None:
    """The Python server over the engine with a rule runner (blocks until killed)."""
    from aiohttp import web

    from ..config import ServerConfig, VmCConfig
    from ..core.engine import LLMEngine, ModelRunner
    from ..gguf.reader import GgufSource
    from .http import OpenAIServer, cors
    from .tokenizer import Tokenizer

    tok = Tokenizer.from_gguf(GgufSource(gguf))
    V = tok.vocab_size

    class RuleRunner(ModelRunner):
        def __init__(self):
            self.num_kv_blocks = max_seqs * (max_len // 16 + 1) + 1
            self.max_model_len = max_len

        def bind_layout(self, layout):
            self.layout = layout

        def execute(self, meta, counts, params, penalties=None):
            L = self.layout
            lidx = meta[L.off_logits_idx:L.off_logits_idx + counts.S]
            ids = meta[L.off_input_ids + lidx].astype(np.int64)
            pos = meta[L.off_positions + lidx].astype(np.int64)
            a, b, c = RULE
            return ((a * ids + b * pos + c) % V).astype(np.int32), np.zeros(counts.S, np.float32)

    cfg = VmCConfig()
    cfg.model.vocab = V
    cfg.model.max_model_len = max_len
    cfg.model.eos_token_ids = list(tok.eos_ids)
    cfg.scheduler.max_num_seqs = max_seqs
    cfg.scheduler.max_num_batched_tokens = max_batched
    cfg.finalize()
    eng = LLMEngine(cfg, RuleRunner())
    srv = OpenAIServer(eng, tok, "vm_c", ServerConfig())
    srv.app.middlewares.append(cors)
    web.run_app(srv.app, host="127.0.0.1", port=port, print=lambda *a: None)


def engine_host_cost(seqs: int, prompt_tokens: int, max_tokens: int, vocab: int = 32000) -> dict:
    """LLMEngine.generate over a runner that applies the rule in launch / wait form (the pipelined
    path the GPU runner takes): wall time per step and the host gap between a step's wait and the next
    launch, which on a GPU is device idle time."""
    from ..config import VmCConfig
    from ..core.engine import LLMEngine, ModelRunner
    from ..core.sampling_params import SamplingParams
    a, b, c = RULE
    max_len = prompt_tokens + max_tokens + 16

    class PipelinedRule(ModelRunner):
        def __init__(self):
            self.num_kv_blocks = seqs * (max_len // 16 + 1) + 1
            self.max_model_len = max_len
            self.gaps, self.t_wait = [], None

        def bind_layout(self, layout):
            self.layout = layout

        def graph_bucket(self, n):
            return n

        def launch(self, meta, counts, params, penalties=None):
            if self.t_wait is not None:
                self.gaps.append(time.perf_counter() - self.t_wait)
            L = self.layout
            lidx = meta[L.off_logits_idx:L.off_logits_idx + counts.S]
            ids = meta[L.off_input_ids + lidx].astype(np.int64)
            pos = meta[L.off_positions + lidx].astype(np.int64)
            return ((a * ids + b * pos + c) % vocab).astype(np.int32), np.zeros(counts.S, np.float32)

        def wait(self, handle):
            self.t_wait = time.perf_counter()
            return handle

        def execute(self, *args):
            return self.wait(self.launch(*args))

    cfg = VmCConfig()
    cfg.model.vocab = vocab
    cfg.model.max_model_len = max_len
    cfg.model.eos_token_ids = [2]
    cfg.scheduler.max_num_seqs = seqs
    cfg.scheduler.max_num_batched_tokens = 2048
    cfg.finalize()
    runner = PipelinedRule()
    eng = LLMEngine(cfg, runner)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(3, vocab, prompt_tokens).tolist() for _ in range(seqs)]
    t0 = time.perf_counter()
    eng.generate(prompts, SamplingParams(temperature=0.8, top_k=40, max_tokens=max_tokens, ignore_eos=True))
    wall = time.perf_counter() - t0
    g = np.array(runner.gaps[len(runner.gaps) // 8:]) * 1e6  # decode steps (after the prefill chunks)
    return {"engine": "core/engine.py (pipelined launch / wait)", "seqs": seqs, "prompt_tokens": prompt_tokens,
            "max_tokens": max_tokens, "steps": eng.step_id, "host_us_per_step": round(wall / eng.step_id * 1e6, 1),
            "gap_wait_to_launch_us_p50": round(float(np.median(g)), 1),
            "gap_wait_to_launch_us_p90": round(float(np.percentile(g, 90)), 1)}


def _free_port() -> int:
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _wait_ready(host: str, port: int, proc: subprocess.Popen, timeout_s: float = 60) -> None:
    t0 = time.time()
    while time.time() - t0 < timeout_s:
        if proc.poll() is not None:
            raise RuntimeError(f"server exited with {proc.returncode}")
        try:
            c = http.client.HTTPConnection(host, port, timeout=2)
            c.request("GET", "/health")
            if c.getresponse().status == 200:
                c.close()
                return
        except OSError:
            pass
        time.sleep(0.1)
    raise RuntimeError("server did not become ready")


def run_load(host: str, port: int, clients: int, requests: int, prompt_tokens: int, max_tokens: int,
             stream: bool, vocab: int = 32000) -> dict:
    rng = np.random.default_rng(0)
    prompts = [rng.integers(3, min(vocab, 30000), prompt_tokens).tolist() for _ in range(requests)]
    lock = threading.Lock()
    nxt = [0]
    ttft, gaps, lat, toks, errors = [], [], [], [0], []

    def worker():
        c = http.client.HTTPConnection(host, port, timeout=300)
        while True:
            with lock:
                i = nxt[0]
                nxt[0] += 1
            if i >= requests:
                break
            body = {"prompt": prompts[i], "max_tokens": max_tokens, "ignore_eos": True, "temperature": 0,
                    "stream": stream, "stream_options": {"include_usage": True}}
            t0 = time.perf_counter()
            try:
                c.request("POST", "/v1/completions", body=json.dumps(body),
                          headers={"Content-Type": "application/json"})
                r = c.getresponse()
                if not stream:
                    j = json.loads(r.read())
                    n = j["usage"]["completion_tokens"]
                    t_first = None
                    my_gaps = []
                else:
                    n, t_first, last, my_gaps = 0, None, None, []
                    buf = b""
                    while True:
                        chunk = r.read1(65536) if hasattr(r, "read1") else r.read(65536)
                        if not chunk:
                            break
                        now = time.perf_counter()
                        buf += chunk
                        while b"\n\n" in buf:
                            ev, buf = buf.split(b"\n\n", 1)
                            if not ev.startswith(b"data: ") or ev == b"data: [DONE]":
                                continue
                            d = json.loads(ev[6:])
                            if d.get("usage"):
                                n = d["usage"]["completion_tokens"]
                            if d.get("choices") and d["choices"][0].get("text"):
                                if t_first is None:
                                    t_first = now - t0
                                elif last is not None:
                                    my_gaps.append(now - last)
                                last = now
                    c.close()
                    c = http.client.HTTPConnection(host, port, timeout=300)
                dt = time.perf_counter() - t0
                with lock:
                    lat.append(dt)
                    toks[0] += n
                    if t_first is not None:
                        ttft.append(t_first)
                    gaps.extend(my_gaps)
            except Exception as e:  # noqa: BLE001  (reported, not raised: the run continues)
                with lock:
                    errors.append(repr(e))
                c.close()
                c = http.client.HTTPConnection(host, port, timeout=300)
        c.close()

    t0 = time.perf_counter()
    th = [threading.Thread(target=worker) for _ in range(clients)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    wall = time.perf_counter() - t0

    def pct(xs, p):
        return float(np.percentile(xs, p) * 1e3) if xs else None

    return {"requests": requests, "clients": clients, "prompt_tokens": prompt_tokens, "max_tokens": max_tokens,
            "stream": stream, "wall_s": round(wall, 3), "requests_per_s": round(requests / wall, 1),
            "completion_tokens_per_s": round(toks[0] / wall, 1), "completion_tokens": toks[0],
            "p50_latency_ms": pct(lat, 50), "p50_ttft_ms": pct(ttft, 50), "p50_chunk_gap_ms": pct(gaps, 50),
            "p99_chunk_gap_ms": pct(gaps, 99), "errors": len(errors), "first_error": errors[0] if errors else None}


def main() -> None:
    ap = argparse.ArgumentParser()
    g = ap.add_mutually_exclusive_group(required=True)
    g.add_argument("--url", help="load-test a running server")
    g.add_argument("--impl", choices=["native", "python"], help="start this server over the rule backend")
    g.add_argument("--engine", action="store_true", help="time the engine's host path alone (no HTTP)")
    g.add_argument("--serve-python", metavar="GGUF", help=argparse.SUPPRESS)
    ap.add_argument("--port", type=int, default=0)
    ap.add_argument("--clients", type=int, default=64)
    ap.add_argument("--requests", type=int, default=512)
    ap.add_argument("--prompt-tokens", type=int, default=64)
    ap.add_argument("--max-tokens", type=int, default=128)
    ap.add_argument("--no-stream", action="store_true")
    ap.add_argument("--max-num-seqs", type=int, default=64)
    ap.add_argument("--max-num-batched-tokens", type=int, default=2048)
    ap.add_argument("--max-model-len", type=int, default=1024)
    a = ap.parse_args()
    if a.engine:
        print(json.dumps(engine_host_cost(a.clients, a.prompt_tokens, a.max_tokens)), flush=True)
        return
    if a.serve_python:
        serve_python_rule(a.serve_python, a.port, a.max_num_seqs, a.max_num_batched_tokens, a.max_model_len)
        return
    if a.url:
        u = urlparse(a.url)
        out = run_load(u.hostname, u.port or 80, a.clients, a.requests, a.prompt_tokens, a.max_tokens,
                       not a.no_stream)
        out["server"] = a.url
        print(json.dumps(out), flush=True)
        return
    with tempfile.TemporaryDirectory() as d:
        gguf = os.path.join(d, "vocab.gguf")
        write_vocab_gguf(gguf)
        port = a.port or _free_port()
        limits = ["--max-num-seqs", str(a.max_num_seqs), "--max-num-batched-tokens", str(a.max_num_batched_tokens),
                  "--max-model-len", str(a.max_model_len)]
        if a.impl == "native":
            from .._build import build_serve_cpu
            cmd = [str(build_serve_cpu()), gguf, "--port", str(port)] + limits
        else:
            cmd = [sys.executable, "-m", "vm_c_b200.server.host_bench", "--serve-python", gguf, "--port", str(port)] + limits
        proc = subprocess.Popen(cmd, stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL,
                                cwd=os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
        try:
            _wait_ready("127.0.0.1", port, proc)
            out = run_load("127.0.0.1", port, a.clients, a.requests, a.prompt_tokens, a.max_tokens, not a.no_stream)
        finally:
            proc.terminate()
            try:
                proc.wait(20)
            except subprocess.TimeoutExpired:
                proc.kill()
                proc.wait()
        out["server"] = {"native": "vmc_serve_cpu (csrc/server, rule backend)",
                         "python": "server/http.py + core/engine.py (rule runner)"}[a.impl]
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
