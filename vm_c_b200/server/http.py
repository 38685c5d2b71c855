"""OpenAI-compatible HTTP server (aiohttp) in front of the engine.

Routes and JSON / SSE shapes follow the reference's HttpServer (src/server/http_server.cpp:316-449):
POST /v1/chat/completions, POST /v1/completions, GET /v1/models, GET /health, GET /version,
POST /tokenize, POST /detokenize; streaming chunks end with ``data: [DONE]``;
``stream_options.include_usage`` adds a usage chunk; reasoning text before ``</think>`` is returned
as ``reasoning_content``. Added: GET /metrics (Prometheus text). A request whose client disconnects
is aborted.

Threading: the engine steps on one dedicated thread (EngineLoop); HTTP handlers submit requests
through the engine's locked intake queue and receive tokens through per-request asyncio queues.
This replaces the reference's shared-state design where HTTP threads mutate scheduler queues
directly (src/main.cpp:617,778 -> src/core/scheduler.cpp:451-468).
"""
from __future__ import annotations

import asyncio
import json
import os
import threading
import time
import uuid
from typing import Any, Optional

from aiohttp import web

from ..core.sampling_params import FinishReason, SamplingParams
from ..utils.logging import get_logger
from .chat import ChatTemplate, ReasoningStream, split_reasoning
from .tokenizer import IncrementalDetokenizer, Tokenizer

log = get_logger("server")
VERSION = "vm_c_b200 0.1.0"
# Request diagnostics (the reference's env switches, src/main.cpp:527-570, 673-700):
# VMC_LOG_PROMPT_VERBOSE=1 logs each prompt in full with its token ids and whether detokenising them
# gives the prompt back; VMC_LOG_DETOK=1 logs every generated token's id and text when a request ends.
_LOG_PROMPT = os.environ.get("VMC_LOG_PROMPT_VERBOSE", "") == "1"
_LOG_DETOK = os.environ.get("VMC_LOG_DETOK", "") == "1"


class EngineLoop(threading.Thread):
    """Steps the engine whenever it has work; sleeps on a condition variable otherwise."""

    def __init__(self, engine, poll_s: float = 0.01, driver=None, step_timeout_s: float = 120.0):
        super().__init__(daemon=True, name="engine-loop")
        self.engine = engine
        self.poll_s = poll_s
        self.driver = driver          # multi-rank driver (broadcasts commands before each step)
        self.cv = threading.Condition()
        self.stop_flag = False
        self.error: Optional[BaseException] = None
        self.failed = False           # a rank failed: the server answers 503 from now on
        from ..parallel.health import StepWatchdog
        self.watchdog = StepWatchdog(step_timeout_s, self._step_timeout) if step_timeout_s > 0 else None

    def _step_timeout(self, step: int, dt: float) -> None:
        log.error("engine step %d stuck for %.1f s; in-flight requests will be failed when it returns", step, dt)

    def wake(self) -> None:
        with self.cv:
            self.cv.notify()

    def run(self) -> None:
        from ..parallel.health import RankFailure
        while not self.stop_flag:
            try:
                if self.watchdog is not None:
                    self.watchdog.begin(self.engine.step_id)
                if self.driver is not None:
                    self.driver.step()
                    continue
                if self.engine.has_unfinished():
                    self.engine.step()
                else:
                    with self.cv:
                        self.cv.wait(self.poll_s)
            except RankFailure as e:  # a peer rank is gone: no further collective can complete
                log.error("stopping the engine: %s", e)
                self.error, self.failed = e, True
                n = self.engine.fail_all(FinishReason.ERROR)
                log.error("failed %d in-flight requests", n)
                break
            except Exception as e:  # keep serving; fail the in-flight requests
                log.exception("engine step failed: %s", e)
                self.error = e
                self.engine.fail_all(FinishReason.ERROR)
                time.sleep(0.1)
            finally:
                if self.watchdog is not None:
                    self.watchdog.end()

    def shutdown(self) -> None:
        self.stop_flag = True
        if self.watchdog is not None:
            self.watchdog.stop()
        self.wake()


def _sampling_from(body: dict, default_max: int) -> SamplingParams:
    # An HTTP request samples with temperature 1, top-p 1 and no top-k unless it says otherwise (the
    # OpenAI defaults, as the reference's parse_chat_request / parse_completion_request apply them:
    # src/server/http_server.cpp:157-162, 236-241), not with the offline SamplingParams defaults.
    sp = SamplingParams(temperature=1.0, top_p=1.0, top_k=0)
    sp.max_tokens = int(body.get("max_completion_tokens") or body.get("max_tokens") or default_max)
    for k in ("temperature", "top_p", "min_p", "repetition_penalty", "frequency_penalty", "presence_penalty"):
        if body.get(k) is not None:
            setattr(sp, k, float(body[k]))
    if body.get("top_k") is not None:
        sp.top_k = int(body["top_k"])
    stop = body.get("stop")
    sp.stop = [stop] if isinstance(stop, str) else list(stop or [])
    sp.stop_token_ids = [int(x) for x in body.get("stop_token_ids") or []]
    sp.ignore_eos = bool(body.get("ignore_eos", False))
    sp.min_tokens = int(body.get("min_tokens", 0))
    if body.get("seed") is not None:
        sp.seed = int(body["seed"])
    kw = body.get("chat_template_kwargs") or {}
    et = kw.get("enable_thinking", body.get("enable_thinking"))
    if et is not None:
        sp.enable_thinking = bool(et)
    sp.logprobs = bool(body.get("logprobs", False))
    return sp


class OpenAIServer:
    def __init__(self, engine, tokenizer: Tokenizer, model_name: str, server_cfg, driver=None):
        self.engine = engine
        self.tok = tokenizer
        self.name = model_name
        self.cfg = server_cfg
        self.fingerprint = server_cfg.system_fingerprint or f"fp_{uuid.uuid4().hex[:10]}"
        bos = tokenizer.tokens[tokenizer.bos_id] if 0 <= tokenizer.bos_id < tokenizer.vocab_size else ""
        eos = tokenizer.tokens[tokenizer.eos_ids[0]] if tokenizer.eos_ids else ""
        self.template = ChatTemplate(tokenizer.chat_template, bos, eos)
        self.loop_thread = EngineLoop(engine, server_cfg.step_interval_ms / 1000.0, driver)
        self.app = web.Application()
        self.app.router.add_post("/v1/chat/completions", self.chat)
        self.app.router.add_post("/v1/completions", self.completions)
        self.app.router.add_get("/v1/models", self.models)
        self.app.router.add_get("/health", self.health)
        self.app.router.add_get("/version", self.version)
        self.app.router.add_post("/tokenize", self.tokenize)
        self.app.router.add_post("/detokenize", self.detokenize)
        self.app.router.add_get("/metrics", self.metrics)
        self.app.on_startup.append(self._start)
        self.app.on_cleanup.append(self._stop)

    async def _start(self, app) -> None:
        if not self.loop_thread.is_alive():
            self.loop_thread.start()

    async def _stop(self, app) -> None:
        self.loop_thread.shutdown()

    # -- helpers ---------------------------------------------------------------------------------
    @staticmethod
    def _err(status: int, msg: str, typ: str = "invalid_request_error") -> web.Response:
        return web.json_response({"error": {"message": msg, "type": typ, "code": status}}, status=status)

    def _submit(self, ids: list[int], sp: SamplingParams):
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()

        def cb(req, toks, finished):
            loop.call_soon_threadsafe(q.put_nowait, (list(toks), finished, req.finish_reason))
        rid = f"cmpl-{uuid.uuid4().hex}"
        self.engine.add_request(ids, sp, request_id=rid, stream_callback=cb)
        self.loop_thread.wake()
        return rid, q

    def _log_prompt(self, prompt: str, ids: list[int]) -> None:
        if _LOG_PROMPT:
            back = self.tok.decode(ids)  # special tokens (BOS) do not count
            log.info("[PROMPT] %d tokens first5=%s last5=%s round-trip=%s text=%r", len(ids), ids[:5], ids[-5:],
                     "Y" if back.lstrip() == prompt.lstrip() else "N", prompt)

    async def _generate(self, ids, sp, detok, on_delta=None):
        """Drive one request; returns (text, n_tokens, finish_reason)."""
        rid, q = self._submit(ids, sp)
        n = 0
        out_ids: list[int] = []
        text = []
        reason = None
        try:
            while True:
                toks, finished, fr = await q.get()
                while not finished and not q.empty():  # the engine ran ahead: take everything queued
                    more, finished, fr = q.get_nowait()
                    toks = toks + more
                n += len(toks)
                if _LOG_DETOK:
                    out_ids += toks
                delta = detok.push(toks, final=finished)
                if detok.stopped:  # a stop string ends the request even when its last token hit a limit
                    if not finished:
                        self.engine.finish_request(rid, FinishReason.STOP)
                    finished, fr = True, FinishReason.STOP
                if delta:
                    text.append(delta)
                    if on_delta:
                        await on_delta(delta, n)
                if finished:
                    reason = fr
                    if _LOG_DETOK:
                        log.info("[DETOK] %s: %s", rid, [(t, self.tok.decode([t], skip_special=False)) for t in out_ids])
                    break
        except (asyncio.CancelledError, ConnectionResetError):
            self.engine.abort_request(rid)
            raise
        return "".join(text), n, reason

    # -- routes ----------------------------------------------------------------------------------
    async def chat(self, request: web.Request) -> web.StreamResponse:
        try:
            body = await request.json()
        except json.JSONDecodeError:
            return self._err(400, "invalid JSON body")
        msgs = body.get("messages")
        if not isinstance(msgs, list) or not msgs:
            return self._err(400, "messages must be a non-empty list")
        sp = _sampling_from(body, self.cfg.default_max_tokens)
        prompt = self.template.render(msgs, bool(body.get("add_generation_prompt", True)), sp.enable_thinking)
        ids = self.tok.encode(prompt, add_bos=not prompt.startswith(self.tok.tokens[self.tok.bos_id])
                              if 0 <= self.tok.bos_id < self.tok.vocab_size else False)
        self._log_prompt(prompt, ids)
        try:
            self._validate(ids)
        except ValueError as e:
            return self._err(400, str(e))
        created = int(time.time())
        cid = f"chatcmpl-{uuid.uuid4().hex}"
        detok = IncrementalDetokenizer(self.tok, sp.stop)
        base = {"id": cid, "created": created, "model": self.name, "system_fingerprint": self.fingerprint}
        if not body.get("stream"):
            text, n, reason = await self._generate(ids, sp, detok)
            reasoning, content = split_reasoning(text, sp.enable_thinking)
            if body.get("echo"):
                content = prompt + content
            msg: dict[str, Any] = {"role": "assistant", "content": content}
            if reasoning:
                msg["reasoning_content"] = reasoning
            return web.json_response({**base, "object": "chat.completion",
                                      "choices": [{"index": 0, "message": msg,
                                                   "finish_reason": (reason or FinishReason.STOP).openai}],
                                      "usage": {"prompt_tokens": len(ids), "completion_tokens": n,
                                                "total_tokens": len(ids) + n}})
        resp = await self._sse_start(request)
        rs = ReasoningStream(sp.enable_thinking)
        chunk = {**base, "object": "chat.completion.chunk"}
        so = body.get("stream_options") or {}
        running_usage = bool(so.get("continuous_usage_stats"))

        async def send(delta_obj, finish=None, n_out=None):
            c = {**chunk, "choices": [{"index": 0, "delta": delta_obj, "finish_reason": finish}]}
            if n_out is not None:
                c["usage"] = {"prompt_tokens": len(ids), "completion_tokens": n_out, "total_tokens": len(ids) + n_out}
            await self._sse(resp, c)

        await send({"role": "assistant", "content": ""})

        async def on_delta(d, n_out):
            r, c = rs.feed(d)
            u = n_out if running_usage else None
            if r:
                await send({"reasoning_content": r}, n_out=u)
            if c:
                await send({"content": c}, n_out=u)

        text, n, reason = await self._generate(ids, sp, detok, on_delta)
        await send({}, (reason or FinishReason.STOP).openai)
        if so.get("include_usage"):
            await self._sse(resp, {**chunk, "choices": [], "usage": {"prompt_tokens": len(ids), "completion_tokens": n,
                                                                     "total_tokens": len(ids) + n}})
        await resp.write(b"data: [DONE]\n\n")
        await resp.write_eof()
        return resp

    async def completions(self, request: web.Request) -> web.StreamResponse:
        try:
            body = await request.json()
        except json.JSONDecodeError:
            return self._err(400, "invalid JSON body")
        prompt = body.get("prompt", "")
        if isinstance(prompt, list):
            if prompt and isinstance(prompt[0], int):
                ids = [int(x) for x in prompt]
                prompt = self.tok.decode(ids, skip_special=False)
            else:  # several prompt strings form one prompt, one per line (as the reference joins them)
                prompt = "\n".join(str(p) for p in prompt)
                ids = self.tok.encode(prompt)
        else:
            ids = self.tok.encode(prompt)
        sp = _sampling_from(body, self.cfg.default_completion_max_tokens)
        self._log_prompt(prompt, ids)
        try:
            self._validate(ids)
        except ValueError as e:
            return self._err(400, str(e))
        base = {"id": f"cmpl-{uuid.uuid4().hex}", "created": int(time.time()), "model": self.name,
                "system_fingerprint": self.fingerprint, "object": "text_completion"}
        detok = IncrementalDetokenizer(self.tok, sp.stop)
        if not body.get("stream"):
            text, n, reason = await self._generate(ids, sp, detok)
            if body.get("echo"):
                text = prompt + text
            return web.json_response({**base, "choices": [{"index": 0, "text": text, "logprobs": None,
                                                           "finish_reason": (reason or FinishReason.STOP).openai}],
                                      "usage": {"prompt_tokens": len(ids), "completion_tokens": n,
                                                "total_tokens": len(ids) + n}})
        resp = await self._sse_start(request)
        # every delta chunk is the same JSON around its text: serialise the rest once
        head, tail = json.dumps({**base, "choices": [{"index": 0, "text": "\x00", "logprobs": None,
                                                      "finish_reason": None}]}).split('"\\u0000"')
        head, tail = ("data: " + head).encode(), (tail + "\n\n").encode()
        so = body.get("stream_options") or {}
        running_usage = bool(so.get("continuous_usage_stats"))

        async def on_delta(d, n_out):
            if running_usage:
                await self._sse(resp, {**base, "choices": [{"index": 0, "text": d, "logprobs": None, "finish_reason": None}],
                                       "usage": {"prompt_tokens": len(ids), "completion_tokens": n_out,
                                                 "total_tokens": len(ids) + n_out}})
            else:
                await resp.write(head + json.dumps(d).encode() + tail)
        text, n, reason = await self._generate(ids, sp, detok, on_delta)
        await self._sse(resp, {**base, "choices": [{"index": 0, "text": "", "logprobs": None,
                                                    "finish_reason": (reason or FinishReason.STOP).openai}]})
        if so.get("include_usage"):
            await self._sse(resp, {**base, "choices": [], "usage": {"prompt_tokens": len(ids), "completion_tokens": n,
                                                                    "total_tokens": len(ids) + n}})
        await resp.write(b"data: [DONE]\n\n")
        await resp.write_eof()
        return resp

    def _validate(self, ids: list[int]) -> None:
        if not ids:
            raise ValueError("empty prompt")
        V = self.engine.cfg.model.vocab
        if max(ids) >= V or min(ids) < 0:
            raise ValueError("prompt contains token ids outside the model vocabulary")

    async def models(self, request):
        t = int(time.time())
        perm = {"id": f"modelperm-{uuid.uuid4().hex[:24]}", "object": "model_permission", "created": t,
                "allow_create_engine": False, "allow_sampling": True, "allow_logprobs": True,
                "allow_search_indices": False, "allow_view": True, "allow_fine_tuning": False, "organization": "*",
                "group": None, "is_blocking": False}
        return web.json_response({"object": "list", "data": [{"id": self.name, "object": "model", "created": t,
                                                              "owned_by": "vm_c", "root": self.name,
                                                              "permission": [perm]}]})

    async def health(self, request):
        if self.loop_thread.error is not None:
            return web.json_response({"status": "error", "error": str(self.loop_thread.error)}, status=503)
        return web.json_response({"status": "ok"})

    async def version(self, request):
        return web.json_response({"version": VERSION})

    async def tokenize(self, request):
        body = await request.json()
        text = body.get("text", body.get("content", body.get("prompt", "")))  # "text": the reference's field
        ids = self.tok.encode(text, add_bos=bool(body.get("add_special", False)))
        return web.json_response({"tokens": ids})

    async def detokenize(self, request):
        body = await request.json()
        text = self.tok.decode(body.get("tokens", []), skip_special=False)
        return web.json_response({"text": text, "content": text})  # "text" as the reference answers

    async def metrics(self, request):
        m = self.engine.metrics.prometheus()
        m += f"vmc_num_running {self.engine.num_running}\nvmc_num_waiting {self.engine.num_waiting}\n"
        return web.Response(text=m, content_type="text/plain")

    @staticmethod
    async def _sse_start(request) -> web.StreamResponse:
        resp = web.StreamResponse(headers={"Content-Type": "text/event-stream", "Cache-Control": "no-cache",
                                           "Access-Control-Allow-Origin": "*"})
        await resp.prepare(request)
        return resp

    @staticmethod
    async def _sse(resp, obj) -> None:
        await resp.write(b"data: " + json.dumps(obj).encode() + b"\n\n")


@web.middleware
async def cors(request, handler):
    if request.method == "OPTIONS":
        resp = web.Response()
    else:
        resp = await handler(request)
    resp.headers.setdefault("Access-Control-Allow-Origin", "*")
    resp.headers.setdefault("Access-Control-Allow-Methods", "GET, POST, OPTIONS")
    resp.headers.setdefault("Access-Control-Allow-Headers", "*")
    return resp


def serve(server: OpenAIServer, host: str, port: int) -> None:
    server.app.middlewares.append(cors)
    web.run_app(server.app, host=host, port=port, print=lambda *a: log.info(*a))
