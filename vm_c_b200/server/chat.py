"""Chat prompt construction and reasoning-content split.

Same behaviour as the reference's HttpServer::build_chat_prompt (src/server/http_server.cpp:278-313):
render the checkpoint's Jinja chat template (tokenizer.chat_template) when present, otherwise a
ChatML prompt; the generation prompt opens a ``<think>`` block when thinking is enabled and inserts
an empty one when it is disabled. The reasoning split follows src/main.cpp:640-661: text before
``</think>`` is reasoning_content, the rest (leading newlines stripped) is content.
"""
from __future__ import annotations

from typing import Optional

THINK_END = "</think>"


def chatml(messages: list[dict], add_generation_prompt: bool = True, enable_thinking: bool = True) -> str:
    out = []
    for m in messages:
        role = m.get("role", "user")
        if role in ("system", "user", "assistant", "tool"):
            out.append(f"<|im_start|>{role}\n{_content(m)}<|im_end|>\n")
    if add_generation_prompt:
        out.append("<|im_start|>assistant\n")
        out.append("<think>\n" if enable_thinking else "<think>\n\n</think>\n\n")
    return "".join(out)


def _content(m: dict) -> str:
    c = m.get("content", "")
    if isinstance(c, list):  # OpenAI content parts
        return "".join(p.get("text", "") for p in c if isinstance(p, dict))
    return c or ""


class ChatTemplate:
    def __init__(self, template: Optional[str], bos_token: str = "", eos_token: str = ""):
        self.source = template
        self.bos, self.eos = bos_token, eos_token
        self._tmpl = None
        if template:
            try:
                import jinja2
                from jinja2.sandbox import ImmutableSandboxedEnvironment
                env = ImmutableSandboxedEnvironment(trim_blocks=True, lstrip_blocks=True,
                                                    extensions=["jinja2.ext.loopcontrols"],
                                                    undefined=jinja2.Undefined)

                def raise_exception(msg):
                    raise jinja2.exceptions.TemplateError(msg)
                env.globals["raise_exception"] = raise_exception
                self._tmpl = env.from_string(template)
            except Exception:  # an unusable template falls back to ChatML (as the reference does)
                self._tmpl = None

    def render(self, messages: list[dict], add_generation_prompt: bool = True, enable_thinking: bool = True) -> str:
        if self._tmpl is not None:
            try:
                msgs = [{"role": m.get("role", "user"), "content": _content(m)} for m in messages]
                s = self._tmpl.render(messages=msgs, add_generation_prompt=add_generation_prompt,
                                      enable_thinking=enable_thinking, bos_token=self.bos, eos_token=self.eos)
                if s:
                    return s
            except Exception:
                pass
        return chatml(messages, add_generation_prompt, enable_thinking)


def split_reasoning(text: str, enable_thinking: bool) -> tuple[str, str]:
    """(reasoning_content, content) of a complete completion."""
    if not enable_thinking:
        return "", text
    k = text.find(THINK_END)
    if k < 0:
        return "", text
    return text[:k], text[k + len(THINK_END):].lstrip("\r\n")


class ReasoningStream:
    """Routes streamed deltas to reasoning_content until ``</think>`` is seen, then to content."""

    def __init__(self, enable_thinking: bool):
        self.in_reasoning = enable_thinking
        self.pending = ""
        self.after_end = False

    def feed(self, delta: str) -> tuple[str, str]:
        if not self.in_reasoning:
            if self.after_end:
                delta = delta.lstrip("\r\n")
                if delta:
                    self.after_end = False
            return "", delta
        self.pending += delta
        k = self.pending.find(THINK_END)
        if k >= 0:
            reasoning, rest = self.pending[:k], self.pending[k + len(THINK_END):]
            self.pending = ""
            self.in_reasoning = False
            rest = rest.lstrip("\r\n")
            self.after_end = not rest
            return reasoning, rest
        # keep a possible partial "</think>" at the end
        keep = 0
        for n in range(1, len(THINK_END)):
            if self.pending.endswith(THINK_END[:n]):
                keep = n
        out, self.pending = self.pending[:len(self.pending) - keep], self.pending[len(self.pending) - keep:]
        return out, ""
