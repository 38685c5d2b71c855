"""Tokenizer and incremental detokenizer built from a GGUF vocabulary.

Covers the reference's tokenizer stack: GgufTokenizer (src/tokenizer/gguf_tokenizer.cpp:39; GPT-2
byte-level BPE) and the llama_vocab tokenizer it switches to at run time (src/main.cpp:15-73,
496-513; SentencePiece-BPE with byte fallback for "llama" vocabularies), and the incremental
detokenizer with stop strings (include/vm_c/tokenizer/incremental_detokenizer.hpp:11-55). The
merge loops run in C++ (csrc/host/tokenizer.cpp); pre-tokenisation, special-token splitting and
byte mapping are here.
"""
from __future__ import annotations

import codecs
import functools
from typing import Iterable, Optional

import regex

from .. import _native

# Pre-tokeniser patterns (public tokenizer definitions).
_PRE = {
    "gpt2": r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+""",
    "llama-bpe": (r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*"""
                  r"""|\s*[\r\n]+|\s+(?!\S)|\s+"""),
    "qwen2": (r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*"""
              r"""|\s*[\r\n]+|\s+(?!\S)|\s+"""),
    # Qwen3.5 vocabularies: combining marks (\p{M}) belong to words
    "qwen35": (r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?[\p{L}\p{M}]+|\p{N}| ?[^\s\p{L}\p{M}\p{N}]+[\r\n]*"""
               r"""|\s*[\r\n]+|\s+(?!\S)|\s+"""),
}
# tokenizer.ggml.pre names that use one of the expressions above (GGUF vocabulary convention)
_PRE_ALIAS = {"llama3": "llama-bpe", "llama-v3": "llama-bpe", "falcon3": "llama-bpe", "falcon-h1": "llama-bpe",
              "pixtral": "llama-bpe", "dbrx": "llama-bpe", "smaug-bpe": "llama-bpe", "deepseek-r1-qwen": "qwen2",
              "gpt-2": "gpt2", "phi-2": "gpt2"}


def pre_family(pre: str) -> str:
    """The pre-tokeniser expression a vocabulary's tokenizer.ggml.pre names (unknown names: gpt2)."""
    pre = _PRE_ALIAS.get(pre, pre)
    return pre if pre in _PRE else "gpt2"

TOKEN_NORMAL, TOKEN_UNKNOWN, TOKEN_CONTROL, TOKEN_USER, TOKEN_UNUSED, TOKEN_BYTE = 1, 2, 3, 4, 5, 6


@functools.lru_cache(maxsize=1)
def _byte_unicode() -> tuple[dict[int, str], dict[str, int]]:
    """GPT-2's reversible byte <-> printable code point mapping."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + \
        list(range(ord("®"), ord("ÿ") + 1))
    b2u, n = {}, 0
    for b in range(256):
        if b in keep:
            b2u[b] = chr(b)
        else:
            b2u[b] = chr(256 + n)
            n += 1
    return b2u, {u: b for b, u in b2u.items()}


class Tokenizer:
    def __init__(self, tokens: list[str], scores: list[float], types: list[int], merges: list[str], model: str,
                 pre: str, bos_id: int, eos_ids: list[int], add_bos: bool, add_space_prefix: bool = True,
                 chat_template: Optional[str] = None, unk_id: int = -1):
        self.tokens = tokens
        self.types = types or [TOKEN_NORMAL] * len(tokens)
        self.model = "gpt2" if model == "gpt2" else "llama"
        self.bos_id, self.eos_ids = bos_id, list(eos_ids)
        self.add_bos = add_bos
        self.add_space_prefix = add_space_prefix
        self.chat_template = chat_template
        self.core = _native.host().BpeTokenizer([t.encode("utf-8", "surrogatepass") for t in tokens],
                                                [float(s) for s in (scores or [0.0] * len(tokens))],
                                                [m.encode("utf-8") for m in merges], self.model)
        if unk_id >= 0:
            self.core.set_unk(unk_id)
        self.pre = regex.compile(_PRE[pre_family(pre)])
        self.special = {t: i for i, t in enumerate(tokens)
                        if self.types[i] in (TOKEN_CONTROL, TOKEN_USER) and t}
        self._special_re = regex.compile("(" + "|".join(regex.escape(t) for t in
                                                         sorted(self.special, key=len, reverse=True)) + ")") \
            if self.special else None
        self._cache: dict[str, list[int]] = {}

    @classmethod
    def from_gguf(cls, src) -> "Tokenizer":
        md = src.metadata
        toks = [t.decode("utf-8", "replace") if isinstance(t, bytes) else t for t in (md("tokenizer.ggml.tokens") or [])]
        if not toks:
            raise ValueError("GGUF has no tokenizer.ggml.tokens")
        merges = [m.decode("utf-8", "replace") if isinstance(m, bytes) else m for m in (md("tokenizer.ggml.merges") or [])]
        eos = md("tokenizer.ggml.eos_token_id", 2)
        eos_ids = [int(eos)]
        eot = md("tokenizer.ggml.eot_token_id", None)
        if eot is not None and int(eot) not in eos_ids:
            eos_ids.append(int(eot))
        return cls(toks, md("tokenizer.ggml.scores") or [], md("tokenizer.ggml.token_type") or [], merges,
                   md("tokenizer.ggml.model", "llama"), md("tokenizer.ggml.pre", "gpt2"),
                   int(md("tokenizer.ggml.bos_token_id", 1)), eos_ids,
                   bool(md("tokenizer.ggml.add_bos_token", True)),
                   bool(md("tokenizer.ggml.add_space_prefix", True)), md("tokenizer.chat_template", None),
                   int(md("tokenizer.ggml.unknown_token_id", -1)))

    @property
    def vocab_size(self) -> int:
        return len(self.tokens)

    # -- encode ---------------------------------------------------------------------------------
    def _encode_text(self, text: str, first: bool) -> list[int]:
        if not text:
            return []
        if self.model == "gpt2":
            b2u, _ = _byte_unicode()
            out: list[int] = []
            for piece in self.pre.findall(text):
                ids = self._cache.get(piece)
                if ids is None:
                    mapped = "".join(b2u[b] for b in piece.encode("utf-8"))
                    ids = self.core.encode_piece(mapped.encode("utf-8"))
                    if len(self._cache) < 100_000:
                        self._cache[piece] = ids
                out.extend(ids)
            return out
        t = text.replace(" ", "▁")
        if first and self.add_space_prefix and not t.startswith("▁"):
            t = "▁" + t
        return self.core.encode_piece(t.encode("utf-8"))

    def encode(self, text: str, add_bos: Optional[bool] = None, parse_special: bool = True) -> list[int]:
        add_bos = self.add_bos if add_bos is None else add_bos
        out = [self.bos_id] if add_bos and self.bos_id >= 0 else []
        parts = self._special_re.split(text) if (parse_special and self._special_re) else [text]
        first = True
        for part in parts:
            if not part:
                continue
            if part in self.special and parse_special:
                out.append(self.special[part])
            else:
                out.extend(self._encode_text(part, first))
            first = False
        return out

    # -- decode ---------------------------------------------------------------------------------
    def token_bytes(self, tid: int) -> bytes:
        if tid < 0 or tid >= len(self.tokens):
            return b""
        t = self.tokens[tid]
        ty = self.types[tid]
        if ty == TOKEN_BYTE or (len(t) == 6 and t.startswith("<0x") and t.endswith(">")):
            try:
                return bytes([int(t[3:5], 16)])
            except ValueError:
                pass
        if self.model == "gpt2":
            _, u2b = _byte_unicode()
            try:
                return bytes(u2b[c] for c in t)
            except KeyError:
                return t.encode("utf-8")
        return t.encode("utf-8")

    def post(self, text: str) -> str:
        """Text-level clean-up of decoded pieces (SentencePiece marks spaces with U+2581)."""
        return text.replace("▁", " ") if self.model == "llama" else text

    def is_special(self, tid: int) -> bool:
        return 0 <= tid < len(self.types) and self.types[tid] in (TOKEN_CONTROL, TOKEN_UNUSED)

    def decode(self, ids: Iterable[int], skip_special: bool = True) -> str:
        data = b"".join(self.token_bytes(i) for i in ids if not (skip_special and self.is_special(i)))
        return self.post(data.decode("utf-8", "replace"))


class IncrementalDetokenizer:
    """Streams text deltas for generated tokens; holds back the bytes of an incomplete trailing UTF-8
    sequence (ill-formed bytes become U+FFFD at once, so one bad byte never stalls the stream) and
    text that may be the start of a stop string."""

    def __init__(self, tok: Tokenizer, stop: Optional[list[str]] = None, skip_special: bool = True):
        self.tok = tok
        self.stop = [s for s in (stop or []) if s]
        self.skip_special = skip_special
        self.dec = codecs.getincrementaldecoder("utf-8")(errors="replace")
        self.text = ""        # decoded, not yet emitted
        self.emitted = ""
        self.stopped = False
        self.hold = max((len(s) for s in self.stop), default=1) - 1

    def push(self, ids: Iterable[int], final: bool = False) -> str:
        if self.stopped:
            return ""
        data = b"".join(self.tok.token_bytes(i) for i in ids
                        if not (self.skip_special and self.tok.is_special(i)))
        self.text += self.tok.post(self.dec.decode(data, final=final))
        for st in self.stop:
            k = self.text.find(st)
            if k >= 0:
                out = self.text[:k]
                self.text = ""
                self.stopped = True
                self.emitted += out
                return out
        if final or self.hold == 0:
            out, self.text = self.text, ""
        else:
            n = max(0, len(self.text) - self.hold)
            out, self.text = self.text[:n], self.text[n:]
        self.emitted += out
        return out
