"""Tensor source over a HuggingFace checkpoint directory (config.json + *.safetensors).

Counterpart of the reference's safetensors branch of ``ModelLoader`` (src/model/model_loader.cpp:
78-296 reads the shards, src/model/weight_layout_plan.cpp:17 maps HF names to shard strategies).
The source presents the checkpoint under the GGUF tensor names and row layout that the weight
loader consumes (``info`` / ``rows`` / ``has`` / ``metadata``, as ``GgufSource``), so the same TP
sharding and tiling run on it:

* names: ``model.layers.{i}.self_attn.q_proj.weight`` -> ``blk.{i}.attn_q.weight`` and so on; a
  Mixtral layer's per-expert ``w1`` / ``w3`` / ``w2`` are presented stacked, as the GGUF
  ``ffn_{gate,up,down}_exps`` tensors (row ``e * F + f``);
* Q/K rows stay in HF order: HF checkpoints rotate halves (``rope_neox`` is set by
  ``model_config_from_hf``), where llama GGUFs store the rows permuted for adjacent-pair RoPE;
* BF16 / F16 / F32 matrices are handed over as their raw bytes (the GEMM reads bf16 tiles); 1-D
  tensors (norm weights) are converted to F32, as GGUF stores them;
* ``metadata`` answers the ``tokenizer.*`` keys from tokenizer.json / tokenizer_config.json for a
  byte-level BPE tokenizer (Llama 3) or a SentencePiece-style BPE with byte fallback (Llama 2 /
  Mistral / Mixtral), so ``Tokenizer.from_gguf`` builds the same tokenizer.
"""
from __future__ import annotations

import glob
import json
import os
import re
from typing import Optional

import numpy as np

from ..config import ModelConfig, model_config_from_hf
from ..gguf.constants import GType
from ..gguf.random_init import TensorSpec
from .safetensors_io import SafetensorsFile

_GT = {"F32": GType.F32, "F16": GType.F16, "BF16": GType.BF16}

_TOP = {"model.embed_tokens.weight": "token_embd.weight", "model.norm.weight": "output_norm.weight",
        "lm_head.weight": "output.weight"}
_LAYER = {"input_layernorm": "attn_norm", "post_attention_layernorm": "ffn_norm",
          "self_attn.q_proj": "attn_q", "self_attn.k_proj": "attn_k", "self_attn.v_proj": "attn_v",
          "self_attn.o_proj": "attn_output", "mlp.gate_proj": "ffn_gate", "mlp.up_proj": "ffn_up",
          "mlp.down_proj": "ffn_down", "block_sparse_moe.gate": "ffn_gate_inp"}
_EXPERT = {"w1": "ffn_gate_exps", "w3": "ffn_up_exps", "w2": "ffn_down_exps"}
_LAYER_RE = re.compile(r"model\.layers\.(\d+)\.(.+)\.weight$")
_EXPERT_RE = re.compile(r"block_sparse_moe\.experts\.(\d+)\.(w[123])$")
_IGNORED = re.compile(r".*\.rotary_emb\.inv_freq$")

SUPPORTED_MODEL_TYPES = ("llama", "mistral", "mixtral")


def gguf_name(hf: str) -> Optional[tuple[str, Optional[int]]]:
    """(GGUF tensor name, expert index or None) of a HF tensor name; None for ignored tensors."""
    if hf in _TOP:
        return _TOP[hf], None
    if _IGNORED.match(hf):
        return None
    m = _LAYER_RE.match(hf)
    if m:
        i, rest = int(m.group(1)), m.group(2)
        if rest in _LAYER:
            return f"blk.{i}.{_LAYER[rest]}.weight", None
        e = _EXPERT_RE.match(rest)
        if e:
            return f"blk.{i}.{_EXPERT[e.group(2)]}.weight", int(e.group(1))
    raise ValueError(f"unsupported tensor {hf!r} in the checkpoint (llama / mistral / mixtral layouts only)")


class _Tensor:
    """One GGUF-named tensor: a single safetensors entry, or the stacked entries of E experts."""

    def __init__(self, name: str):
        self.name = name
        self.parts: dict[int, tuple[SafetensorsFile, str]] = {}
        self.dtype = ""
        self.shape: list[int] = []

    def add(self, f: SafetensorsFile, hf: str, expert: Optional[int]) -> None:
        e = f.entries[hf]
        if e.dtype not in _GT:
            raise ValueError(f"{hf}: dtype {e.dtype} is not supported (BF16, F16 or F32 weights)")
        if self.parts and (e.dtype != self.dtype or e.shape != self.shape):
            raise ValueError(f"{hf}: experts of {self.name} differ in dtype or shape")
        self.dtype, self.shape = e.dtype, list(e.shape)
        self.parts[-1 if expert is None else expert] = (f, hf)

    @property
    def n_parts(self) -> int:
        return len(self.parts)

    @property
    def part_rows(self) -> int:
        return int(np.prod(self.shape[:-1])) if len(self.shape) > 1 else 1

    @property
    def ne(self) -> list[int]:
        ne = list(reversed(self.shape)) if self.shape else [1]
        if -1 not in self.parts:
            ne.append(self.n_parts)
        return ne


class HfSource:
    def __init__(self, path: str):
        d = path if os.path.isdir(path) else os.path.dirname(os.path.abspath(path))
        self.path, self.dir = path, d
        if not os.path.exists(os.path.join(d, "config.json")):
            raise FileNotFoundError(f"{d}: no config.json beside the safetensors checkpoint")
        self.hf_config = json.load(open(os.path.join(d, "config.json")))
        mt = self.hf_config.get("model_type", "llama")
        if mt not in SUPPORTED_MODEL_TYPES:
            raise ValueError(f"unsupported model_type {mt!r} (supported: {', '.join(SUPPORTED_MODEL_TYPES)})")
        if os.path.isdir(path):
            idx = os.path.join(d, "model.safetensors.index.json")
            if os.path.exists(idx):
                files = sorted(set(json.load(open(idx))["weight_map"].values()))
                files = [os.path.join(d, f) for f in files]
            else:
                files = sorted(glob.glob(os.path.join(d, "*.safetensors")))
        else:
            files = [path]
        if not files:
            raise FileNotFoundError(f"{d}: no .safetensors files")
        self.files = [SafetensorsFile(f) for f in files]
        self.tensors: dict[str, _Tensor] = {}
        for f in self.files:
            for hf in f.entries:
                g = gguf_name(hf)
                if g is None:
                    continue
                name, expert = g
                self.tensors.setdefault(name, _Tensor(name)).add(f, hf, expert)
        for t in self.tensors.values():
            if -1 not in t.parts and sorted(t.parts) != list(range(t.n_parts)):
                raise ValueError(f"{t.name}: expert indices are not contiguous from 0")
        self._tok: Optional[dict] = None

    # ---------------------------------------------------------------------------------------------
    def model_config(self) -> ModelConfig:
        m = model_config_from_hf(self.dir)
        m.name = self.hf_config.get("_name_or_path", "") or os.path.basename(os.path.normpath(self.dir))
        if "output.weight" not in self.tensors:
            m.tie_embeddings = True
        emb = self.tensors.get("token_embd.weight")
        if emb is None:
            raise ValueError("checkpoint has no model.embed_tokens.weight")
        if emb.shape[0] != m.vocab:
            raise ValueError(f"config vocab_size {m.vocab} != embedding rows {emb.shape[0]}")
        return m

    def has(self, name: str) -> bool:
        return name in self.tensors

    def info(self, name: str) -> TensorSpec:
        t = self.tensors[name]
        g = GType.F32 if len(t.shape) <= 1 else _GT[t.dtype]
        return TensorSpec(name, t.ne, int(g))

    def rows(self, name: str, r0: int = 0, r1: Optional[int] = None):
        """Rows [r0, r1) in GGUF order: raw bytes (uint8) for BF16 / F16, float32 for F32 and 1-D."""
        import torch
        t = self.tensors[name]
        P = t.part_rows
        total = P * t.n_parts
        r1 = total if r1 is None else r1
        if not 0 <= r0 <= r1 <= total:
            raise IndexError(f"{name}: rows [{r0}, {r1}) out of [0, {total})")
        keys = [-1] if -1 in t.parts else list(range(t.n_parts))
        chunks = []
        for j, k in enumerate(keys):
            a, b = max(r0, j * P), min(r1, (j + 1) * P)
            if a >= b:
                continue
            f, hf = t.parts[k]
            chunks.append(np.array(f.rows_bytes(hf, a - j * P, b - j * P)))  # copies the slice
        raw = np.concatenate(chunks, 0) if len(chunks) != 1 else chunks[0]
        if len(t.shape) <= 1 or t.dtype == "F32":
            if t.dtype == "F32":
                return torch.from_numpy(raw.view(np.float32))
            return torch.from_numpy(raw.view(np.int16)).view(
                torch.bfloat16 if t.dtype == "BF16" else torch.float16).float()
        return torch.from_numpy(raw)

    # ---------------------------------------------------------------------------------------------
    def metadata(self, key: str, default=None):
        if not key.startswith("tokenizer."):
            return default
        if self._tok is None:
            self._tok = _tokenizer_metadata(self.dir, self.hf_config)
        return self._tok.get(key, default)


def _token_id(tok, vocab: dict) -> Optional[int]:
    if isinstance(tok, dict):
        tok = tok.get("content")
    return vocab.get(tok) if isinstance(tok, str) else None


def _special_ids(d: str, hf_config: dict, vocab: dict) -> tuple[dict, int, int]:
    tc_path = os.path.join(d, "tokenizer_config.json")
    tc = json.load(open(tc_path, encoding="utf-8")) if os.path.exists(tc_path) else {}
    bos = _token_id(tc.get("bos_token"), vocab)
    eos = _token_id(tc.get("eos_token"), vocab)
    bos = hf_config.get("bos_token_id", 1) if bos is None else bos
    cfg_eos = hf_config.get("eos_token_id", 2)
    eos = (cfg_eos[0] if isinstance(cfg_eos, list) else cfg_eos) if eos is None else eos
    return tc, int(bos), int(eos)


def _spm_metadata(tj, model, vocab, tokens, types, merges, added, n, d, hf_config) -> dict:
    """SentencePiece-style BPE (byte fallback, "▁" for spaces) as the GGUF "llama" tokenizer: the
    native SPM merger takes the adjacent pair whose merged token scores highest, so each merged token
    scores minus its merge rank (the earliest merge wins, as in BPE)."""
    scores = [0.0] * n
    for r, m in enumerate(merges):
        a, _, b = m.partition(" ")
        i = vocab.get(a + b)
        if i is not None and scores[i] == 0.0:
            scores[i] = -float(r + 1)
    for i, t in enumerate(tokens):
        if len(t) == 6 and t.startswith("<0x") and t.endswith(">"):
            types[i] = 6  # byte
    unk = model.get("unk_token")
    unk_id = vocab.get(unk, -1) if isinstance(unk, str) else -1
    if unk_id >= 0:
        types[unk_id] = 2
    for a in added:
        types[int(a["id"])] = 3 if a.get("special") else 4
    norm = json.dumps(tj.get("normalizer") or {})
    pre = tj.get("pre_tokenizer") or {}
    prefix = '"Prepend"' in norm or (pre.get("type") == "Metaspace" and
                                      pre.get("prepend_scheme", "always") in ("always", "first"))
    tc, bos, eos = _special_ids(d, hf_config, vocab)
    md = {"tokenizer.ggml.model": "llama", "tokenizer.ggml.tokens": tokens, "tokenizer.ggml.scores": scores,
          "tokenizer.ggml.token_type": types, "tokenizer.ggml.bos_token_id": bos,
          "tokenizer.ggml.eos_token_id": eos, "tokenizer.ggml.add_space_prefix": bool(prefix),
          "tokenizer.ggml.add_bos_token": bool(tc.get("add_bos_token", True)),
          "tokenizer.ggml.unknown_token_id": unk_id}
    ct = tc.get("chat_template")
    if isinstance(ct, list):
        ct = next((c.get("template") for c in ct if c.get("name") == "default"), None)
    if ct:
        md["tokenizer.chat_template"] = ct
    return md



def _pre_family(pre_tokenizer: dict) -> str:
    """The GGUF pre-tokeniser family of a tokenizer.json pre_tokenizer, from its split expression:
    "llama-bpe" (digits in groups of three), "qwen2" (single digits), "qwen35" (single digits, combining
    marks join words), else "gpt2"."""
    regs: list[str] = []

    def walk(x):
        if isinstance(x, dict):
            pat = x.get("pattern")
            if isinstance(pat, dict) and isinstance(pat.get("Regex"), str):
                regs.append(pat["Regex"])
            for v in x.values():
                walk(v)
        elif isinstance(x, list):
            for v in x:
                walk(v)
    walk(pre_tokenizer)
    for r in regs:
        if "(?i:'s|'t|'re|'ve|'m|'ll|'d)" in r:
            if "\\p{M}" in r:
                return "qwen35"
            return "llama-bpe" if "\\p{N}{1,3}" in r else "qwen2"
    return "gpt2"

def _tokenizer_metadata(d: str, hf_config: dict) -> dict:
    """GGUF tokenizer.* keys from tokenizer.json (byte-level BPE) and tokenizer_config.json."""
    p = os.path.join(d, "tokenizer.json")
    if not os.path.exists(p):
        return {}
    tj = json.load(open(p, encoding="utf-8"))
    model = tj.get("model") or {}
    if model.get("type") != "BPE":
        raise ValueError("tokenizer.json: only BPE tokenizers are supported (byte-level, as Llama 3, or "
                         "SentencePiece-style with byte fallback, as Llama 2 / Mistral); give a GGUF file "
                         "with --tokenizer for others")
    spm = bool(model.get("byte_fallback"))
    vocab = dict(model.get("vocab") or {})
    added = tj.get("added_tokens") or []
    for a in added:
        vocab[a["content"]] = int(a["id"])
    n = max(vocab.values()) + 1 if vocab else 0
    n = max(n, int(hf_config.get("vocab_size", 0)))
    tokens = [f"[PAD{i}]" for i in range(n)]
    types = [1] * n  # normal
    for tok, i in vocab.items():
        tokens[i] = tok
    for i in range(n):
        if tokens[i] == f"[PAD{i}]":
            types[i] = 5  # unused
    for a in added:
        types[int(a["id"])] = 3 if a.get("special") else 4  # control / user-defined
    merges = [m if isinstance(m, str) else " ".join(m) for m in (model.get("merges") or [])]
    if spm:
        return _spm_metadata(tj, model, vocab, tokens, types, merges, added, n, d, hf_config)
    pre = _pre_family(tj.get("pre_tokenizer") or {})
    tc_path = os.path.join(d, "tokenizer_config.json")
    tc = json.load(open(tc_path, encoding="utf-8")) if os.path.exists(tc_path) else {}
    bos = _token_id(tc.get("bos_token"), vocab)
    eos = _token_id(tc.get("eos_token"), vocab)
    bos = hf_config.get("bos_token_id", 1) if bos is None else bos
    cfg_eos = hf_config.get("eos_token_id", 2)
    eos = (cfg_eos[0] if isinstance(cfg_eos, list) else cfg_eos) if eos is None else eos
    md = {"tokenizer.ggml.model": "gpt2", "tokenizer.ggml.pre": pre, "tokenizer.ggml.tokens": tokens,
          "tokenizer.ggml.token_type": types, "tokenizer.ggml.merges": merges,
          "tokenizer.ggml.bos_token_id": int(bos), "tokenizer.ggml.eos_token_id": int(eos),
          "tokenizer.ggml.add_space_prefix": False}
    if isinstance(cfg_eos, list):
        extra = [int(x) for x in cfg_eos if int(x) != int(eos)]
        if extra:
            md["tokenizer.ggml.eot_token_id"] = extra[0]
    if "add_bos_token" in tc:
        md["tokenizer.ggml.add_bos_token"] = bool(tc["add_bos_token"])
    else:
        bos_tok = tokens[int(bos)] if 0 <= int(bos) < n else None
        md["tokenizer.ggml.add_bos_token"] = bool(bos_tok) and bos_tok in json.dumps(tj.get("post_processor") or {})
    ct = tc.get("chat_template")
    if isinstance(ct, list):
        ct = next((c.get("template") for c in ct if c.get("name") == "default"), None)
    if ct:
        md["tokenizer.chat_template"] = ct
    return md
