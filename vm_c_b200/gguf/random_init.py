"""Seeded random-init checkpoints of the benchmark architectures.

Two producers of identical tensor layouts:
  * ``write_random_gguf``: CPU, numpy normal(0, std) + the C++ quantisers -> a GGUF file (used for
    small models and for the server / CLI).
  * ``GpuRandomSource``: the same tensors generated directly on a GPU (torch CUDA Philox normal +
    the on-device quantisers of csrc/kernels/weights.cu), returning GGUF block bytes in device
    memory. Used for multi-GB models on a fresh GPU box where writing and re-reading a file would
    dominate start-up.

Quantisation mixes follow llama.cpp's naming: "Q4_K_M" (Q4_K, with Q6_K for output.weight and for
attn_v / ffn_down in the layers selected by llama.cpp's use_more_bits rule), "Q4_K", "Q8_0",
"BF16", "F16", "F32". Norm weights are F32; a tensor whose row length is not a multiple of the
block size stays F16 (llama.cpp convention).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from ..config import ModelConfig
from .constants import BLOCK, FILE_TYPE, GType, VType, blk, row_bytes

PRESETS: dict[str, ModelConfig] = {
    # config 1: tiny llama (CPU oracle)
    "tiny-llama": ModelConfig(name="tiny-llama", n_layers=4, hidden=256, n_heads=8, n_kv_heads=4, head_dim=32, ffn=688,
                              vocab=32000, rms_eps=1e-5, rope_theta=10000.0, context_length=2048,
                              bos_token_id=1, eos_token_ids=[2]),
    # config 2 / 5 target: Llama-3-8B architecture
    "llama3-8b": ModelConfig(name="llama3-8b", n_layers=32, hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128,
                             ffn=14336, vocab=128256, rms_eps=1e-5, rope_theta=500000.0, context_length=8192,
                             bos_token_id=128000, eos_token_ids=[128001, 128009]),
    # config 3: Llama-3-70B architecture
    "llama3-70b": ModelConfig(name="llama3-70b", n_layers=80, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128,
                              ffn=28672, vocab=128256, rms_eps=1e-5, rope_theta=500000.0, context_length=8192,
                              bos_token_id=128000, eos_token_ids=[128001, 128009]),
    # config 4: Mixtral-8x7B architecture
    "mixtral-8x7b": ModelConfig(name="mixtral-8x7b", n_layers=32, hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128,
                                ffn=14336, vocab=32000, rms_eps=1e-5, rope_theta=1000000.0, context_length=32768,
                                n_experts=8, n_experts_used=2, bos_token_id=1, eos_token_ids=[2]),
    # small Mixtral-architecture model for tests (4 experts, top-2)
    "tiny-mixtral": ModelConfig(name="tiny-mixtral", n_layers=2, hidden=256, n_heads=8, n_kv_heads=4, head_dim=32,
                                ffn=512, vocab=32000, rms_eps=1e-5, rope_theta=10000.0, context_length=2048,
                                n_experts=4, n_experts_used=2, bos_token_id=1, eos_token_ids=[2]),
    # small Mixtral-architecture model with 8 experts (expert parallelism up to 8 ranks)
    "tiny-mixtral8": ModelConfig(name="tiny-mixtral8", n_layers=2, hidden=256, n_heads=8, n_kv_heads=8, head_dim=32,
                                 ffn=512, vocab=32000, rms_eps=1e-5, rope_theta=10000.0, context_length=2048,
                                 n_experts=8, n_experts_used=2, bos_token_id=1, eos_token_ids=[2]),
    # small hybrid gated delta-net model (Qwen3.5-MoE architecture): layers 0-2 GDN, layer 3 full
    # attention with partial RoPE, 4 experts (top-2) plus a shared expert
    "tiny-qwen35moe": ModelConfig(arch="qwen35moe", name="tiny-qwen35moe", n_layers=4, hidden=256, n_heads=4,
                                  n_kv_heads=2, head_dim=64, ffn=256, vocab=32000, rms_eps=1e-6,
                                  rope_theta=10000000.0, rope_neox=True, context_length=2048, n_experts=4,
                                  n_experts_used=2, bos_token_id=1, eos_token_ids=[2], rope_dims=16, ssm_conv=4,
                                  ssm_state=64, ssm_k_heads=2, ssm_v_heads=4, full_attn_interval=4, ffn_shexp=256),
    # config 5 draft model
    "draft-16l-2048": ModelConfig(name="draft-16l-2048", n_layers=16, hidden=2048, n_heads=32, n_kv_heads=8,
                                  head_dim=64, ffn=8192, vocab=128256, rms_eps=1e-5, rope_theta=500000.0,
                                  context_length=8192, bos_token_id=128000, eos_token_ids=[128001, 128009]),
}


def preset(name: str) -> ModelConfig:
    from copy import deepcopy
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; known: {sorted(PRESETS)}")
    return deepcopy(PRESETS[name])


def use_more_bits(i: int, n: int) -> bool:
    return i < n // 8 or i >= 7 * n // 8 or (i - n // 8) % 3 == 2


@dataclass
class TensorSpec:
    name: str
    ne: list[int]       # GGUF order: ne[0] = row length
    gtype: int
    std: float = 0.02
    const: float | None = None   # constant fill (norm weights)

    @property
    def rows(self) -> int:
        r = 1
        for d in self.ne[1:]:
            r *= d
        return r

    @property
    def nbytes(self) -> int:
        return row_bytes(self.gtype, self.ne[0]) * self.rows


def _fit(gtype: int, K: int) -> int:
    be = BLOCK[GType(gtype)][0]
    return gtype if K % be == 0 else int(GType.F16)


def _hybrid_plan(cfg: ModelConfig, t) -> list[TensorSpec]:
    """Tensors of a qwen35moe GGUF (reference: src/official/llama/models/qwen35moe.cpp:62-112)."""
    H, F, V, L, D = cfg.hidden, cfg.ffn, cfg.vocab, cfg.n_layers, cfg.head_dim
    Ds, Hk, Hv, E, Fs = cfg.ssm_state, cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.n_experts, cfg.ffn_shexp
    conv_dim = 2 * Hk * Ds + Hv * Ds
    f32 = int(GType.F32)
    specs = [TensorSpec("token_embd.weight", [H, V], t("embd", None, H))]
    for i in range(L - cfg.nextn_layers):
        b = f"blk.{i}."
        specs.append(TensorSpec(b + "attn_norm.weight", [H], f32, const=1.0))
        specs.append(TensorSpec(b + "post_attention_norm.weight", [H], f32, const=1.0))
        if cfg.is_recurrent(i):
            specs += [TensorSpec(b + "attn_qkv.weight", [H, conv_dim], t("attn_qkv", i, H)),
                      TensorSpec(b + "attn_gate.weight", [H, Hv * Ds], t("attn_gate", i, H)),
                      TensorSpec(b + "ssm_conv1d.weight", [cfg.ssm_conv, conv_dim], f32, std=0.3),
                      TensorSpec(b + "ssm_dt.bias", [Hv], f32, std=0.1),
                      TensorSpec(b + "ssm_a", [Hv], f32, const=-0.5),
                      TensorSpec(b + "ssm_beta.weight", [H, Hv], f32),
                      TensorSpec(b + "ssm_alpha.weight", [H, Hv], f32),
                      TensorSpec(b + "ssm_norm.weight", [Ds], f32, const=1.0),
                      TensorSpec(b + "ssm_out.weight", [Hv * Ds, H], t("ssm_out", i, Hv * Ds))]
        else:
            specs += [TensorSpec(b + "attn_q.weight", [H, 2 * cfg.n_heads * D], t("attn_q", i, H)),
                      TensorSpec(b + "attn_k.weight", [H, cfg.kv_size], t("attn_k", i, H)),
                      TensorSpec(b + "attn_v.weight", [H, cfg.kv_size], t("attn_v", i, H)),
                      TensorSpec(b + "attn_output.weight", [cfg.q_size, H], t("attn_output", i, cfg.q_size)),
                      TensorSpec(b + "attn_q_norm.weight", [D], f32, const=1.0),
                      TensorSpec(b + "attn_k_norm.weight", [D], f32, const=1.0)]
        specs += [TensorSpec(b + "ffn_gate_inp.weight", [H, E], f32),
                  TensorSpec(b + "ffn_gate_exps.weight", [H, F, E], t("ffn_gate", i, H)),
                  TensorSpec(b + "ffn_up_exps.weight", [H, F, E], t("ffn_up", i, H)),
                  TensorSpec(b + "ffn_down_exps.weight", [F, H, E], t("ffn_down", i, F)),
                  TensorSpec(b + "ffn_gate_inp_shexp.weight", [H], f32),
                  TensorSpec(b + "ffn_gate_shexp.weight", [H, Fs], t("ffn_gate", i, H)),
                  TensorSpec(b + "ffn_up_shexp.weight", [H, Fs], t("ffn_up", i, H)),
                  TensorSpec(b + "ffn_down_shexp.weight", [Fs, H], t("ffn_down", i, Fs))]
    specs.append(TensorSpec("output_norm.weight", [H], f32, const=1.0))
    if not cfg.tie_embeddings:
        specs.append(TensorSpec("output.weight", [H, V], t("output", None, H)))
    return specs


def tensor_plan(cfg: ModelConfig, mix: str) -> list[TensorSpec]:
    H, F, V, L = cfg.hidden, cfg.ffn, cfg.vocab, cfg.n_layers
    q, kv = cfg.q_size, cfg.kv_size
    base = {"Q4_K_M": GType.Q4_K, "Q4_K": GType.Q4_K, "Q8_0": GType.Q8_0, "BF16": GType.BF16,
            "F16": GType.F16, "F32": GType.F32}[mix]

    def t(kind: str, i: int | None, K: int) -> int:
        g = base
        if mix == "Q4_K_M":
            if kind == "output":
                g = GType.Q6_K
            elif kind in ("attn_v", "ffn_down") and use_more_bits(i, L):
                g = GType.Q6_K
        return _fit(int(g), K)

    if cfg.is_hybrid:
        return _hybrid_plan(cfg, t)
    specs = [TensorSpec("token_embd.weight", [H, V], t("embd", None, H))]
    for i in range(L):
        specs.append(TensorSpec(blk(i, "attn_norm"), [H], int(GType.F32), const=1.0))
        specs.append(TensorSpec(blk(i, "attn_q"), [H, q], t("attn_q", i, H)))
        specs.append(TensorSpec(blk(i, "attn_k"), [H, kv], t("attn_k", i, H)))
        specs.append(TensorSpec(blk(i, "attn_v"), [H, kv], t("attn_v", i, H)))
        specs.append(TensorSpec(blk(i, "attn_output"), [q, H], t("attn_output", i, q)))
        specs.append(TensorSpec(blk(i, "ffn_norm"), [H], int(GType.F32), const=1.0))
        if cfg.is_moe:
            E = cfg.n_experts
            specs.append(TensorSpec(blk(i, "ffn_gate_inp"), [H, E], int(GType.F32)))
            specs.append(TensorSpec(blk(i, "ffn_gate_exps"), [H, F, E], t("ffn_gate", i, H)))
            specs.append(TensorSpec(blk(i, "ffn_up_exps"), [H, F, E], t("ffn_up", i, H)))
            specs.append(TensorSpec(blk(i, "ffn_down_exps"), [F, H, E], t("ffn_down", i, F)))
        else:
            specs.append(TensorSpec(blk(i, "ffn_gate"), [H, F], t("ffn_gate", i, H)))
            specs.append(TensorSpec(blk(i, "ffn_up"), [H, F], t("ffn_up", i, H)))
            specs.append(TensorSpec(blk(i, "ffn_down"), [F, H], t("ffn_down", i, F)))
    specs.append(TensorSpec("output_norm.weight", [H], int(GType.F32), const=1.0))
    if not cfg.tie_embeddings:
        specs.append(TensorSpec("output.weight", [H, V], t("output", None, H)))
    return specs


def synthetic_vocab(V: int) -> tuple[list[str], list[float], list[int]]:
    """SentencePiece-style vocabulary: <unk>, <s>, </s>, 256 byte tokens, printable pieces, fillers."""
    toks = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)]
    types = [2, 3, 3] + [6] * 256
    pieces = []
    for c in range(32, 127):
        pieces.append(chr(c))
    for c in "abcdefghijklmnopqrstuvwxyz":
        pieces.append("▁" + c)
    for a in "etaoinshrdlu":
        for b in "etaoinshrdlu":
            pieces.append(a + b)
            pieces.append("▁" + a + b)
    seen = set(toks)
    for p in pieces:
        if p not in seen and len(toks) < V:
            toks.append(p)
            types.append(1)
            seen.add(p)
    i = 0
    while len(toks) < V:
        toks.append(f"<filler_{i}>")
        types.append(4)
        i += 1
    scores = [0.0] * 3 + [0.0] * 256 + [-float(len(p)) * 0.0 - i * 1e-4 for i, p in enumerate(toks[259:])]
    return toks[:V], scores[:V], types[:V]


def gguf_metadata(cfg: ModelConfig, mix: str) -> list[tuple[str, int, object, int]]:
    """(key, value type, value, array element type) entries of a llama-architecture GGUF."""
    a = "qwen35moe" if cfg.is_hybrid else "llama"
    md = [
        ("general.architecture", VType.STRING, a, 0),
        ("general.name", VType.STRING, cfg.name or "random-init", 0),
        ("general.file_type", VType.UINT32, FILE_TYPE.get(mix, 0), 0),
        (f"{a}.block_count", VType.UINT32, cfg.n_layers, 0),
        (f"{a}.embedding_length", VType.UINT32, cfg.hidden, 0),
        (f"{a}.feed_forward_length", VType.UINT32, cfg.ffn, 0),
        (f"{a}.attention.head_count", VType.UINT32, cfg.n_heads, 0),
        (f"{a}.attention.head_count_kv", VType.UINT32, cfg.n_kv_heads, 0),
        (f"{a}.attention.key_length", VType.UINT32, cfg.head_dim, 0),
        (f"{a}.attention.value_length", VType.UINT32, cfg.head_dim, 0),
        (f"{a}.attention.layer_norm_rms_epsilon", VType.FLOAT32, cfg.rms_eps, 0),
        (f"{a}.rope.freq_base", VType.FLOAT32, cfg.rope_theta, 0),
        (f"{a}.rope.dimension_count", VType.UINT32, cfg.head_dim, 0),
        (f"{a}.context_length", VType.UINT32, cfg.context_length, 0),
        (f"{a}.vocab_size", VType.UINT32, cfg.vocab, 0),
        # vm_c's GGUF parser requires this key (src/model/gguf_model_loader.cpp:471-482); written so
        # that the same file is accepted by the reference.
        (f"{a}.full_attention_interval", VType.UINT32, 1, 0),
    ]
    if cfg.is_moe:
        md.append((f"{a}.expert_count", VType.UINT32, cfg.n_experts, 0))
        md.append((f"{a}.expert_used_count", VType.UINT32, cfg.n_experts_used, 0))
    if cfg.is_hybrid:
        md = [m for m in md if m[0] not in (f"{a}.full_attention_interval", f"{a}.rope.dimension_count")]
        md += [(f"{a}.expert_feed_forward_length", VType.UINT32, cfg.ffn, 0),
               (f"{a}.expert_shared_feed_forward_length", VType.UINT32, cfg.ffn_shexp, 0),
               (f"{a}.rope.dimension_count", VType.UINT32, cfg.rope_dims or cfg.head_dim, 0),
               (f"{a}.ssm.conv_kernel", VType.UINT32, cfg.ssm_conv, 0),
               (f"{a}.ssm.inner_size", VType.UINT32, cfg.ssm_v_heads * cfg.ssm_state, 0),
               (f"{a}.ssm.state_size", VType.UINT32, cfg.ssm_state, 0),
               (f"{a}.ssm.time_step_rank", VType.UINT32, cfg.ssm_v_heads, 0),
               (f"{a}.ssm.group_count", VType.UINT32, cfg.ssm_k_heads, 0),
               (f"{a}.full_attention_interval", VType.UINT32, cfg.full_attn_interval, 0),
               (f"{a}.nextn_predict_layers", VType.UINT32, cfg.nextn_layers, 0)]
    toks, scores, types = synthetic_vocab(cfg.vocab)
    md += [
        ("tokenizer.ggml.model", VType.STRING, "llama", 0),
        ("tokenizer.ggml.tokens", VType.ARRAY, toks, int(VType.STRING)),
        ("tokenizer.ggml.scores", VType.ARRAY, scores, int(VType.FLOAT32)),
        ("tokenizer.ggml.token_type", VType.ARRAY, types, int(VType.INT32)),
        ("tokenizer.ggml.bos_token_id", VType.UINT32, cfg.bos_token_id if cfg.bos_token_id < cfg.vocab else 1, 0),
        ("tokenizer.ggml.eos_token_id", VType.UINT32, cfg.eos_token_ids[0] if cfg.eos_token_ids[0] < cfg.vocab else 2, 0),
        ("tokenizer.ggml.unknown_token_id", VType.UINT32, 0, 0),
        ("tokenizer.ggml.add_bos_token", VType.BOOL, True, 0),
    ]
    return md


def _np_values(spec: TensorSpec, rng: np.random.Generator) -> np.ndarray:
    K = spec.ne[0]
    if spec.const is not None:
        return np.full((spec.rows, K), spec.const, dtype=np.float32)
    return (rng.standard_normal((spec.rows, K), dtype=np.float32) * spec.std).astype(np.float32)


def write_random_gguf(path: str, cfg: ModelConfig, mix: str = "Q8_0", seed: int = 0) -> list[TensorSpec]:
    """Write a seeded random-init GGUF (weights ~ normal(0, 0.02) before quantisation)."""
    from .. import _native
    h = _native.host()
    specs = tensor_plan(cfg, mix)
    w = h.GgufWriter(32)
    for key, vt, val, et in gguf_metadata(cfg, mix):
        w.set(key, int(vt), val, int(et))
    for s in specs:
        w.add_tensor(s.name, s.ne, int(s.gtype))
    rng = np.random.default_rng(seed)
    # Draw every tensor's values in file order from one stream so the file depends only on seed.

    def produce(i: int):
        s = specs[i]
        vals = _np_values(s, rng)
        if s.gtype == GType.F32:
            return np.ascontiguousarray(vals)
        return h.quantize(int(s.gtype), vals)

    w.write(path, produce)
    return specs


class GpuRandomSource:
    """Generates the tensors of ``tensor_plan`` on a CUDA device, in GGUF block format."""

    def __init__(self, cfg: ModelConfig, mix: str, seed: int = 0, device="cuda"):
        import torch
        self.cfg, self.mix, self.seed = cfg, mix, seed
        self.device = torch.device(device)
        self.specs = {s.name: s for s in tensor_plan(cfg, mix)}
        self.order = {s.name: i for i, s in enumerate(tensor_plan(cfg, mix))}

    def has(self, name: str) -> bool:
        return name in self.specs

    def info(self, name: str) -> TensorSpec:
        return self.specs[name]

    def rows(self, name: str, r0: int = 0, r1: int | None = None):
        """GGUF bytes of rows [r0, r1) of tensor `name` as a uint8 [rows, row_bytes] CUDA tensor
        (F32 tensors are returned as float32 [rows, K])."""
        import torch
        from .. import ops
        s = self.specs[name]
        K = s.ne[0]
        r1 = s.rows if r1 is None else r1
        chunk_rows = max(1, (1 << 25) // K)
        outs = []
        for c0 in range((r0 // chunk_rows) * chunk_rows, r1, chunk_rows):
            c1 = min(c0 + chunk_rows, s.rows)
            g = torch.Generator(device=self.device)
            g.manual_seed((self.seed * 1_000_003 + self.order[name] * 7919 + c0 // chunk_rows) & 0x7fffffffffffffff)
            if s.const is not None:
                vals = torch.full((c1 - c0, K), s.const, dtype=torch.float32, device=self.device)
            else:
                vals = torch.randn((c1 - c0, K), generator=g, dtype=torch.float32, device=self.device) * s.std
            lo, hi = max(r0, c0) - c0, min(r1, c1) - c0
            vals = vals[lo:hi]
            if s.gtype == GType.F32:
                outs.append(vals.contiguous())
            elif s.gtype == GType.F16:
                outs.append(vals.half().view(torch.uint8).reshape(hi - lo, -1))
            elif s.gtype == GType.BF16:
                outs.append(vals.bfloat16().view(torch.uint8).reshape(hi - lo, -1))
            else:
                outs.append(ops.quantize_blocks(s.gtype, vals))
        return torch.cat(outs, 0) if len(outs) > 1 else outs[0]
