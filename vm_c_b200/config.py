"""Typed configuration: model / cache / parallel / scheduler / offload / server.

Mirrors the reference's VmCConfig (include/vm_c/core/config.hpp:12-236: ModelConfig,
CacheConfig :147-167, ParallelConfig :169-173, SchedulerConfig :182-205, ServerConfig :207-224)
and its defaults (block 16, gpu_memory_utilization 0.90, max_num_seqs 128, max_num_batched_tokens
max(2048, max_model_len) — src/core/engine.cpp:455-462). Model fields are filled from GGUF
metadata (src/model/gguf_model_loader.cpp:397-534 parse_gguf_config) or a HF config.json
(src/core/config.cpp:27 load_model_config_from_json); unlike the reference, missing
`full_attention_interval`, `context_length` and `key_length` are accepted.
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, field, asdict
from pathlib import Path
from typing import Optional


@dataclass
class ModelConfig:
    arch: str = "llama"
    name: str = ""
    n_layers: int = 32
    hidden: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rms_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_neox: bool = False          # llama GGUFs rotate adjacent pairs ("norm" mode)
    rope_scaling: Optional[dict] = None
    context_length: int = 8192
    max_model_len: int = 0           # 0: derive from context_length
    n_experts: int = 0
    n_experts_used: int = 0
    bos_token_id: int = 1
    eos_token_ids: list[int] = field(default_factory=lambda: [2])
    tie_embeddings: bool = False
    # Hybrid gated delta-net models (arch "qwen35moe"); zero for llama / mixtral.
    rope_dims: int = 0               # rotated dims per head (0: head_dim)
    ssm_conv: int = 0                # causal conv kernel size
    ssm_state: int = 0               # GDN head dim (key = value)
    ssm_k_heads: int = 0             # GDN key heads (ssm.group_count)
    ssm_v_heads: int = 0             # GDN value heads (ssm.time_step_rank)
    full_attn_interval: int = 0      # every n-th layer is full attention
    ffn_shexp: int = 0               # shared-expert FFN width
    nextn_layers: int = 0            # trailing MTP blocks (not run in the main pass)

    @property
    def is_hybrid(self) -> bool:
        return self.arch == "qwen35moe"

    def is_recurrent(self, i: int) -> bool:
        """Layer i is a gated delta-net layer (reference: qwen35moe.cpp:24-29 of load_arch_hparams)."""
        return (self.is_hybrid and i < self.n_layers - self.nextn_layers
                and (i + 1) % max(1, self.full_attn_interval) != 0)

    @property
    def q_size(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def is_moe(self) -> bool:
        return self.n_experts > 0

    def num_params(self) -> int:
        h, f, v = self.hidden, self.ffn, self.vocab
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        mlp = 3 * h * f * (self.n_experts if self.is_moe else 1) + (h * self.n_experts if self.is_moe else 0)
        per_layer = attn + mlp + 2 * h
        return self.n_layers * per_layer + v * h * (1 if self.tie_embeddings else 2) + h

    def validate(self) -> None:
        if self.n_heads % self.n_kv_heads:
            raise ValueError("n_heads must be a multiple of n_kv_heads")
        if self.head_dim not in (32, 64, 128):
            raise ValueError(f"head_dim {self.head_dim} unsupported (32, 64, 128)")


@dataclass
class CacheConfig:
    block_size: int = 16
    gpu_memory_utilization: float = 0.90
    gpu_safety_margin_mb: int = 256
    kv_cache_dtype: str = "auto"
    tq_rotation_seed: int = 0        # TurboQuant: 0 = plain Hadamard; else random signs per layer / KV head
    num_gpu_blocks: int = 0          # 0: size from free memory
    enable_prefix_caching: bool = True
    cpu_offload_gb: float = 0.0
    cpu_offload_params: list[str] = field(default_factory=list)
    kv_offloading_size: float = 0.0
    expert_gpu_cache_capacity: int = 0
    expert_cache_update_period: int = 0
    expert_cache_history_window: int = 0


@dataclass
class ParallelConfig:
    tensor_parallel_size: int = 1
    expert_parallel_size: int = 1
    gpu_devices: list[int] = field(default_factory=list)
    comm_backend: str = "fused"       # "fused" (peer-memory kernels) or "nccl" (baseline)


@dataclass
class SchedulerConfig:
    max_num_seqs: int = 128
    max_num_batched_tokens: int = 0   # 0: max(2048, max_model_len)
    enable_chunked_prefill: bool = True
    long_prefill_token_threshold: int = 0
    scheduling_policy: str = "decode_first"   # or "fair"
    max_prefill_per_batch: int = 0
    decode_latency_target_ms: int = 100
    preempt_prefill_on_latency: bool = True
    decode_reserved_tokens: int = 0


@dataclass
class OffloadConfig:
    offload_group_size: int = 0
    offload_num_in_group: int = 1
    offload_prefetch_step: int = 1
    kv_offloading_backend: str = "native"


@dataclass
class SpecConfig:
    method: str = ""                  # "", "draft", "mtp"
    draft_model: str = ""
    draft_n_max: int = 5
    draft_n_min: int = 0
    draft_p_min: float = 0.0
    tree: str = ""                    # e.g. "2,2,1" branching per depth; "" = linear chain


@dataclass
class ServerConfig:
    host: str = "0.0.0.0"
    port: int = 8000
    served_model_name: str = ""
    system_fingerprint: str = ""
    thread_pool_size: int = 8
    poll_interval_ms: int = 500
    step_interval_ms: int = 10
    default_max_tokens: int = 4096
    default_completion_max_tokens: int = 16


@dataclass
class VmCConfig:
    model: ModelConfig = field(default_factory=ModelConfig)
    cache: CacheConfig = field(default_factory=CacheConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)
    offload: OffloadConfig = field(default_factory=OffloadConfig)
    spec: SpecConfig = field(default_factory=SpecConfig)
    server: ServerConfig = field(default_factory=ServerConfig)

    def finalize(self) -> "VmCConfig":
        m = self.model
        if m.max_model_len <= 0:
            m.max_model_len = m.context_length
        m.max_model_len = max(16, m.max_model_len)
        if self.scheduler.max_num_batched_tokens <= 0:
            self.scheduler.max_num_batched_tokens = max(2048, m.max_model_len)
        if self.scheduler.max_num_batched_tokens < self.scheduler.max_num_seqs:
            raise ValueError(f"--max-num-batched-tokens ({self.scheduler.max_num_batched_tokens}) must be >= "
                             f"--max-num-seqs ({self.scheduler.max_num_seqs})")
        m.validate()
        return self

    def to_dict(self) -> dict:
        return asdict(self)


# ------------------------------------------------------------------------------------------------
# GGUF metadata -> ModelConfig


def _g(f, key, default=None):
    if not f.has(key):
        return default
    v = f.get(key)
    if isinstance(v, bytes):
        return v.decode("utf-8", "replace")
    return v


def model_config_from_gguf(f) -> ModelConfig:
    """Fill a ModelConfig from an opened GgufFile (vm_c_b200._native.host().GgufFile)."""
    arch = _g(f, "general.architecture", "llama")
    if arch == "qwen35moe":
        return _qwen35moe_config(f)
    if arch not in ("llama", "mixtral"):
        raise ValueError(f"unsupported GGUF architecture {arch!r} (supported: llama, mixtral)")
    a = "llama" if arch in ("llama", "mixtral") and f.has("llama.block_count") else arch
    m = ModelConfig(arch="llama")
    m.name = _g(f, "general.name", "") or ""
    m.n_layers = int(_g(f, f"{a}.block_count"))
    m.hidden = int(_g(f, f"{a}.embedding_length"))
    m.ffn = int(_g(f, f"{a}.feed_forward_length"))
    m.n_heads = int(_g(f, f"{a}.attention.head_count"))
    kvh = _g(f, f"{a}.attention.head_count_kv", m.n_heads)
    m.n_kv_heads = int(kvh[0] if isinstance(kvh, list) else kvh)
    m.head_dim = int(_g(f, f"{a}.attention.key_length", m.hidden // m.n_heads))
    m.rms_eps = float(_g(f, f"{a}.attention.layer_norm_rms_epsilon", 1e-5))
    m.rope_theta = float(_g(f, f"{a}.rope.freq_base", 10000.0))
    m.context_length = int(_g(f, f"{a}.context_length", 4096))
    m.n_experts = int(_g(f, f"{a}.expert_count", 0) or 0)
    m.n_experts_used = int(_g(f, f"{a}.expert_used_count", 0) or 0)
    st = _g(f, f"{a}.rope.scaling.type", None)
    if st and st != "none":
        m.rope_scaling = {"type": st, "factor": float(_g(f, f"{a}.rope.scaling.factor", 1.0)),
                          "original_context_length": int(_g(f, f"{a}.rope.scaling.original_context_length",
                                                             m.context_length))}
    tokens = f.get("tokenizer.ggml.tokens") if f.has("tokenizer.ggml.tokens") else None
    vocab = _g(f, f"{a}.vocab_size", None)
    if vocab is None:
        if tokens is not None:
            vocab = len(tokens)
        else:
            emb = [t for t in f.tensors() if t["name"] == "token_embd.weight"]
            vocab = emb[0]["ne"][1]
    m.vocab = int(vocab)
    m.bos_token_id = int(_g(f, "tokenizer.ggml.bos_token_id", 1))
    eos = _g(f, "tokenizer.ggml.eos_token_id", 2)
    m.eos_token_ids = [int(eos)]
    eot = _g(f, "tokenizer.ggml.eot_token_id", None)
    if eot is not None and int(eot) not in m.eos_token_ids:
        m.eos_token_ids.append(int(eot))
    names = {t["name"] for t in f.tensors()}
    m.tie_embeddings = "output.weight" not in names
    return m


def _qwen35moe_config(f) -> ModelConfig:
    """Hybrid Qwen3.5-MoE hyper-parameters (reference: src/official/llama/models/qwen35moe.cpp:5-42)."""
    a = "qwen35moe"
    m = ModelConfig(arch=a)
    m.name = _g(f, "general.name", "") or ""
    m.n_layers = int(_g(f, f"{a}.block_count"))
    m.hidden = int(_g(f, f"{a}.embedding_length"))
    m.n_heads = int(_g(f, f"{a}.attention.head_count"))
    kvh = _g(f, f"{a}.attention.head_count_kv", m.n_heads)
    m.n_kv_heads = int(kvh[0] if isinstance(kvh, list) else kvh)
    m.head_dim = int(_g(f, f"{a}.attention.key_length", m.hidden // m.n_heads))
    m.rms_eps = float(_g(f, f"{a}.attention.layer_norm_rms_epsilon", 1e-6))
    m.rope_theta = float(_g(f, f"{a}.rope.freq_base", 10000000.0))
    m.rope_neox = True
    m.rope_dims = int(_g(f, f"{a}.rope.dimension_count", m.head_dim))
    m.context_length = int(_g(f, f"{a}.context_length", 4096))
    m.n_experts = int(_g(f, f"{a}.expert_count", 0) or 0)
    m.n_experts_used = int(_g(f, f"{a}.expert_used_count", 0) or 0)
    ff = _g(f, f"{a}.feed_forward_length", 0) or 0
    m.ffn = int(_g(f, f"{a}.expert_feed_forward_length", 0) or (ff // max(1, m.n_experts_used)))
    m.ffn_shexp = int(_g(f, f"{a}.expert_shared_feed_forward_length", 0) or ff)
    m.ssm_conv = int(_g(f, f"{a}.ssm.conv_kernel"))
    m.ssm_state = int(_g(f, f"{a}.ssm.state_size"))
    m.ssm_k_heads = int(_g(f, f"{a}.ssm.group_count"))
    m.ssm_v_heads = int(_g(f, f"{a}.ssm.time_step_rank"))
    m.full_attn_interval = int(_g(f, f"{a}.full_attention_interval", 4))
    m.nextn_layers = int(_g(f, f"{a}.nextn_predict_layers", 0) or 0)
    if m.nextn_layers >= m.n_layers:
        raise ValueError("nextn_predict_layers must be smaller than block_count")
    names = {t["name"] for t in f.tensors()}
    tokens = f.get("tokenizer.ggml.tokens") if f.has("tokenizer.ggml.tokens") else None
    vocab = _g(f, f"{a}.vocab_size", None)
    if vocab is None:
        vocab = len(tokens) if tokens is not None else \
            [t for t in f.tensors() if t["name"] == "token_embd.weight"][0]["ne"][1]
    m.vocab = int(vocab)
    m.bos_token_id = int(_g(f, "tokenizer.ggml.bos_token_id", 1))
    m.eos_token_ids = [int(_g(f, "tokenizer.ggml.eos_token_id", 2))]
    m.tie_embeddings = "output.weight" not in names
    return m


def _hybrid_schedule(tc: dict, n_layers: int) -> int:
    """full_attention_interval of a config's layer schedule (0: no linear-attention layers)."""
    types = tc.get("layer_types")
    if types:
        if "linear_attention" not in types:
            return 0
        full = [i for i, t in enumerate(types) if t == "full_attention"]
        iv = full[0] + 1 if full else 0
        if not iv or any(types[i] != ("full_attention" if (i + 1) % iv == 0 else "linear_attention")
                         for i in range(len(types))):
            raise ValueError("layer_types: only a periodic schedule (every n-th layer full attention) is supported")
        return iv
    return int(tc["full_attention_interval"]) if tc.get("full_attention_interval") else 0


def model_config_from_hf(model_dir: str) -> ModelConfig:
    """ModelConfig from a HuggingFace config.json (reference: src/core/config.cpp:27-200, including the
    nested text_config, the expert-count spellings, the shared expert and the gated delta-net
    dimensions of hybrid models). Keys present with a null value count as absent."""
    cfg = json.loads((Path(model_dir) / "config.json").read_text())
    tc = cfg["text_config"] if isinstance(cfg.get("text_config"), dict) else cfg
    m = ModelConfig()
    m.arch = "llama"
    m.n_layers = tc["num_hidden_layers"]
    m.hidden = tc["hidden_size"]
    m.n_heads = tc["num_attention_heads"]
    m.n_kv_heads = tc.get("num_key_value_heads") or m.n_heads
    m.head_dim = tc.get("head_dim") or m.hidden // m.n_heads
    m.ffn = tc["intermediate_size"]
    m.vocab = tc.get("vocab_size") or cfg["vocab_size"]
    m.rms_eps = tc.get("rms_norm_eps") or 1e-5
    rp = tc.get("rope_parameters") if isinstance(tc.get("rope_parameters"), dict) else {}
    m.rope_theta = tc.get("rope_theta") or rp.get("rope_theta") or 10000.0
    m.rope_neox = True  # HF checkpoints keep the rotate-half layout
    m.rope_scaling = tc.get("rope_scaling")
    prf = tc.get("partial_rotary_factor") or rp.get("partial_rotary_factor")
    if prf:
        m.rope_dims = int(m.head_dim * float(prf))
    m.context_length = tc.get("max_position_embeddings") or 4096
    sw = tc.get("sliding_window")
    if sw and sw < m.context_length:
        # The attention kernels have no sliding-window mask; up to the window length full attention
        # equals windowed attention, so the context is capped there and outputs stay exact.
        m.context_length = int(sw)
    m.n_experts = tc.get("n_routed_experts") or tc.get("num_local_experts") or tc.get("num_experts") or 0
    m.n_experts_used = tc.get("num_experts_per_tok") or 0
    if m.n_experts and tc.get("moe_intermediate_size"):
        m.ffn = int(tc["moe_intermediate_size"])
    m.ffn_shexp = int(tc.get("shared_expert_intermediate_size") or 0)
    iv = _hybrid_schedule(tc, m.n_layers)
    if iv:
        m.arch = "qwen35moe"
        m.full_attn_interval = iv
        m.ssm_conv = int(tc.get("linear_conv_kernel_dim") or 4)
        kd, vd = tc.get("linear_key_head_dim"), tc.get("linear_value_head_dim")
        if kd and vd and kd != vd:
            raise ValueError("gated delta-net layers need equal key and value head dims")
        m.ssm_state = int(kd or vd or 0)
        m.ssm_k_heads = int(tc.get("linear_num_key_heads") or 0)
        m.ssm_v_heads = int(tc.get("linear_num_value_heads") or 0)
        m.nextn_layers = 0  # MTP blocks live outside num_hidden_layers in HF checkpoints
    m.bos_token_id = cfg.get("bos_token_id", tc.get("bos_token_id", 1)) or 1
    eos = cfg.get("eos_token_id", tc.get("eos_token_id", 2))
    m.eos_token_ids = list(eos) if isinstance(eos, list) else [eos]
    m.tie_embeddings = bool(cfg.get("tie_word_embeddings", tc.get("tie_word_embeddings", False)))
    return m


def rope_inv_freq(m: ModelConfig) -> list[float]:
    """Per-pair inverse frequencies, including Llama-3 style frequency scaling."""
    d = m.head_dim
    inv = [1.0 / (m.rope_theta ** (2 * i / d)) for i in range(d // 2)]
    sc = m.rope_scaling or {}
    typ = sc.get("rope_type", sc.get("type"))
    if typ == "llama3":
        factor = sc.get("factor", 8.0)
        lf, hf = sc.get("low_freq_factor", 1.0), sc.get("high_freq_factor", 4.0)
        old = sc.get("original_max_position_embeddings", sc.get("original_context_length", 8192))
        lw, hw = old / lf, old / hf
        out = []
        for f in inv:
            wl = 2 * math.pi / f
            if wl < hw:
                out.append(f)
            elif wl > lw:
                out.append(f / factor)
            else:
                s = (old / wl - lf) / (hf - lf)
                out.append((1 - s) * f / factor + s * f)
        inv = out
    elif typ == "linear":
        inv = [f / sc.get("factor", 1.0) for f in inv]
    return inv
