"""User-facing entry point: ``LLM(model, ...)`` builds config, weights, runner and engine on this rank.

``model`` is a GGUF path, a HuggingFace checkpoint directory (config.json + *.safetensors; BF16 / F16 /
F32 weights run as bf16 tiles), or ``random:<preset>[:<mix>[:<seed>]]`` for a seeded random-init model
of a benchmark architecture generated on the GPU (e.g. ``random:llama3-8b:Q4_K_M``).
"""
from __future__ import annotations

from typing import Optional

from .config import VmCConfig
from .core.engine import LLMEngine
from .core.sampling_params import RequestOutput, SamplingParams


def make_source(model: str, device="cuda"):
    if model.startswith("random:"):
        from .gguf.random_init import GpuRandomSource, preset
        parts = model.split(":")
        name = parts[1]
        mix = parts[2] if len(parts) > 2 else "Q8_0"
        seed = int(parts[3]) if len(parts) > 3 else 0
        cfg = preset(name)
        return GpuRandomSource(cfg, mix, seed, device), cfg
    import os
    if os.path.isdir(model) or model.endswith(".safetensors"):
        from .hf.source import HfSource
        src = HfSource(model)
        return src, src.model_config()
    from .gguf.reader import GgufSource
    src = GgufSource(model)
    return src, src.model_config()


class LLM:
    def __init__(self, model: str, *, max_model_len: int = 0, max_num_seqs: int = 128,
                 max_num_batched_tokens: int = 0, num_gpu_blocks: int = 0, gpu_memory_utilization: float = 0.9,
                 enable_prefix_caching: bool = True, enable_chunked_prefill: bool = True,
                 long_prefill_token_threshold: int = 0, scheduling_policy: str = "decode_first",
                 use_cuda_graphs: bool = True, device: Optional[str] = None, tp_rank: int = 0, tp_size: int = 1,
                 ep_size: int = 1, kv_cache_dtype: str = "auto", tq_rotation_seed: int = 0, draft_model: str = "",
                 num_speculative_tokens: int = 5, spec_tree: str = "", cpu_offload_gb: float = 0.0,
                 cpu_offload_params=(),
                 comm=None, config: Optional[VmCConfig] = None, warmup: bool = True):
        import torch
        dev = device or (f"cuda:{torch.cuda.current_device()}" if torch.cuda.is_available() else "cuda")
        src, mcfg = make_source(model, dev)
        cfg = config or VmCConfig()
        cfg.model = mcfg
        if max_model_len:
            cfg.model.max_model_len = max_model_len
        cfg.scheduler.max_num_seqs = max_num_seqs
        cfg.scheduler.max_num_batched_tokens = max_num_batched_tokens
        cfg.scheduler.enable_chunked_prefill = enable_chunked_prefill
        cfg.scheduler.long_prefill_token_threshold = long_prefill_token_threshold
        cfg.scheduler.scheduling_policy = scheduling_policy
        cfg.cache.num_gpu_blocks = num_gpu_blocks
        cfg.cache.gpu_memory_utilization = gpu_memory_utilization
        cfg.cache.enable_prefix_caching = enable_prefix_caching
        if cpu_offload_gb:
            cfg.cache.cpu_offload_gb = cpu_offload_gb
            cfg.cache.cpu_offload_params = list(cpu_offload_params)
        if config is None or kv_cache_dtype != "auto":
            cfg.cache.kv_cache_dtype = kv_cache_dtype
        if config is None or tq_rotation_seed:
            cfg.cache.tq_rotation_seed = tq_rotation_seed
        if draft_model:
            cfg.spec.method = "draft"
            cfg.spec.draft_model = draft_model
            cfg.spec.draft_n_max = num_speculative_tokens
            cfg.spec.tree = spec_tree
        cfg.parallel.tensor_parallel_size = tp_size
        cfg.parallel.expert_parallel_size = ep_size
        cfg.finalize()
        self.cfg = cfg
        self.source = src
        from .models.runner import GpuModelRunner
        self.runner = GpuModelRunner(cfg, src, dev, tp_rank, tp_size, comm=comm, use_graphs=use_cuda_graphs)
        self.engine = LLMEngine(cfg, self.runner)
        if warmup:
            self.runner.warmup()

    def generate(self, prompt_token_ids: list[list[int]],
                 params: SamplingParams | list[SamplingParams] | None = None) -> list[RequestOutput]:
        return self.engine.generate(prompt_token_ids, params)

    def shutdown(self) -> None:
        self.runner.release_graphs()
