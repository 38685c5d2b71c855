"""``vm_c_server`` command line: the reference's CLI surface on the B200 engine.

Usage: python -m vm_c_b200.cli <model.gguf | random:preset[:mix[:seed]]> [options]

Flags and defaults follow the reference's parse_args (src/main.cpp:129-319) and config defaults
(include/vm_c/core/config.hpp:147-224). Added: --expert-parallel-size, --comm-backend,
--draft-model, --spec-tree, --num-gpu-blocks, --scheduling-policy. Flags the reference parses but
never uses (the kv-offloading and expert-cache groups) are accepted and reported as inactive.

Tensor parallelism runs one process per GPU: with --tensor-parallel-size N the CLI spawns N worker
processes (rank 0 serves HTTP and broadcasts each step's new requests to the others).

--native replaces this process with the PyTorch-free runtime's server (`vmc_run MODEL --serve`,
csrc/runtime/vmc_run.cpp + csrc/server/): one GPU, a Llama or Mixtral GGUF, bf16 paged KV. Options
that runtime does not have are refused with a message rather than ignored.
"""
from __future__ import annotations

import argparse
import os
import sys

from .config import VmCConfig


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="vm_c_server", description="OpenAI-compatible LLM server for B200")
    ap.add_argument("model", help="GGUF checkpoint path, a HuggingFace checkpoint directory (config.json + *.safetensors, "
                    "llama / mistral / mixtral), or random:<preset>[:<mix>[:<seed>]]")
    ap.add_argument("--tokenizer", default="", help="GGUF file whose vocabulary to use (default: the model's)")
    ap.add_argument("--kv-cache-dtype", default="auto",
                    choices=["auto", "float16", "bfloat16", "fp8_e4m3", "fp8_e5m2", "int8_per_token_head",
                             "fp8_per_token_head", "nvfp4", "turboquant_4bit_nc", "turboquant_k8v4",
                             "turboquant_k3v4_nc", "turboquant_3bit_nc"])
    ap.add_argument("--tq-rotation-seed", type=int, default=0,
                    help="TurboQuant: 0 = normalised Hadamard rotation; otherwise random sign flips per layer and "
                         "KV head before it (a seeded random orthogonal rotation)")
    ap.add_argument("--max-model-len", type=int, default=0)
    ap.add_argument("--gpu-memory-utilization", type=float, default=0.90)
    ap.add_argument("--gpu-safety-margin-mb", type=int, default=256)
    ap.add_argument("--num-gpu-blocks", type=int, default=0)
    ap.add_argument("--spec-method", default="", choices=["", "draft", "mtp", "none"])
    ap.add_argument("--spec-draft-n-max", type=int, default=5)
    ap.add_argument("--spec-draft-n-min", type=int, default=0)
    ap.add_argument("--spec-draft-p-min", type=float, default=0.0)
    ap.add_argument("--draft-model", default="")
    ap.add_argument("--spec-tree", default="", help="branching per draft depth, e.g. 2,2,1 (default: chain)")
    ap.add_argument("--tensor-parallel-size", "-tp", type=int, default=1)
    ap.add_argument("--expert-parallel-size", type=int, default=1)
    ap.add_argument("--gpu-devices", default="", help="comma-separated device ids")
    ap.add_argument("--comm-backend", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--served-model-name", default="")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--system-fingerprint", default="")
    ap.add_argument("--thread-pool-size", type=int, default=8)
    ap.add_argument("--poll-interval", type=int, default=500, help="ms")
    ap.add_argument("--cpu-offload-gb", type=float, default=0.0)
    ap.add_argument("--cpu-offload-params", default="")
    ap.add_argument("--max-num-seqs", type=int, default=128)
    ap.add_argument("--max-num-batched-tokens", type=int, default=0)
    g = ap.add_mutually_exclusive_group()
    g.add_argument("--enable-prefix-caching", dest="prefix_caching", action="store_true", default=True)
    g.add_argument("--disable-prefix-caching", dest="prefix_caching", action="store_false")
    g2 = ap.add_mutually_exclusive_group()
    g2.add_argument("--enable-chunked-prefill", dest="chunked_prefill", action="store_true", default=True)
    g2.add_argument("--disable-chunked-prefill", dest="chunked_prefill", action="store_false")
    ap.add_argument("--long-prefill-token-threshold", type=int, default=0)
    ap.add_argument("--scheduling-policy", default="decode_first", choices=["decode_first", "fair"])
    ap.add_argument("--native", action="store_true",
                    help="serve with the native runtime (vmc_run --serve: no Python or PyTorch in the server process)")
    # accepted for compatibility; inactive in the reference as well
    ap.add_argument("--kv-offloading-size", type=float, default=0.0)
    ap.add_argument("--kv-offloading-backend", default="native")
    ap.add_argument("--offload-group-size", type=int, default=0)
    ap.add_argument("--offload-prefetch-step", type=int, default=1)
    ap.add_argument("--expert-gpu-cache", type=int, default=0)
    ap.add_argument("--expert-cache-update-period", type=int, default=0)
    ap.add_argument("--expert-cache-history-window", type=int, default=0)
    return ap


def config_from_args(a) -> VmCConfig:
    cfg = VmCConfig()
    cfg.model.max_model_len = a.max_model_len
    c = cfg.cache
    c.kv_cache_dtype = a.kv_cache_dtype
    c.tq_rotation_seed = a.tq_rotation_seed
    c.gpu_memory_utilization = a.gpu_memory_utilization
    c.gpu_safety_margin_mb = a.gpu_safety_margin_mb
    c.num_gpu_blocks = a.num_gpu_blocks
    c.enable_prefix_caching = a.prefix_caching
    c.cpu_offload_gb = a.cpu_offload_gb
    c.cpu_offload_params = [p for p in a.cpu_offload_params.split(",") if p]
    c.kv_offloading_size = a.kv_offloading_size
    c.expert_gpu_cache_capacity = a.expert_gpu_cache
    c.expert_cache_update_period = a.expert_cache_update_period
    c.expert_cache_history_window = a.expert_cache_history_window
    p = cfg.parallel
    p.tensor_parallel_size = a.tensor_parallel_size
    p.expert_parallel_size = a.expert_parallel_size
    p.gpu_devices = [int(x) for x in a.gpu_devices.split(",") if x.strip()]
    p.comm_backend = a.comm_backend
    s = cfg.scheduler
    s.max_num_seqs = a.max_num_seqs
    s.max_num_batched_tokens = a.max_num_batched_tokens
    s.enable_chunked_prefill = a.chunked_prefill
    s.long_prefill_token_threshold = a.long_prefill_token_threshold
    s.scheduling_policy = a.scheduling_policy
    cfg.offload.offload_group_size = a.offload_group_size
    cfg.offload.offload_prefetch_step = a.offload_prefetch_step
    cfg.offload.kv_offloading_backend = a.kv_offloading_backend
    sp = cfg.spec
    sp.method = "" if a.spec_method == "none" else a.spec_method
    sp.draft_model = a.draft_model
    sp.draft_n_max = a.spec_draft_n_max
    sp.draft_n_min = a.spec_draft_n_min
    sp.draft_p_min = a.spec_draft_p_min
    sp.tree = a.spec_tree
    sv = cfg.server
    sv.host, sv.port = a.host, a.port
    sv.served_model_name = a.served_model_name
    sv.system_fingerprint = a.system_fingerprint
    sv.thread_pool_size = a.thread_pool_size
    sv.poll_interval_ms = a.poll_interval
    return cfg


def inactive_flags(a) -> list[str]:
    out = []
    if a.kv_offloading_size:
        out.append("--kv-offloading-size")
    if a.expert_gpu_cache:
        out.append("--expert-gpu-cache")
    if a.offload_group_size:
        out.append("--offload-group-size")
    return out


def run_rank(rank: int, world: int, a, cfg: VmCConfig) -> None:
    import torch
    from .llm import make_source
    from .utils.logging import get_logger
    log = get_logger("cli")
    devices = cfg.parallel.gpu_devices or list(range(world))
    dev = devices[rank]
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29517")
        os.environ["RANK"], os.environ["WORLD_SIZE"], os.environ["LOCAL_RANK"] = str(rank), str(world), str(dev)
    torch.cuda.set_device(dev)
    comm = None
    if world > 1:
        from .parallel.comm import NcclComm, init_distributed
        init_distributed()
        if cfg.parallel.comm_backend == "fused":
            from .parallel.fused import FusedComm
            comm = FusedComm()
        else:
            comm = NcclComm()
    src, mcfg = make_source(a.model, f"cuda:{dev}")
    mlen = cfg.model.max_model_len
    cfg.model = mcfg
    cfg.model.max_model_len = mlen
    cfg.finalize()
    log.info("resolved config: %s", cfg.to_dict())
    for f in inactive_flags(a):
        log.warning("%s is accepted for compatibility but has no effect", f)
    from .core.engine import LLMEngine
    from .models.runner import GpuModelRunner
    runner = GpuModelRunner(cfg, src, f"cuda:{dev}", rank, world, comm=comm)
    engine = LLMEngine(cfg, runner)
    runner.warmup()
    driver = None
    if world > 1:
        from .parallel.driver import StepDriver
        driver = StepDriver(engine)
    if rank != 0:
        driver.follow()
        return
    from .gguf.reader import GgufSource
    from .server.http import OpenAIServer, serve
    from .server.tokenizer import Tokenizer
    tok_src = GgufSource(a.tokenizer) if a.tokenizer else (src if hasattr(src, "metadata") else None)
    if tok_src is not None and not tok_src.metadata("tokenizer.ggml.tokens"):
        log.warning("%s has no tokenizer vocabulary; using a synthetic one (give --tokenizer)", a.tokenizer or a.model)
        tok_src = None
    if tok_src is None:
        from .gguf.random_init import synthetic_vocab
        toks, scores, types = synthetic_vocab(cfg.model.vocab)
        tokenizer = Tokenizer(toks, scores, types, [], "llama", "gpt2", cfg.model.bos_token_id,
                              cfg.model.eos_token_ids, True)
    else:
        tokenizer = Tokenizer.from_gguf(tok_src)
    name = cfg.server.served_model_name or os.path.basename(os.path.normpath(a.model))
    srv = OpenAIServer(engine, tokenizer, name, cfg.server, driver=driver)
    serve(srv, cfg.server.host, cfg.server.port)


def native_argv(a) -> list[str]:
    """The `vmc_run --serve` command line for these options; ValueError for an option it lacks."""
    from ._build import EXT_DIR
    bad = []
    if a.tensor_parallel_size > 1 or a.expert_parallel_size > 1:
        bad.append("tensor / expert parallelism")
    if a.spec_method not in ("", "none") or a.draft_model:
        bad.append("speculative decoding")
    if a.kv_cache_dtype not in ("auto", "bfloat16"):
        bad.append(f"--kv-cache-dtype {a.kv_cache_dtype}")
    if a.cpu_offload_gb or a.cpu_offload_params:
        bad.append("CPU weight offload")
    if a.tokenizer:
        bad.append("--tokenizer")
    if a.scheduling_policy != "decode_first" or not a.chunked_prefill or not a.prefix_caching:
        bad.append("scheduler policy options")
    if a.model.startswith("random:") or os.path.isdir(a.model):
        bad.append("random: and HuggingFace checkpoints (the native runtime reads GGUF files)")
    if bad:
        raise ValueError("--native does not support: " + "; ".join(bad))
    argv = [str(EXT_DIR / "runtime" / "vmc_run"), a.model, "--serve", "--host", a.host, "--port", str(a.port),
            "--max-num-seqs", str(a.max_num_seqs)]
    if a.served_model_name:
        argv += ["--model-name", a.served_model_name]
    if a.max_num_batched_tokens > 0:
        argv += ["--max-num-batched-tokens", str(a.max_num_batched_tokens)]
    if a.max_model_len > 0:
        argv += ["--max-model-len", str(a.max_model_len)]
    if a.num_gpu_blocks > 0:
        argv += ["--num-blocks", str(a.num_gpu_blocks)]
    return argv


def main(argv=None) -> None:
    a = build_parser().parse_args(argv)
    if a.native:
        try:
            args = native_argv(a)
        except ValueError as e:
            raise SystemExit(str(e))
        if not os.path.exists(args[0]):
            from ._build import build_runtime
            build_runtime()
        if a.gpu_devices:
            os.environ["CUDA_VISIBLE_DEVICES"] = a.gpu_devices.split(",")[0]
        os.execv(args[0], args)
    cfg = config_from_args(a)
    world = cfg.parallel.tensor_parallel_size
    if world <= 1:
        run_rank(0, 1, a, cfg)
        return
    import torch.multiprocessing as mp
    mp.spawn(run_rank, args=(world, a, cfg), nprocs=world, join=True)


if __name__ == "__main__":
    main(sys.argv[1:])
