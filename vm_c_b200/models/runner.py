"""GPU model runner: owns weights, KV cache, step buffers and the decode CUDA graphs of one rank.

Replaces the reference's per-rank LlamaRuntime + ggml CUDA-graph machinery
(src/official/llama_runtime.cpp:178-538, ggml-cuda.cu:4308-4520): decode-only steps replay a CUDA
graph captured per batch-size bucket (the whole layer stack, lm_head and sampler in one graph);
prefill / mixed steps run the same kernels eagerly. Per step there is one pinned H2D copy of the
metadata written by the native scheduler, one of the sampling parameters, and one D2H copy of the
sampled ids followed by an event wait.
"""
from __future__ import annotations

import math
import time
from typing import Optional

import numpy as np
import torch

from .. import ops
from ..config import VmCConfig
from ..core.engine import ModelRunner, StepCounts
from ..utils.logging import get_logger
from .llama import LlamaModel, StepMeta, load_weights

log = get_logger("runner")

GRAPH_BUCKETS = [1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256]


def kv_bytes_per_block(cfg: VmCConfig, hkv_local: int, dtype_bytes: int = 2, n_layers: int = 0) -> int:
    """KV bytes of one block over the layers that keep a KV cache (all layers unless n_layers is given:
    the full-attention layers of a hybrid model)."""
    m = cfg.model
    L = n_layers or m.n_layers
    if is_turboquant(cfg.cache.kv_cache_dtype):
        from .. import _native
        slot = _native.host().tq_layout(cfg.cache.kv_cache_dtype, m.head_dim)["slot_aligned"]
        return L * cfg.cache.block_size * hkv_local * slot
    return L * 2 * hkv_local * cfg.cache.block_size * m.head_dim * dtype_bytes


def is_turboquant(kv_cache_dtype: str) -> bool:
    return kv_cache_dtype.startswith("turboquant")


def check_kv_cache_dtype(kv_cache_dtype: str) -> None:
    """bf16 pages (auto / bfloat16) and the four TurboQuant layouts are implemented; the other
    names the reference's flag accepts are rejected here instead of silently served as bf16."""
    ok = ("auto", "bfloat16", "bf16", "turboquant_4bit_nc", "turboquant_k8v4", "turboquant_k3v4_nc",
          "turboquant_3bit_nc")
    if kv_cache_dtype not in ok:
        raise ValueError(f"--kv-cache-dtype {kv_cache_dtype!r} is not supported (supported: {', '.join(ok)})")


class GpuModelRunner(ModelRunner):
    def __init__(self, cfg: VmCConfig, source, device="cuda", tp_rank: int = 0, tp_size: int = 1, comm=None,
                 use_graphs: bool = True, weights=None):
        self.cfg = cfg
        self.dev = torch.device(device)
        torch.cuda.set_device(self.dev)
        self.tp_rank, self.tp_size = tp_rank, tp_size
        m = cfg.model
        t0 = time.perf_counter()
        self.weights = weights if weights is not None else load_weights(source, m, self.dev, tp_rank, tp_size,
                                                                                 cfg.parallel.expert_parallel_size)
        log.info("weights loaded: %.2f GB in %.1fs", self.weights.bytes_total / 1e9, time.perf_counter() - t0)
        from .offload import apply_offload
        self.offload = apply_offload(self.weights, cfg.cache.cpu_offload_gb, cfg.cache.cpu_offload_params, self.dev)
        s = cfg.scheduler
        self.max_model_len = m.max_model_len
        sp = cfg.spec
        if sp.method == "mtp":
            raise ValueError("--spec-method mtp needs next-n prediction layers, which the supported model "
                             "families do not have; use --spec-method draft --draft-model <gguf>")
        self.spec_tree = [int(x) for x in sp.tree.split(",") if x.strip()] if (sp.method == "draft" and sp.tree) else []
        if self.spec_tree:
            from ..speculative.tree import TokenTree
            self.spec_k = TokenTree(self.spec_tree).N - 1   # look-ahead slots: every non-root tree node
        else:
            self.spec_k = sp.draft_n_max if sp.method == "draft" else 0
        self.num_lookahead_tokens = self.spec_k
        max_seqs = max(s.max_num_seqs, 1)
        # Sampled rows: one per request, or k + 1 per request when speculative verification runs.
        self.max_samples = max_seqs * (1 + self.spec_k)
        self.max_tokens = max(s.max_num_batched_tokens, self.max_samples)
        self.buckets = [b for b in GRAPH_BUCKETS if b <= max_seqs]
        if use_graphs and self.buckets and self.buckets[-1] < max_seqs:
            self.buckets.append(max_seqs)
        from ..utils.trace import HiddenTracer
        self.tracer = HiddenTracer.from_env()
        if self.tracer is not None and use_graphs:
            log.warning("VMC_LOG_HIDDEN / VMC_LOG_LOGITS set: decode steps run eagerly (no CUDA graphs)")
            use_graphs = False
        if m.is_hybrid:
            # Qwen3.5-MoE: one GPU, eager steps, bf16 KV, no speculation or offload (models/qwen35.py)
            if sp.method:
                raise ValueError("speculative decoding is not implemented for GGUF architecture 'qwen35moe'")
            if is_turboquant(cfg.cache.kv_cache_dtype):
                raise ValueError("TurboQuant KV caches are not implemented for GGUF architecture 'qwen35moe'")
            if cfg.cache.cpu_offload_gb > 0:
                raise ValueError("CPU weight offload is not implemented for GGUF architecture 'qwen35moe'")
            use_graphs = False
        self.use_graphs = use_graphs
        if m.is_hybrid:
            from .qwen35 import HybridModel
            self.model = HybridModel(self.weights, self.max_tokens, self.max_samples, m.max_model_len, max_seqs)
        else:
            self.model = LlamaModel(self.weights, self.max_tokens, self.max_samples, m.max_model_len + self.spec_k,
                                    comm=comm, attn_splits=16)
        self.comm = comm
        sms = torch.cuda.get_device_properties(self.dev).multi_processor_count
        self._decode_slots = sms * max(1, ops.C().attn_decode_ctas_per_sm(self.model.D))
        # KV cache: bf16 [L, num_blocks, 2, Hkv_local, block_size, D], or TurboQuant slots
        # uint8 [L, num_blocks, block_size, Hkv_local, slot]; zero-filled (finite).
        check_kv_cache_dtype(cfg.cache.kv_cache_dtype)
        self.tq = None
        if is_turboquant(cfg.cache.kv_cache_dtype):
            self.tq = ops.TqTables(cfg.cache.kv_cache_dtype, m.head_dim, self.dev, rot_seed=cfg.cache.tq_rotation_seed)
        self.model.tq = self.tq
        self.model.tracer = self.tracer
        n_kv_layers = getattr(self.model, "n_kv_layers", m.n_layers)
        per_block = kv_bytes_per_block(cfg, self.model.hkv, n_layers=n_kv_layers)
        max_blocks_per_seq = (m.max_model_len + cfg.cache.block_size - 1) // cfg.cache.block_size + 1
        want = cfg.cache.num_gpu_blocks
        if want <= 0:
            torch.cuda.synchronize(self.dev)
            free, total = torch.cuda.mem_get_info(self.dev)
            budget = int(total * cfg.cache.gpu_memory_utilization) - (total - free) \
                - cfg.cache.gpu_safety_margin_mb * (1 << 20) - (1 << 30)
            want = max(16, budget // per_block)
            want = min(want, 2 * s.max_num_seqs * max_blocks_per_seq + 1)
        self.num_kv_blocks = int(want)
        if self.tq is None:
            self.kv = torch.zeros(n_kv_layers, self.num_kv_blocks, 2, self.model.hkv, cfg.cache.block_size,
                                  m.head_dim, dtype=torch.bfloat16, device=self.dev)
        else:
            self.kv = torch.zeros(m.n_layers, self.num_kv_blocks, cfg.cache.block_size, self.model.hkv,
                                  self.tq.slot_bytes, dtype=torch.uint8, device=self.dev)
        self.kv_bytes_per_token = per_block // cfg.cache.block_size
        log.info("KV cache (%s): %d blocks x %d tokens (%.2f GB, %d bytes/token on this rank)",
                 cfg.cache.kv_cache_dtype, self.num_kv_blocks, cfg.cache.block_size,
                 self.kv.numel() * self.kv.element_size() / 1e9, self.kv_bytes_per_token)
        self.params_dev = torch.zeros(self.max_tokens * 40, dtype=torch.uint8, device=self.dev)
        self.params_host = torch.zeros(self.max_tokens * 40, dtype=torch.uint8).pin_memory()
        self.tok_dev = torch.zeros(self.max_tokens, dtype=torch.int32, device=self.dev)
        self.lp_dev = torch.zeros(self.max_tokens, dtype=torch.float32, device=self.dev)
        self.tok_host = torch.zeros(self.max_tokens, dtype=torch.int32).pin_memory()
        self.lp_host = torch.zeros(self.max_tokens, dtype=torch.float32).pin_memory()
        self.done = torch.cuda.Event()
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_launches: dict[int, int] = {}
        self.launch_count = 0      # kernels of this framework launched by executed steps
        self.h2d_bytes = 0         # per-step inputs copied from pinned host memory
        self.d2h_bytes = 0         # per-step results read back
        self.meta_dev: Optional[torch.Tensor] = None
        self.layout = None
        self.stream = torch.cuda.current_stream(self.dev)

    # -- engine hooks ------------------------------------------------------------------------------
    def max_graph_batch(self) -> int:
        return self.buckets[-1] if (self.use_graphs and self.buckets) else 0

    def graph_bucket(self, R: int) -> int:
        if not self.use_graphs:
            return 0
        for b in self.buckets:
            if b >= R:
                return b
        return 0

    def alloc_meta(self, total: int) -> torch.Tensor:
        self.meta_host = torch.zeros(total, dtype=torch.int32).pin_memory()
        self.meta_dev = torch.zeros(total, dtype=torch.int32, device=self.dev)
        return self.meta_host

    def bind_layout(self, layout) -> None:
        self.layout = layout
        if self.spec_k and self.spec is None:
            self._init_spec()
        L = layout
        md = self.meta_dev
        self.v_ids = md[L.off_input_ids:L.off_input_ids + L.max_tokens]
        self.v_pos = md[L.off_positions:L.off_positions + L.max_tokens]
        self.v_slots = md[L.off_slot_mapping:L.off_slot_mapping + L.max_tokens]
        self.v_qs = md[L.off_q_start:L.off_q_start + L.max_reqs + 1]
        self.v_ctx = md[L.off_ctx_len:L.off_ctx_len + L.max_reqs]
        self.v_lidx = md[L.off_logits_idx:L.off_logits_idx + L.max_reqs]
        self.v_sslot = md[L.off_seq_slot:L.off_seq_slot + L.max_reqs]
        self.v_bt = md[L.off_block_tables:L.off_block_tables + L.max_reqs * L.max_blocks_per_seq].view(
            L.max_reqs, L.max_blocks_per_seq)

    # -- speculative decoding ------------------------------------------------------------------------
    spec = None

    def _init_spec(self) -> None:
        from .. import _native
        from ..llm import make_source
        from ..speculative.draft import DraftSpeculator
        from ..speculative.tree import TreeSpeculator
        sp = self.cfg.spec
        if not sp.draft_model:
            raise ValueError("--spec-method draft needs --draft-model")
        src, dcfg = make_source(sp.draft_model, str(self.dev))
        spec_layout = _native.host().BatchLayout(self.max_tokens, self.max_samples, self.layout.max_blocks_per_seq)
        self.tok_spec = torch.zeros(self.max_samples, dtype=torch.int32, device=self.dev)
        self.tok_spec_host = torch.zeros(self.max_samples, dtype=torch.int32).pin_memory()
        if self.spec_tree:
            if self.tq is not None:
                raise ValueError("token-tree speculation needs a bf16 KV cache (the accepted branch is moved in place)")
            self.spec = TreeSpeculator(self, src, dcfg, self.spec_tree, comm=self.comm, layout=spec_layout)
            log.info("speculative decoding: draft %s, token tree %s (%d nodes)", sp.draft_model, self.spec_tree,
                     self.spec_k + 1)
        else:
            self.spec = DraftSpeculator(self, src, dcfg, self.spec_k, comm=self.comm, layout=spec_layout)
            log.info("speculative decoding: draft %s, k = %d", sp.draft_model, self.spec_k)

    def _meta(self, T, R, S, nd, max_qlen) -> StepMeta:
        return StepMeta(self.v_ids, self.v_pos, self.v_slots, self.v_qs, self.v_ctx, self.v_bt, self.v_lidx,
                        T=T, R=R, S=S, num_decode=nd, max_qlen=max_qlen, seq_slot=self.v_sslot)

    def _attn_splits(self, nd: int) -> int:
        return ops.decode_splits(nd * self.model.hkv, self._decode_slots)

    def _forward(self, m: StepMeta, pen=None) -> None:
        self.model.attn_splits = self._attn_splits(m.num_decode)
        params = self.params_dev
        self.model.forward(self.kv, m, params, self.tok_dev, self.lp_dev, pre_sample=pen)

    def _upload(self, meta: torch.Tensor, params: np.ndarray) -> None:
        nb = params.nbytes
        self.params_host[:nb].numpy()[:] = params.view(np.uint8)
        self.meta_dev.copy_(meta, non_blocking=True)
        self.params_dev[:nb].copy_(self.params_host[:nb], non_blocking=True)

    def execute(self, meta, counts: StepCounts, params: np.ndarray, penalties=None):
        return self.wait(self.launch(meta, counts, params, penalties))

    def synchronize(self) -> None:
        torch.cuda.synchronize(self.dev)

    def wait(self, S: int):
        """Block until the launched step's sampled ids are on the host."""
        self.done.synchronize()
        return self.tok_host[:S].numpy().copy(), self.lp_host[:S].numpy().copy()

    def launch(self, meta, counts: StepCounts, params: np.ndarray, penalties=None) -> int:
        """Issue one step (uploads, kernels, read-back of the sampled ids) without waiting for it."""
        if counts.R_pad > 0 and penalties is None and counts.R_pad not in self.graphs:
            self._capture(counts.R_pad)   # before the upload: capture uses the device buffers
        self._upload(meta, params)
        pen = None
        if penalties is not None:
            if self.tp_size > 1:
                # the lm_head is vocabulary-parallel: this rank's logits hold tokens [v0, v1) only
                v0, v1 = self.model.w.vocab_begin, self.model.w.vocab_end
                rows_np, toks_np, cnts_np = penalties
                keep = (toks_np >= v0) & (toks_np < v1)
                penalties = (rows_np[keep], (toks_np[keep] - v0).astype(np.int32), cnts_np[keep])
            rows, toks, cnts = (torch.from_numpy(np.ascontiguousarray(a)).to(self.dev, non_blocking=True)
                                for a in penalties)
            n = rows.numel()

            def pen(model):  # applied to the logits before sampling
                ops.apply_penalties(model.ws.logits, rows, toks, cnts, self.params_dev, n)
        if counts.R_pad > 0 and pen is None:
            B = counts.R_pad
            g = self.graphs.get(B)
            if g is None:
                g = self._capture(B)
            g.replay()
            self.launch_count += self.graph_launches[B]
            S = counts.S
        else:
            n0 = ops.LAUNCHES[0]
            self._forward(self._meta(counts.T, counts.R, counts.S, counts.num_decode, counts.max_qlen), pen)
            self.launch_count += ops.LAUNCHES[0] - n0
            S = counts.S
        if self.tracer is not None:
            self.tracer.flush()
        self.tok_host[:S].copy_(self.tok_dev[:S], non_blocking=True)
        self.lp_host[:S].copy_(self.lp_dev[:S], non_blocking=True)
        self.h2d_bytes += meta.numel() * 4 + params.nbytes
        self.d2h_bytes += S * 8
        self.done.record()
        return S

    def full_logits(self, S: int):
        """Host copy of the last step's full-vocabulary logits of its S sampled rows (after any
        penalties): the gathered vocabulary shards under tensor parallelism."""
        if self.tp_size > 1:
            return self.comm.gather_logits(self.model, S).float().cpu()
        return self.model.ws.logits[:S].float().cpu()

    # -- CUDA graphs -------------------------------------------------------------------------------
    def _fake_decode_meta(self, B: int) -> None:
        """Metadata for a batch of B padding decode rows (no KV writes, empty contexts)."""
        L = self.layout
        h = np.zeros(L.total, dtype=np.int32)
        h[L.off_slot_mapping:L.off_slot_mapping + B] = -1
        h[L.off_q_start:L.off_q_start + B + 1] = np.arange(B + 1)
        h[L.off_logits_idx:L.off_logits_idx + B] = np.arange(B)
        self.meta_dev.copy_(torch.from_numpy(h))
        self.params_dev.zero_()

    def _capture(self, B: int) -> torch.cuda.CUDAGraph:
        self._fake_decode_meta(B)
        m = self._meta(B, B, B, B, 1)
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._forward(m)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        n0 = ops.LAUNCHES[0]
        with torch.cuda.graph(g, stream=s):
            self._forward(m)
        self.graph_launches[B] = ops.LAUNCHES[0] - n0
        torch.cuda.synchronize(self.dev)
        self.graphs[B] = g
        return g

    def warmup(self, capture: bool = True) -> None:
        """Compile-free warm-up: one eager prefill-shaped step and capture of every decode bucket."""
        if capture and self.use_graphs:
            t0 = time.perf_counter()
            for B in self.buckets:
                if B not in self.graphs:
                    self._capture(B)
            log.info("captured %d decode graphs in %.1fs", len(self.graphs), time.perf_counter() - t0)

    def release_graphs(self) -> None:
        self.graphs.clear()
        torch.cuda.synchronize(self.dev)
