"""Headline benchmark: output tokens/s of the serving engine on BASELINE config 2.

Config: Llama-3-8B architecture, random-init Q4_K_M weights (generated on the device in GGUF block
format), 64 concurrent requests, each a 1024-token uniform-random prompt with 256 greedy output
tokens, paged KV block size 16 with bf16 KV, tensor parallel over N GPUs (one process per GPU).

One bench "step" = one complete serving run of the 64 requests (continuous batching with chunked
prefill, decode-first scheduling) through the engine; fresh random prompts every run (no prefix
cache reuse). W untimed runs, then K timed runs bracketed by barrier + synchronize, timed with CUDA
events on the launching stream, max over ranks. value = total output tokens / time (whole job).

`--impl reference` runs the reference (houjiaxxin/vm_c) through its own public API, or reports why
it cannot.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "output tok/s (box, device-timed, max over ranks) @TP1/2/4/8; p50 TTFT/ITL"
MODEL = "Llama-3-8B (random-init, Q4_K_M GGUF)"
REF_EXE = os.path.join(ROOT, "baseline", "_ref", "vmc_ref_bench")
REFERENCE_TP_UNAVAILABLE = (
    "the reference's multi-GPU path is its full engine (TPRuntime + NcclComm, src/distributed/), which does not "
    "build as shipped: src/model/gguf_model_loader.cpp:6,11 include vm_c/model/tensor_schema.hpp and "
    "vm_c/vmc_engine/ggml_weight.hpp, which do not exist (TensorSchema, ShardContext, TpShardMode and "
    "compute_quant_alloc_bytes are defined nowhere); its single-GPU forward (vendored libllama + ggml-cuda) is "
    "what the N=1 reference arm runs")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="random:llama3-8b:Q4_K_M:0")
    ap.add_argument("--num-reqs", type=int, default=64)
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--gen-len", type=int, default=256)
    ap.add_argument("--max-num-batched-tokens", type=int, default=2048)
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--comm", default=os.environ.get("VMC_COMM", "fused"), choices=["nccl", "fused"])
    ap.add_argument("--e2e-steps", type=int, default=1)
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5],
                    help="BASELINE.json config: 2 Llama-3-8B Q4_K_M (default, the headline), 3 Llama-3-70B Q8_0 with "
                         "TurboQuant KV, 4 Mixtral-8x7B Q4_K expert-parallel, 5 speculative decoding (draft model, tree)")
    ap.add_argument("--kv-cache-dtype", default="")
    ap.add_argument("--moe-mode", default="a2a", choices=["a2a", "allreduce"],
                    help="config 4: expert-parallel all-to-all over peer memory, or the partial-sum all-reduce")
    ap.add_argument("--spec-tree", default="2,2,1", help="config 5: token-tree branching per depth")
    ap.add_argument("--self-draft", action="store_true", help="config 5: the target drafts for itself (upper bound)")
    a = ap.parse_args()
    cfgs = {3: ("random:llama3-70b:Q8_0:0", 128, 2048, 512), 4: ("random:mixtral-8x7b:Q4_K:0", 256, 512, 256),
            5: ("random:llama3-8b:BF16:0", 32, 512, 256)}
    if a.config in cfgs:
        m, R, P, G = cfgs[a.config]
        a.model = m if a.model == "random:llama3-8b:Q4_K_M:0" else a.model
        a.num_reqs, a.prompt_len, a.gen_len = R, P, G
    if a.config == 3 and not a.kv_cache_dtype:
        a.kv_cache_dtype = "turboquant_4bit_nc"
    if a.config == 4 and a.moe_mode == "allreduce":
        a.comm = "nccl"
    return a


WEIGHTS = {2: "Q4_K_M", 3: "Q8_0", 4: "Q4_K", 5: "BF16 (target) and Q8_0 (draft)"}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.path = tempfile.mktemp(prefix="vmc_clocks_", suffix=".csv")
        self.p = None

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.close()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "samples": len(sm),
                "reasons": sorted(reasons)}


def reference_arm(args):
    """The reference through its own forward-pass API: its vendored libllama + ggml-cuda, built offline from
    the reference tree by baseline/build_ref.sh into baseline/_ref, driven by baseline/ref_bench.cpp (decode-
    first continuous batching of the same workload, the reference engine's GPU sampler). Nothing of this
    repository's engine, models or kernels is loaded in this process or the driver."""
    import numpy as np
    base = {"impl": "reference", "metric": METRIC, "n_gpus": args.gpus}
    if args.gpus > 1:
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({**base, "unavailable": REFERENCE_TP_UNAVAILABLE}), flush=True)
        return
    if not os.path.exists(REF_EXE):
        print(json.dumps({**base, "unavailable": "reference arm not built (run baseline/build_ref.sh)"}), flush=True)
        return
    R, P, G = args.num_reqs, args.prompt_len, args.gen_len
    tmp = tempfile.mkdtemp(prefix="vmc_ref_")
    gguf = os.path.join(tmp, "model.gguf")
    preset, mix = (args.model.split(":") + ["", "", ""])[1:3]
    def failed(what, r):
        tail = " | ".join((r.stderr or "").strip().splitlines()[-3:])
        print(json.dumps({**base, "unavailable": f"reference {what} failed (rc {r.returncode}): {tail}"}), flush=True)

    r = subprocess.run([REF_EXE, "gen", "--preset", preset or "llama3-8b", "--mix", mix or "Q4_K_M", "--seed", "0",
                        "--out", gguf], capture_output=True, text=True)
    if r.returncode != 0:
        return failed("checkpoint generation", r)
    rng = np.random.default_rng(1_000)
    prompts = rng.integers(0, 128256 if (preset or "llama3-8b") == "llama3-8b" else 32000, (R, P)).astype(np.int32)
    pfile = os.path.join(tmp, "prompts.bin")
    with open(pfile, "wb") as f:
        f.write(np.asarray([R, P], np.int32).tobytes())
        f.write(prompts.tobytes())
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    clocks.start()
    t0 = time.perf_counter()
    out = subprocess.run([REF_EXE, "bench", "--model", gguf, "--prompts", pfile, "--gen", str(G), "--batch",
                          str(args.max_num_batched_tokens), "--runs", str(args.steps), "--warmup", str(args.warmup)],
                         capture_output=True, text=True)
    wall = time.perf_counter() - t0
    clk = clocks.stop()
    if out.returncode != 0:
        os.unlink(gguf)
        return failed("serving run", out)
    r = json.loads([ln for ln in out.stdout.splitlines() if ln.startswith("{")][-1])
    os.unlink(gguf)
    value = r["tok_per_s"]
    line = {**base, "value": value, "unit": "output tokens/s", "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": r["ms_per_run"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16 KV, Q4_K_M weights (ggml-cuda kernels)",
            "data": "synthetic: random-init Q4_K_M GGUF written by the reference's own ggml quantisers; "
                    "uniform-random prompt token ids (seeded)",
            "config": {"model": MODEL, "global_batch": R, "seq_len": P, "gen_len": G, "parallelism": "tp1",
                       "kv_cache": "bf16 (libllama cache)", "max_num_batched_tokens": args.max_num_batched_tokens,
                       "path": "reference libllama llama_decode + ggml-cuda, reference GPU sampler",
                       "l2": "inputs larger than L2 (4.9 GB weights + KV streamed every step)",
                       "step": "one full serving run of global_batch requests"},
            "p50_ttft_ms": r["p50_ttft_ms"], "p50_itl_ms": r["p50_itl_ms"],
            "e2e": {"value": round(args.steps * R * G / r["ms_wall_total"] * 1e3, 2),
                    "unit": "output tokens/s (host wall clock of the timed runs)",
                    "h2d_bytes_per_step": r["h2d_bytes_per_run"], "d2h_bytes_per_step": r["d2h_bytes_per_run"]},
            "gpu_launches": None, "clocks": clk, "process_wall_s": round(wall, 1)}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    import numpy as np
    import torch
    import torch.distributed as dist

    from vm_c_b200 import ops
    from vm_c_b200.core.sampling_params import SamplingParams
    from vm_c_b200.llm import LLM
    from vm_c_b200.parallel.comm import NcclComm, init_distributed

    rank, world, local = init_distributed()
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"
    torch.cuda.set_device(local)
    comm = None
    if world > 1:
        if args.comm == "fused":
            from vm_c_b200.parallel.fused import FusedComm
            comm = FusedComm()
        else:
            comm = NcclComm()
    R, P, G = args.num_reqs, args.prompt_len, args.gen_len
    max_len = P + G + 16
    extra = {}
    if args.kv_cache_dtype:
        extra["kv_cache_dtype"] = args.kv_cache_dtype
    if args.config == 4:
        extra["ep_size"] = world
    if args.config == 5:
        extra.update(draft_model=args.model if args.self_draft else "random:draft-16l-2048:Q8_0:0",
                     spec_tree=args.spec_tree, num_speculative_tokens=5)
    llm = LLM(args.model, max_model_len=max(2048, max_len), max_num_seqs=R,
              max_num_batched_tokens=args.max_num_batched_tokens, num_gpu_blocks=R * ((max_len + 15) // 16 + 4) + 64,
              enable_prefix_caching=True, use_cuda_graphs=not args.no_graphs, tp_rank=rank, tp_size=world, comm=comm,
              device=f"cuda:{local}", **extra)
    eng = llm.engine
    V = llm.cfg.model.vocab
    sp = SamplingParams.greedy_params(max_tokens=G, ignore_eos=True)

    def prompts(run):
        rng = np.random.default_rng(1_000 + run)   # the same prompts on every rank
        return [rng.integers(0, V, P).tolist() for _ in range(R)]

    def one_run(run):
        eng.bm.reset_prefix_cache()
        outs = eng.generate(prompts(run), sp)
        n = sum(len(o.output_token_ids) for o in outs)
        assert n == R * G, n
        return outs

    def barrier():
        if world > 1:
            dist.barrier()

    for w in range(args.warmup):
        one_run(w)
    torch.cuda.synchronize()
    barrier()
    # --- timed region (device-timed) ---
    clocks = ClockSampler(local)
    clocks.start()
    eng.metrics.__init__()
    launches0 = llm.runner.launch_count if hasattr(llm.runner, "launch_count") else 0
    bytes0 = (llm.runner.h2d_bytes, llm.runner.d2h_bytes) if hasattr(llm.runner, "h2d_bytes") else (0, 0)
    torch.cuda.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    all_outs = []
    for k in range(args.steps):
        all_outs += one_run(args.warmup + k)
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    launches = (llm.runner.launch_count - launches0) // max(1, args.steps) if hasattr(llm.runner, "launch_count") else None
    h2d = (llm.runner.h2d_bytes - bytes0[0]) // max(1, args.steps) if hasattr(llm.runner, "h2d_bytes") else None
    d2h = (llm.runner.d2h_bytes - bytes0[1]) // max(1, args.steps) if hasattr(llm.runner, "d2h_bytes") else None
    summ = eng.metrics.summary()
    total_tokens = args.steps * R * G
    value = total_tokens / (ms / 1e3)
    # --- end-to-end through the public API (host token lists in, host outputs back) ---
    barrier()
    t0 = time.perf_counter()
    for k in range(args.e2e_steps):
        outs = llm.generate(prompts(10_000 + k), sp)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e = args.e2e_steps * R * G / float(te.item())
    err = ops.device_error(f"cuda:{local}")
    extra_keys = {}
    if args.config != 2:
        extra_keys["bench_config"] = args.config
    if args.kv_cache_dtype:
        # KV cache bytes per token of the whole model (all ranks)
        extra_keys["kv_bytes_per_token"] = int(llm.runner.kv_bytes_per_token) * world
    if args.config == 4:
        extra_keys["moe_mode"] = args.moe_mode
    spec = getattr(llm.runner, "spec", None)
    if spec is not None:
        st = spec.stats.as_dict()
        extra_keys["spec"] = {"tree": args.spec_tree, "self_draft": args.self_draft, **st,
                              "accepted_tok_per_s": round(value, 2)}
    wgb = llm.runner.weights.bytes_total / 1e9
    if rank == 0:
        model_name = {3: "Llama-3-70B (random-init, Q8_0 GGUF)", 4: "Mixtral-8x7B (random-init, Q4_K GGUF)",
                      5: "Llama-3-8B (random-init, BF16 GGUF) + 16-layer draft (Q8_0)"}.get(args.config, MODEL)
        par = f"ep{world}+tp{world}" if args.config == 4 else f"tp{world}"
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "output tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": f"synthetic: random-init {WEIGHTS.get(args.config, 'Q4_K_M')} weights generated on device in GGUF "
                    "block format; uniform-random prompt token ids (seeded, fresh per run)",
            "config": {"model": model_name, "global_batch": R, "seq_len": P, "gen_len": G, "parallelism": par,
                       "kv_cache": args.kv_cache_dtype or "paged bf16, block 16",
                       "max_num_batched_tokens": args.max_num_batched_tokens,
                       "comm": args.comm if world > 1 else "none",
                       "l2": f"inputs larger than L2 ({wgb:.1f} GB of weights per rank + KV streamed every step)",
                       "step": "one full serving run of global_batch requests"},
            "p50_ttft_ms": round(summ["p50_ttft_ms"], 2), "p50_itl_ms": round(summ["p50_itl_ms"], 3),
            "e2e": {"value": round(e2e, 2), "unit": "output tokens/s (LLM.generate, wall clock)",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches, "clocks": clk, "device_error": err, **extra_keys,
        }
        print(json.dumps(line), flush=True)
    llm.shutdown()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
