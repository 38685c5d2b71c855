"""Per-kernel device-time breakdown of serving steps, at any tensor-parallel size.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m vm_c_b200.utils.step_profile [--comm fused]

Serves the 8B config's shape (random-init Q4_K_M weights, ``--requests`` requests of ``--prompt``
tokens) through the engine, and on every rank:

  1. times ``--steps`` decode steps with CUDA events (no profiler attached): the device time per step,
     max over ranks -- the inter-token latency the serving bench reports;
  2. records the same number of decode steps, and separately the first prefill step of a fresh
     batch, under torch.profiler (CUPTI kernel records, CUDA-graph replays included), and sums the
     device time of every kernel per step.

Rank 0 prints each phase's kernels grouped by family (GEMM, attention, reduce-scatter + norm +
all-gather, sampling, NCCL, other) with the microseconds per step and the launches per step, max
over ranks. Kernel durations under the profiler are serialised records; read them as shares of the
step, not as a bench number. With programmatic dependent launch a kernel starts before its
predecessor ends and its record includes that wait: run with VMC_PDL=0 for per-kernel durations
(the CUDA-event step time is then the time without PDL). The reference has no equivalent (its per-op timing is ggml's
GGML_SCHED debug output); this is the breakdown behind the decode-latency analysis.
"""
from __future__ import annotations

import argparse
import json
import re

import numpy as np
import torch
import torch.distributed as dist

FAMILIES = [
    ("gemm", re.compile(r"gemm")),
    ("attention", re.compile(r"attn|attention|flash")),
    ("rs_norm_ag", re.compile(r"rs_norm_ag|moe_combine_norm")),
    ("moe", re.compile(r"moe")),
    ("sampling", re.compile(r"sample|argmax|topk|gumbel")),
    ("nccl", re.compile(r"nccl", re.I)),
    ("norm_rope_embed", re.compile(r"rmsnorm|rope|embed|norm")),
]


def family(name: str) -> str:
    for f, rx in FAMILIES:
        if rx.search(name):
            return f
    return "other"


def short(name: str) -> str:
    """Kernel name without return type, namespaces and argument list (template arguments kept)."""
    name = re.sub(r"^void ", "", name)
    name = name.replace("(anonymous namespace)::", "").replace("vmc::", "")
    depth, cut = 0, len(name)
    for i, ch in enumerate(name):   # the first '(' outside template brackets starts the arguments
        if ch == "<":
            depth += 1
        elif ch == ">":
            depth -= 1
        elif ch == "(" and depth == 0:
            cut = i
            break
    name = name[:cut]
    return name if len(name) < 90 else name[:87] + "..."


def kernel_table(prof, nsteps: int) -> dict:
    out: dict[str, list[float]] = {}
    for e in prof.key_averages():
        t = float(getattr(e, "self_device_time_total", 0.0) or 0.0)
        if t <= 0:   # host-side records (launch API calls) carry no device time
            continue
        k = short(e.key)
        v = out.setdefault(k, [0.0, 0.0])
        v[0] += t / nsteps
        v[1] += e.count / nsteps
    return out


def merge_max(tables: list[dict]) -> dict:
    keys = set().union(*[t.keys() for t in tables])
    return {k: [max(t.get(k, [0, 0])[0] for t in tables), max(t.get(k, [0, 0])[1] for t in tables)] for k in keys}


def report(title: str, tab: dict, step_us: float | None) -> list[str]:
    lines = [f"== {title}" + (f": {step_us:.1f} us per step (CUDA events, max over ranks)" if step_us else "")]
    fams: dict[str, list[float]] = {}
    for k, (us, n) in tab.items():
        f = fams.setdefault(family(k), [0.0, 0.0])
        f[0] += us
        f[1] += n
    tot = sum(v[0] for v in fams.values())
    lines.append(f"   kernel time per step {tot:.1f} us (sum of serialised kernel records)")
    for f, (us, n) in sorted(fams.items(), key=lambda x: -x[1][0]):
        lines.append(f"   {f:16s} {us:9.1f} us  {100 * us / max(tot, 1e-9):5.1f}%  {n:7.1f} launches")
    lines.append("   top kernels:")
    for k, (us, n) in sorted(tab.items(), key=lambda x: -x[1][0])[:14]:
        lines.append(f"     {us:9.1f} us {n:7.1f}x  {k}")
    return lines


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="random:llama3-8b:Q4_K_M:0")
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--comm", choices=["fused", "nccl"], default="fused")
    ap.add_argument("--json", default="")
    ap.add_argument("--host-profile", action="store_true",
                    help="also run the timed decode steps under cProfile and print the top host functions")
    a = ap.parse_args()

    from ..core.sampling_params import SamplingParams
    from ..llm import LLM
    from ..parallel.comm import NcclComm, init_distributed
    rank, world, local = init_distributed(timeout_s=300)
    torch.cuda.set_device(local)
    comm = None
    if world > 1:
        if a.comm == "fused":
            from ..parallel.fused import FusedComm
            comm = FusedComm()
        else:
            comm = NcclComm()
    R, P = a.requests, a.prompt
    llm = LLM(a.model, max_model_len=max(2048, P + 300), max_num_seqs=R, max_num_batched_tokens=2048,
              num_gpu_blocks=2 * R * ((P + 300) // 16 + 1) + 64, tp_rank=rank, tp_size=world, comm=comm,
              device=f"cuda:{local}")
    eng = llm.engine
    rng = np.random.default_rng(0)
    sp = SamplingParams.greedy_params(max_tokens=a.steps * 3 + 16, ignore_eos=True)

    def add_batch():
        return [eng.add_request(rng.integers(0, llm.cfg.model.vocab, P).tolist(), sp) for _ in range(R)]

    # warm-up: serve a first batch until every request decodes (requests join the scheduler at the
    # next step, so the loop follows the returned request objects)
    reqs = add_batch()
    while any(len(r.output_token_ids) < 2 for r in reqs):
        eng.step()
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize()
    # 1) decode steps, CUDA events
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(a.steps):
        eng.step()
    ev1.record()
    torch.cuda.synchronize()
    t = torch.tensor([ev0.elapsed_time(ev1) * 1e3 / a.steps], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dec_us = float(t.item())
    host_lines = []
    if a.host_profile:
        import cProfile
        import io
        import pstats
        import time
        pr = cProfile.Profile()
        t0 = time.perf_counter()
        pr.enable()
        for _ in range(a.steps):
            eng.step()
        pr.disable()
        torch.cuda.synchronize()
        host_ms = (time.perf_counter() - t0) * 1e3 / a.steps
        buf = io.StringIO()
        pstats.Stats(pr, stream=buf).sort_stats("cumulative").print_stats(25)
        host_lines = [f"== host profile of {a.steps} decode steps: {host_ms:.2f} ms per step (wall, under cProfile)"]
        host_lines += buf.getvalue().splitlines()
    # 2) decode steps under the profiler
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(a.steps):
            eng.step()
        torch.cuda.synchronize()
    dec_tab = kernel_table(prof, a.steps)
    # finish the batch, then one profiled prefill step of a fresh one
    while eng.has_unfinished():
        eng.step()
    torch.cuda.synchronize()
    add_batch()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        eng.step()
        torch.cuda.synchronize()
    pre_tab = kernel_table(prof, 1)
    while eng.has_unfinished():
        eng.step()
    torch.cuda.synchronize()
    tabs = [None] * world if world > 1 else [(dec_tab, pre_tab)]
    if world > 1:
        dist.all_gather_object(tabs, (dec_tab, pre_tab))
    if rank == 0:
        dec = merge_max([x[0] for x in tabs])
        pre = merge_max([x[1] for x in tabs])
        lines = [f"step profile: {a.model}, {R} requests x {P}-token prompts, tp{world}, comm {a.comm if world > 1 else 'none'}"]
        lines += report(f"decode step ({R} tokens)", dec, dec_us)
        lines += report("first prefill step of a fresh batch (2048 tokens)", pre, None)
        lines += host_lines
        print("\n".join(lines), flush=True)
        if a.json:
            json.dump({"decode_us": dec_us, "decode": dec, "prefill": pre, "tp": world}, open(a.json, "w"))
    llm.shutdown()
    if comm is not None and hasattr(comm, "close"):
        comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
