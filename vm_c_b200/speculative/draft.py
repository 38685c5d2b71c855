"""Draft-model speculative decoding (greedy verification).

The reference only has MTP speculation: one running request, a linear chain from the model's own
next-n layers (src/core/engine.cpp:636-638, src/speculative/mtp_engine.cpp:220-441). Here a
separate, smaller draft model (its own GGUF, same vocabulary) proposes k tokens for every running
greedy request of a decode step, and the target verifies all of them in one forward pass:

  1. draft catch-up + first proposal: the draft processes the tokens it has not seen (the step's
     input token, plus the last proposal of the previous step if all k were accepted) and emits
     d1 greedily; k - 1 more single-token draft steps emit d2..dk;
  2. the target runs [x0, d1, ..., dk] per request as one (k+1)-token chunk (causal attention over
     the paged cache, KV written for all k + 1 positions into the slots the scheduler reserved as
     look-ahead) and takes the greedy token g_i at every position;
  3. the accepted tokens are the longest prefix with d_{i+1} == g_i, plus the target's token after
     it (so every step yields 1..k+1 tokens); the scheduler counts the verified tokens as computed,
     and KV written past the accepted prefix is simply overwritten later.

The draft keeps its own paged KV cache with the same block ids as the target (one block manager),
so both caches are addressed by the same slot mapping. Steps that are not speculated (prefill
chunks, sampled requests, penalties) run the draft on the same batch ("shadow") to keep its cache
complete. Output equals plain greedy decoding of the target up to floating-point ties.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from ..models.llama import LlamaModel, StepMeta, load_weights


@dataclass
class SpecStats:
    steps: int = 0
    proposed: int = 0
    accepted: int = 0
    emitted: int = 0
    verify_s: float = 0.0
    draft_s: float = 0.0
    per_pos_accept: list = field(default_factory=list)

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.proposed if self.proposed else 0.0

    def as_dict(self) -> dict:
        return dict(steps=self.steps, proposed=self.proposed, accepted=self.accepted, emitted=self.emitted,
                    acceptance_rate=round(self.acceptance_rate, 4),
                    tokens_per_step=round(self.emitted / self.steps, 3) if self.steps else 0.0,
                    verify_ms_per_step=round(1e3 * self.verify_s / self.steps, 3) if self.steps else 0.0,
                    draft_ms_per_step=round(1e3 * self.draft_s / self.steps, 3) if self.steps else 0.0,
                    per_position_accept=list(self.per_pos_accept))


class _NoFuse:
    """Communication view for the draft model: the NCCL path only (the fused peer-memory buffers
    are sized for the target's hidden size)."""

    def __init__(self, comm):
        self._c = comm

    def all_reduce(self, t):
        return self._c.all_reduce(t)

    def sample_vocab_parallel(self, *a, **k):
        return self._c.sample_vocab_parallel(*a, **k)


class DraftSpeculator:
    """Owns the draft model, its KV cache and its own step metadata buffers.

    `layout` sizes the speculator's metadata (k + 1 sampled rows per request); the engine-built
    metadata of the step is read from the runner's pinned buffer with the runner's layout."""

    def __init__(self, runner, draft_source, draft_cfg, k: int, comm=None, layout=None):
        if draft_cfg.vocab != runner.cfg.model.vocab:
            raise ValueError(f"draft vocabulary {draft_cfg.vocab} != target vocabulary {runner.cfg.model.vocab}")
        if k < 1 or k > 16:
            raise ValueError("speculation length must be in 1..16")
        self.runner = runner
        self.k = k
        dev = runner.dev
        self.dev = dev
        draft_cfg.max_model_len = runner.cfg.model.max_model_len
        self.weights = load_weights(draft_source, draft_cfg, dev, runner.tp_rank, runner.tp_size)
        self.model = LlamaModel(self.weights, runner.max_tokens, runner.max_samples, draft_cfg.max_model_len + k,
                                comm=_NoFuse(comm) if comm is not None else None, attn_splits=0)
        self.bs = bs = runner.cfg.cache.block_size
        self.kv = torch.zeros(draft_cfg.n_layers, runner.num_kv_blocks, 2, self.model.hkv, bs, draft_cfg.head_dim,
                              dtype=torch.bfloat16, device=dev)
        self.extra: dict[int, tuple[int, int]] = {}  # request id -> (token, position) not yet in draft KV
        L = layout if layout is not None else runner.layout
        self.L = L
        self.RL = runner.layout  # layout of the engine-built metadata
        self.meta_host = torch.zeros(L.total, dtype=torch.int32).pin_memory()
        self.meta_dev = torch.zeros(L.total, dtype=torch.int32, device=dev)
        md = self.meta_dev
        self.v = dict(
            ids=md[L.off_input_ids:L.off_input_ids + L.max_tokens],
            pos=md[L.off_positions:L.off_positions + L.max_tokens],
            slots=md[L.off_slot_mapping:L.off_slot_mapping + L.max_tokens],
            qs=md[L.off_q_start:L.off_q_start + L.max_reqs + 1],
            ctx=md[L.off_ctx_len:L.off_ctx_len + L.max_reqs],
            lidx=md[L.off_logits_idx:L.off_logits_idx + L.max_reqs],
            bt=md[L.off_block_tables:L.off_block_tables + L.max_reqs * L.max_blocks_per_seq].view(
                L.max_reqs, L.max_blocks_per_seq))
        S = runner.max_samples
        self.params = torch.zeros(S * 40, dtype=torch.uint8, device=dev)   # temperature 0: greedy
        self.tok_dev = torch.zeros(S, dtype=torch.int32, device=dev)
        self.tok_host = torch.zeros(S, dtype=torch.int32).pin_memory()
        self.stats = SpecStats(per_pos_accept=[0] * k)
        self._copied = torch.cuda.Event()
        self._batch_ids: list[int] | None = None

    # -- metadata ----------------------------------------------------------------------------------
    def _meta(self, T, R, S, nd, max_qlen) -> StepMeta:
        v = self.v
        return StepMeta(v["ids"], v["pos"], v["slots"], v["qs"], v["ctx"], v["bt"], v["lidx"], T=T, R=R, S=S,
                        num_decode=nd, max_qlen=max_qlen)

    def _upload(self, ids, pos, slots, qs, ctx, lidx, bt) -> None:
        L = self.L
        self._copied.synchronize()  # the previous copy out of the pinned buffer has finished
        h = self.meta_host.numpy()
        h[L.off_input_ids:L.off_input_ids + len(ids)] = ids
        h[L.off_positions:L.off_positions + len(pos)] = pos
        h[L.off_slot_mapping:L.off_slot_mapping + len(slots)] = slots
        h[L.off_q_start:L.off_q_start + len(qs)] = qs
        h[L.off_ctx_len:L.off_ctx_len + len(ctx)] = ctx
        h[L.off_logits_idx:L.off_logits_idx + len(lidx)] = lidx
        nb = bt.shape[1]
        blk = h[L.off_block_tables:L.off_block_tables + L.max_reqs * L.max_blocks_per_seq].reshape(
            L.max_reqs, L.max_blocks_per_seq)
        blk[:bt.shape[0], :nb] = bt
        self.meta_dev.copy_(self.meta_host, non_blocking=True)
        self._copied.record()

    def _run(self, m: StepMeta) -> np.ndarray:
        self.model.attn_splits = 1
        self.model.forward(self.kv, m, self.params, self.tok_dev, None)
        self.tok_host[:m.S].copy_(self.tok_dev[:m.S], non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return self.tok_host[:m.S].numpy().copy()

    # -- non-speculated steps ------------------------------------------------------------------------
    def set_batch(self, request_ids) -> None:
        """Request id of every row of the step the engine just built (plan entry order)."""
        self._batch_ids = [int(x) for x in request_ids]

    def forget(self, request_id: int) -> None:
        self.extra.pop(int(request_id), None)

    def shadow(self, counts) -> None:
        """Run the draft on the batch the target just ran (same device metadata), so that its cache
        holds the same tokens. Pending proposals of requests in the batch are processed first."""
        self._catch_up(counts)
        r = self.runner
        m = StepMeta(r.v_ids, r.v_pos, r.v_slots, r.v_qs, r.v_ctx, r.v_bt, r.v_lidx, T=counts.T, R=counts.R,
                     S=counts.S, num_decode=counts.num_decode, max_qlen=counts.max_qlen)
        self.model.attn_splits = 1
        self.model.forward(self.kv, m, self.params, self.tok_dev, None)

    def _catch_up(self, counts) -> None:
        if not self.extra or self._batch_ids is None:
            return
        L = self.RL
        h = self.runner.meta_host.numpy()
        ids_of = self._batch_ids[:counts.R]
        rows = [i for i, rid in enumerate(ids_of) if rid in self.extra]
        if not rows:
            return
        bt_all = h[L.off_block_tables:L.off_block_tables + L.max_reqs * L.max_blocks_per_seq].reshape(
            L.max_reqs, L.max_blocks_per_seq)
        toks, pos, slots, bts, ctx = [], [], [], [], []
        for i in rows:
            t, p = self.extra.pop(ids_of[i])
            toks.append(t)
            pos.append(p)
            slots.append(int(bt_all[i, p // self.bs]) * self.bs + p % self.bs)
            bts.append(bt_all[i])
            ctx.append(p + 1)
        n = len(rows)
        self._upload(np.array(toks), np.array(pos), np.array(slots), np.arange(n + 1), np.array(ctx), np.arange(n),
                     np.stack(bts))
        self.model.attn_splits = 1
        self.model.forward(self.kv, self._meta(n, n, n, n, 1), self.params, self.tok_dev, None)

    # -- speculative decode step ---------------------------------------------------------------------
    def step(self, request_ids, counts) -> list[list[int]]:
        """Speculative step for an all-decode batch whose metadata the engine built (one token per
        request). Returns the new tokens of every request (1..k+1 each)."""
        L, k, r = self.RL, self.k, self.runner
        h = r.meta_host.numpy()
        R = counts.R
        ids = [int(x) for x in request_ids]
        qs = h[L.off_q_start:L.off_q_start + R + 1]
        x0 = h[L.off_input_ids + qs[:-1]]
        p0 = h[L.off_positions + qs[:-1]]
        bt = h[L.off_block_tables:L.off_block_tables + R * L.max_blocks_per_seq].reshape(R, L.max_blocks_per_seq).copy()

        bs = self.bs

        def slot(i, p):
            return int(bt[i, p // bs]) * bs + p % bs

        t0 = time.perf_counter()
        # 1) draft: catch-up tokens + x0 in one pass, then k - 1 single-token passes.
        toks, pos, slots, qsd = [], [], [], [0]
        for i in range(R):
            e = self.extra.pop(ids[i], None)
            if e is not None:
                toks.append(e[0])
                pos.append(e[1])
                slots.append(slot(i, e[1]))
            toks.append(int(x0[i]))
            pos.append(int(p0[i]))
            slots.append(slot(i, int(p0[i])))
            qsd.append(len(toks))
        qsd = np.array(qsd)
        T1 = len(toks)
        multi = T1 > R
        self._upload(np.array(toks), np.array(pos), np.array(slots), qsd, p0 + 1, qsd[1:] - 1, bt)
        drafts = np.zeros((R, k), dtype=np.int64)
        drafts[:, 0] = self._run(self._meta(T1, R, R, 0 if multi else R, int(np.max(np.diff(qsd)))))
        for j in range(1, k):
            pj = p0 + j
            self._upload(drafts[:, j - 1], pj, np.array([slot(i, int(pj[i])) for i in range(R)]), np.arange(R + 1),
                         pj + 1, np.arange(R), bt)
            drafts[:, j] = self._run(self._meta(R, R, R, R, 1))
        t1 = time.perf_counter()
        # 2) target verification: [x0, d1..dk] per request, greedy token at every position.
        n = k + 1
        vt = np.concatenate([x0[:, None], drafts], 1).reshape(-1)
        vp = (p0[:, None] + np.arange(n)[None, :]).reshape(-1)
        vs = np.array([slot(i, int(vp[i * n + j])) for i in range(R) for j in range(n)])
        self._upload(vt, vp, vs, np.arange(R + 1) * n, p0 + n, np.arange(R * n), bt)
        r.model.attn_splits = 1
        r.model.forward(r.kv, self._meta(R * n, R, R * n, 0, n), self.params, r.tok_spec, None)
        r.tok_spec_host[:R * n].copy_(r.tok_spec[:R * n], non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        g = r.tok_spec_host[:R * n].numpy().reshape(R, n)
        t2 = time.perf_counter()
        # 3) acceptance: longest matching prefix plus the target's next token.
        out = []
        for i in range(R):
            a = 0
            while a < k and drafts[i, a] == g[i, a]:
                self.stats.per_pos_accept[a] += 1
                a += 1
            out.append([int(t) for t in drafts[i, :a]] + [int(g[i, a])])
            if a == k:  # the draft has not processed its last proposal yet
                self.extra[ids[i]] = (int(drafts[i, k - 1]), int(p0[i]) + k)
            self.stats.accepted += a
            self.stats.emitted += a + 1
        self.stats.proposed += R * k
        self.stats.steps += 1
        self.stats.draft_s += t1 - t0
        self.stats.verify_s += t2 - t1
        return out


# ---------------------------------------------------------------------------------------------------
# Sampled requests: rejection-sampling verification (speculative sampling).
#
# For a request sampled from the filtered distribution p = F(target logits) (temperature, top-k,
# top-p, min-p applied as the GPU sampler applies them), the draft samples d_{j+1} from its own
# filtered distribution q_j; the target accepts d_{j+1} with probability min(1, p_j(d) / q_j(d)),
# and at the first rejection samples from normalize(max(p_j - q_j, 0)); if all k are accepted a
# bonus token is sampled from p_k. Every emitted token is distributed exactly as plain sampling
# from the target would be (Leviathan et al., "Fast Inference from Transformers via Speculative
# Decoding", ICML 2023; Chen et al., "Accelerating Large Language Model Decoding with Speculative
# Sampling", 2023). Greedy rows of the same batch use one-hot distributions, which reduces to the
# greedy rule. The random stream differs from the non-speculative sampler's, so individual sampled
# outputs are not reproduced token for token — their distribution is. Under tensor parallelism the
# vocab-parallel logit shards are all-gathered (every rank computes the same p and q), and rank 0's
# draft tokens, acceptance decisions and resampled tokens are broadcast, so every rank writes the
# same tokens into its cache and issues the same collectives in the next step.

_MAX_CAND = 1024  # candidate cap of the GPU sampler's restricted path


def filtered_probs(logits: torch.Tensor, temp: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
                   min_p: torch.Tensor) -> torch.Tensor:
    """Row-wise sampling distribution of the GPU sampler: temperature, then (when any filter is
    set) the top-k set (at most 1024 candidates), the top-p prefix of it and the min-p cut;
    temperature <= 0 or top_k == 1 gives a one-hot at the argmax. fp32 [n, V]."""
    n, V = logits.shape
    greedy = (temp <= 0) | (top_k == 1)
    t = torch.where(greedy, torch.ones_like(temp), temp)
    x = logits.float() / t[:, None]
    out = torch.softmax(x, -1)
    restricted = (top_k > 0) | (top_p < 1) | (min_p > 0)
    if bool(restricted.any()):
        kcap = min(_MAX_CAND, V)
        vals, idx = torch.topk(x, kcap, dim=-1)            # descending
        k = torch.where(top_k > 0, torch.clamp(top_k, max=kcap), torch.full_like(top_k, kcap))
        pos = torch.arange(kcap, device=x.device)[None, :]
        keep = pos < k[:, None]
        pv = torch.softmax(vals.masked_fill(~keep, float("-inf")), -1)
        cum = torch.cumsum(pv, -1)
        # top-p: keep the smallest prefix whose mass reaches top_p
        keep &= (cum - pv) < top_p[:, None]
        # min-p: p_i >= min_p * p_max
        keep &= pv >= (min_p[:, None] * pv[:, :1])
        keep[:, 0] = True
        pr = torch.zeros_like(x).scatter_(1, idx, pv.masked_fill(~keep, 0.0))
        pr = pr / pr.sum(-1, keepdim=True)
        out = torch.where(restricted[:, None], pr, out)
    if bool(greedy.any()):
        onehot = torch.zeros_like(out).scatter_(1, logits.argmax(-1, keepdim=True), 1.0)
        out = torch.where(greedy[:, None], onehot, out)
    return out


class _RowParams:
    def __init__(self, params, dev):
        self.temp = torch.tensor([p.temperature for p in params], dtype=torch.float32, device=dev)
        self.top_k = torch.tensor([p.top_k for p in params], dtype=torch.int64, device=dev)
        self.top_p = torch.tensor([p.top_p for p in params], dtype=torch.float32, device=dev)
        self.min_p = torch.tensor([p.min_p for p in params], dtype=torch.float32, device=dev)

    def probs(self, logits: torch.Tensor, reps: int = 1) -> torch.Tensor:
        f = (lambda t: t.repeat_interleave(reps)) if reps > 1 else (lambda t: t)
        return filtered_probs(logits, f(self.temp), f(self.top_k), f(self.top_p), f(self.min_p))


def gather_vocab(model, rows: int) -> torch.Tensor:
    """Full-vocabulary logits [rows, V] from the vocab-parallel shards of `model` (rank order is
    vocabulary order); every rank receives the same tensor."""
    lg = model.ws.logits[:rows]
    if model.tp == 1:
        return lg
    import torch.distributed as dist
    parts = [torch.empty_like(lg) for _ in range(model.tp)]
    dist.all_gather(parts, lg.contiguous())
    return torch.cat(parts, -1)


def from_rank0(t: torch.Tensor, tp: int) -> torch.Tensor:
    """Rank 0's values of `t` on every rank (tensor parallelism: all ranks must take the same draft
    tokens and acceptance decisions, so their caches and their next collectives stay identical)."""
    if tp > 1:
        import torch.distributed as dist
        t = t.contiguous()
        dist.broadcast(t, src=0)
    return t


def _sampled_step(self, request_ids, counts, params, seed: int) -> list[list[int]]:
    """Speculative step with rejection-sampling verification (see the section comment above)."""
    L, k, r = self.RL, self.k, self.runner
    tp = self.model.tp
    h = r.meta_host.numpy()
    R = counts.R
    ids = [int(x) for x in request_ids]
    qs = h[L.off_q_start:L.off_q_start + R + 1]
    x0 = h[L.off_input_ids + qs[:-1]]
    p0 = h[L.off_positions + qs[:-1]]
    bt = h[L.off_block_tables:L.off_block_tables + R * L.max_blocks_per_seq].reshape(R, L.max_blocks_per_seq).copy()
    bs = self.bs
    dev = self.dev
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed & 0x7fffffffffffffff)
    rp = _RowParams(params, dev)
    V = self.model.v_local * tp

    def slot(i, p):
        return int(bt[i, p // bs]) * bs + p % bs

    t0 = time.perf_counter()
    toks, pos, slots, qsd = [], [], [], [0]
    for i in range(R):
        e = self.extra.pop(ids[i], None)
        if e is not None:
            toks.append(e[0]); pos.append(e[1]); slots.append(slot(i, e[1]))
        toks.append(int(x0[i])); pos.append(int(p0[i])); slots.append(slot(i, int(p0[i])))
        qsd.append(len(toks))
    qsd = np.array(qsd)
    T1 = len(toks)
    self._upload(np.array(toks), np.array(pos), np.array(slots), qsd, p0 + 1, qsd[1:] - 1, bt)
    qdist = torch.empty(R, k, V, device=dev)
    drafts = torch.empty(R, k, dtype=torch.int64, device=dev)
    self.model.attn_splits = 1
    self.model.forward(self.kv, self._meta(T1, R, R, 0 if T1 > R else R, int(np.max(np.diff(qsd)))), self.params,
                       self.tok_dev, None)
    for j in range(k):
        qdist[:, j] = rp.probs(gather_vocab(self.model, R))
        drafts[:, j] = from_rank0(torch.multinomial(qdist[:, j], 1, generator=gen).squeeze(1), tp)
        if j + 1 < k:
            pj = p0 + j + 1
            dj = drafts[:, j].cpu().numpy()
            self._upload(dj, pj, np.array([slot(i, int(pj[i])) for i in range(R)]), np.arange(R + 1), pj + 1,
                         np.arange(R), bt)
            self.model.forward(self.kv, self._meta(R, R, R, R, 1), self.params, self.tok_dev, None)
    dr = drafts.cpu().numpy()
    t1 = time.perf_counter()
    n = k + 1
    vt = np.concatenate([x0[:, None], dr], 1).reshape(-1)
    vp = (p0[:, None] + np.arange(n)[None, :]).reshape(-1)
    vs = np.array([slot(i, int(vp[i * n + j])) for i in range(R) for j in range(n)])
    self._upload(vt, vp, vs, np.arange(R + 1) * n, p0 + n, np.arange(R * n), bt)
    r.model.attn_splits = 1
    r.model.forward(r.kv, self._meta(R * n, R, R * n, 0, n), self.params, r.tok_spec, None)
    pdist = rp.probs(gather_vocab(r.model, R * n), reps=n).view(R, n, V)
    # acceptance of d_{j+1} with probability min(1, p_j(d) / q_j(d))
    pd = torch.gather(pdist[:, :k], 2, drafts[:, :, None]).squeeze(2)
    qd = torch.gather(qdist, 2, drafts[:, :, None]).squeeze(2)
    u = torch.rand(R, k, device=dev, generator=gen)
    acc = from_rank0((u * qd < pd).to(torch.uint8), tp).bool().cpu().numpy()
    a_len = np.array([int(np.argmin(row)) if not row.all() else k for row in acc])
    # the token after the accepted prefix: residual at the first rejection, p_k if all accepted
    rows = torch.arange(R, device=dev)
    ja = torch.from_numpy(a_len).to(dev)
    pj = pdist[rows, ja]
    qj = torch.where((ja < k)[:, None], qdist[rows, torch.clamp(ja, max=k - 1)], torch.zeros_like(pj))
    res = torch.clamp(pj - qj, min=0.0)
    mass = res.sum(-1, keepdim=True)
    res = torch.where(mass > 0, res / mass.clamp_min(1e-30), pj)
    nxt = from_rank0(torch.multinomial(res, 1, generator=gen).squeeze(1), tp).cpu().numpy()
    t2 = time.perf_counter()
    out = []
    for i in range(R):
        a = int(a_len[i])
        for j in range(a):
            self.stats.per_pos_accept[j] += 1
        out.append([int(t) for t in dr[i, :a]] + [int(nxt[i])])
        if a == k:
            self.extra[ids[i]] = (int(dr[i, k - 1]), int(p0[i]) + k)
        self.stats.accepted += a
        self.stats.emitted += a + 1
    self.stats.proposed += R * k
    self.stats.steps += 1
    self.stats.draft_s += t1 - t0
    self.stats.verify_s += t2 - t1
    return out


DraftSpeculator.sampled_step = _sampled_step
DraftSpeculator.supports_sampling = True
