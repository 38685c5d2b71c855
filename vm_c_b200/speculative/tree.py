"""Token-tree speculative decoding (greedy verification) with a draft model.

Not in the reference (its MTP path verifies one linear chain for one request,
src/speculative/mtp_engine.cpp:220-441). The tree shape is given per depth, e.g. ``--spec-tree
2,2,1``: the root (the step's input token x0) gets the draft's top-2 next tokens as children, each
of them its top-2, each of those its top-1 — 1 + 2 + 4 + 4 = 11 nodes, numbered breadth-first.

One step, for every running greedy request of an all-decode batch:

  1. draft: catch-up + root in one pass (as in the linear speculator), then one pass per depth over
     that depth's frontier; node i is written into the KV cache at position p0 + i (p0 = the root's
     position) and attends to the context and to its own ancestors only (attention tree masks over
     the last positions of the sequence); the children of a node are the draft's top-b tokens;
  2. target: one pass over all N nodes with the same masks; RoPE positions are p0 + depth, so a
     node sees exactly the sequence its branch would have;
  3. acceptance: from the root, follow the child whose token equals the target's greedy token at
     the current node; the accepted tokens are that branch plus the target's token after it;
  4. the accepted nodes' KV rows (target and draft caches, every layer) are moved to positions
     p0 + 1, p0 + 2, ... (one kernel; reads before writes), so the cache holds the committed
     sequence contiguously, as after plain decoding.

The scheduler reserves N - 1 look-ahead slots per decode and counts the accepted tokens as
computed. Output equals plain greedy decoding of the target up to floating-point ties.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from .draft import DraftSpeculator


class TokenTree:
    """Breadth-first node layout of a tree with `branching[d]` children per node at depth d."""

    def __init__(self, branching: list[int]):
        if not branching or any(b < 1 for b in branching):
            raise ValueError("tree branching must be a non-empty list of positive integers")
        self.branching = list(branching)
        parent, depth = [-1], [0]
        level = [0]
        self.level_start = [0]
        for d, b in enumerate(branching, 1):
            self.level_start.append(len(parent))
            nxt = []
            for u in level:
                for _ in range(b):
                    parent.append(u)
                    depth.append(d)
                    nxt.append(len(parent) - 1)
            level = nxt
        self.level_start.append(len(parent))
        if len(parent) > 64:
            raise ValueError(f"token tree has {len(parent)} nodes; at most 64 are supported")
        self.parent = np.array(parent)
        self.depth = np.array(depth)
        self.N = len(parent)
        self.D = len(branching)
        self.children = [[] for _ in range(self.N)]
        for i in range(1, self.N):
            self.children[parent[i]].append(i)
        masks = np.zeros(self.N, dtype=np.uint64)
        for i in range(self.N):
            masks[i] = np.uint64(1 << i) | (masks[parent[i]] if i else np.uint64(0))
        self.masks = masks.view(np.int64)

    def level(self, d: int) -> range:
        return range(self.level_start[d], self.level_start[d + 1])


class TreeSpeculator(DraftSpeculator):
    supports_sampling = False  # greedy verification only: sampled requests take the plain path
    def __init__(self, runner, draft_source, draft_cfg, branching: list[int], comm=None, layout=None):
        self.tree = TokenTree(branching)
        super().__init__(runner, draft_source, draft_cfg, self.tree.N - 1, comm=comm, layout=layout)
        self.stats.per_pos_accept = [0] * self.tree.D
        dev = self.dev
        mr = runner.max_samples
        self.mask_dev = torch.zeros(mr, dtype=torch.int64, device=dev)
        self.mask_host = torch.zeros(mr, dtype=torch.int64).pin_memory()
        nreq = max(1, mr // self.tree.N)
        self.mv_host = torch.zeros(3, nreq, 16, dtype=torch.int32).pin_memory()
        self.mv_dev = torch.zeros(3, nreq, 16, dtype=torch.int32, device=dev)

    # ---------------------------------------------------------------------------------------------
    def _masks(self, per_req: np.ndarray, R: int) -> torch.Tensor:
        n = per_req.size
        self.mask_host[:R * n].numpy()[:] = np.tile(per_req, R)
        self.mask_dev[:R * n].copy_(self.mask_host[:R * n], non_blocking=True)
        return self.mask_dev[:R * n]

    def _topk(self, model, S: int, k: int) -> np.ndarray:
        """Top-k token ids of the first S logits rows of `model` (vocab-parallel shards merged)."""
        lg = model.ws.logits[:S]
        v, i = torch.topk(lg, k, dim=-1)
        i = i + model.w.vocab_begin
        if model.tp > 1:
            import torch.distributed as dist
            vs = [torch.empty_like(v) for _ in range(model.tp)]
            is_ = [torch.empty_like(i) for _ in range(model.tp)]
            dist.all_gather(vs, v)
            dist.all_gather(is_, i)
            v, i = torch.cat(vs, -1), torch.cat(is_, -1)
            v, j = torch.topk(v, k, dim=-1)
            i = torch.gather(i, -1, j)
        return i.cpu().numpy()

    # ---------------------------------------------------------------------------------------------
    def step(self, request_ids, counts) -> list[list[int]]:
        L, tree, r = self.RL, self.tree, self.runner
        N, D = tree.N, tree.D
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

        tok = np.zeros((R, N), dtype=np.int64)
        tok[:, 0] = x0
        t0 = time.perf_counter()
        # 1) draft: catch-up + root, then one pass per depth over the frontier.
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
        multi = T1 > R
        self.model.attn_splits = 1
        self.model.forward(self.kv, self._meta(T1, R, R, 0 if multi else R, int(np.max(np.diff(qsd)))), self.params,
                           self.tok_dev, None)
        parents = list(tree.level(0))  # frontier whose children come next
        top = self._topk(self.model, R, tree.branching[0]).reshape(R, 1, -1)
        for d in range(1, D + 1):
            lvl = tree.level(d)
            for n_, u in enumerate(lvl):
                par = tree.parent[u]
                k = tree.children[par].index(u)
                tok[:, u] = top[:, parents.index(par), k]
            if d == D:
                break
            F = len(lvl)
            span = lvl.stop  # positions p0 .. p0 + span - 1 hold the tree so far
            ptok = tok[:, lvl.start:lvl.stop].reshape(-1)
            ppos = (p0[:, None] + d).repeat(F, 1).reshape(-1)
            pslots = np.array([slot(i, int(p0[i]) + u) for i in range(R) for u in lvl])
            self._upload(ptok, ppos, pslots, np.arange(R + 1) * F, p0 + span, np.arange(R * F), bt)
            m = self._meta(R * F, R, R * F, 0, F)
            m.tree_mask, m.tree_span = self._masks(tree.masks[:span][lvl.start:lvl.stop], R), span
            self.model.forward(self.kv, m, self.params, self.tok_dev, None)
            top = self._topk(self.model, R * F, tree.branching[d]).reshape(R, F, -1)
            parents = list(lvl)
        t1 = time.perf_counter()
        # 2) target verification over all N nodes.
        vt = tok.reshape(-1)
        vp = (p0[:, None] + tree.depth[None, :]).reshape(-1)
        vs = np.array([slot(i, int(p0[i]) + u) for i in range(R) for u in range(N)])
        self._upload(vt, vp, vs, np.arange(R + 1) * N, p0 + N, np.arange(R * N), bt)
        mv = self._meta(R * N, R, R * N, 0, N)
        mv.tree_mask, mv.tree_span = self._masks(tree.masks, R), N
        r.model.attn_splits = 1
        r.model.forward(r.kv, mv, self.params, r.tok_spec, None)
        r.tok_spec_host[:R * N].copy_(r.tok_spec[:R * N], non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        g = r.tok_spec_host[:R * N].numpy().reshape(R, N)
        t2 = time.perf_counter()
        # 3) acceptance and 4) KV compaction.
        out = []
        mvh = self.mv_host.numpy()
        mvh[2, :R, 0] = 0
        any_move = False
        for i in range(R):
            u, path = 0, []
            while tree.children[u]:
                nxt = [c for c in tree.children[u] if tok[i, c] == g[i, u]]
                if not nxt:
                    break
                u = nxt[0]
                path.append(u)
                self.stats.per_pos_accept[len(path) - 1] += 1
            out.append([int(tok[i, c]) for c in path] + [int(g[i, u])])
            n = 0
            for dpt, c in enumerate(path, 1):
                if c != dpt:
                    mvh[0, i, n] = slot(i, int(p0[i]) + c)
                    mvh[1, i, n] = slot(i, int(p0[i]) + dpt)
                    n += 1
            mvh[2, i, 0] = n
            any_move |= n > 0
            if len(path) == D:  # a leaf: the draft never processed its token
                self.extra[ids[i]] = (int(tok[i, path[-1]]), int(p0[i]) + D)
            self.stats.accepted += len(path)
            self.stats.emitted += len(path) + 1
        if any_move:
            self.mv_dev[:, :R].copy_(self.mv_host[:, :R], non_blocking=True)
            src, dst, cnt = self.mv_dev[0, :R], self.mv_dev[1, :R], self.mv_dev[2, :R, 0].contiguous()
            from .. import ops
            ops.kv_move(r.kv, r.model.hkv, r.model.D, src.contiguous(), dst.contiguous(), cnt, R, 16)
            ops.kv_move(self.kv, self.model.hkv, self.model.D, src.contiguous(), dst.contiguous(), cnt, R, 16)
        self.stats.proposed += R * D
        self.stats.steps += 1
        self.stats.draft_s += t1 - t0
        self.stats.verify_s += t2 - t1
        return out
