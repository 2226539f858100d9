"""Expert-parallel batched decode restated on the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The library's batched step (lastro-rust_b200/csrc/batch.cu, the C5 configuration) partitions a batch of sequences
over `world` ranks and its MoE experts over the same ranks, and moves MoE rows between them.  This module restates
that data flow with the oracle's arithmetic (the reference's CPU path, rust/moe-rt/src/cpu.rs and block.rs), so the
exchange semantics can be checked against the single-rank oracle without a GPU:

- sequences are rank-major: rank r decodes its own contiguous share, attention and the dense layers stay local;
- every layer, each rank routes its tokens (router GEMV, optional per-layer bias, top-k in block.rs:81-89's order,
  softmax over the k) and dispatches each (token, pair) whose expert another rank owns to that rank (owner[e], the
  placement table; E / world experts per rank);
- an owner orders the pairs it received by (its local index of the expert, sender rank, the sender's pair order) --
  the library's grouping -- and computes each pair's expert output, y = W_down[e] . silu(W_gate[e] x) * (W_up[e] x);
- the results go back to their senders, which combine them in routing order: y = sum_j w_j * y_j (cpu.rs:141-148),
  then x += residual_multiplier * y.

Each output row depends only on its own token, and the combine keeps routing order, so a sequence's logits and routes
must equal its own single-rank oracle session bit for bit, whatever the world size and placement.  `gather(obj)` is
the group's all-gather (a list of every rank's `obj`, in rank order): torch.distributed.all_gather_object under gloo,
or [obj] for one rank.  Only tests import this module.
"""
from __future__ import annotations

import numpy as np

import oracle as O


def local_index(owner):
    """local[e]: e's index among its owner's experts, in ascending expert id."""
    seen, local = {}, []
    for r in owner:
        local.append(seen.get(r, 0))
        seen[r] = seen.get(r, 0) + 1
    return local


class EPRank:
    """One rank of an expert-parallel group decoding its sequences on an oracle model."""

    def __init__(self, model: O.Model, pool: O.Pool, rank: int, world: int, owner, gather, bias=None):
        c = model.cfg
        self.model, self.pool, self.rank, self.world, self.gather = model, pool, rank, world, gather
        self.owner = [int(x) for x in owner]
        assert len(self.owner) == c["experts"] and all(0 <= r < world for r in self.owner)
        self.local = local_index(self.owner)
        self.bias = None if bias is None else np.asarray(bias, np.float32)
        H, I, E = c["hidden"], c["inter"], c["experts"]
        self.w = []
        for l in range(c["layers"]):
            self.w.append((model.tensor(l, 8, E * H).reshape(E, H),            # router
                           model.tensor(l, 9, E * 2 * I * H).reshape(E, 2 * I, H),  # gate_up
                           model.tensor(l, 10, E * H * I).reshape(E, H, I)))    # down

    def moe(self, l: int, xs):
        """Layer l's MoE block for this rank's tokens xs [n, H] through the exchange: (y [n, H], ids [n, k])."""
        c = self.model.cfg
        H, I, E, k = c["hidden"], c["inter"], c["experts"], c["k"]
        router, gate_up, down = self.w[l]
        n = len(xs)
        ids = np.empty((n, k), np.int32)
        wts = np.empty((n, k), np.float32)
        for t, x in enumerate(xs):
            logits = O.gemv(self.pool, router, E, H, x)
            if self.bias is not None:
                logits = (logits + self.bias[l]).astype(np.float32)
            ids[t], wts[t] = O.routing(logits, k)
        # dispatch: per destination rank, this rank's (token, pair, expert, row) in token then pair order
        out = [[] for _ in range(self.world)]
        for t in range(n):
            for j in range(k):
                e = int(ids[t, j])
                out[self.owner[e]].append((t, j, e, xs[t]))
        inbox = self.gather(out)  # inbox[s][d]: what sender s dispatched to rank d
        # group: the pairs this rank owns, by (local expert, sender, sender's order); each computed on its own row
        recv = [(self.local[e], s, i, t, j, e, x)
                for s in range(self.world) for i, (t, j, e, x) in enumerate(inbox[s][self.rank])]
        recv.sort(key=lambda r: (r[0], r[1], r[2]))
        back = [[] for _ in range(self.world)]
        for _, s, _, t, j, e, x in recv:
            a = O.swiglu(O.gemv(self.pool, gate_up[e], 2 * I, H, x))
            back[s].append((t, j, O.gemv(self.pool, down[e], H, I, a)))
        returned = self.gather(back)  # returned[o][s]: owner o's results for sender s
        ys = np.zeros((n, k, H), np.float32)
        got = np.zeros((n, k), bool)
        for o in range(self.world):
            for t, j, y in returned[o][self.rank]:
                ys[t, j] = y
                got[t, j] = True
        assert got.all(), "every pair came back exactly once"
        # combine in routing order (cpu.rs:141-148: acc += w_j * y_j, from zero)
        y = np.zeros((n, H), np.float32)
        for j in range(k):
            y = (y + wts[:, j:j + 1] * ys[:, j]).astype(np.float32)
        return y, ids

    def step(self, sessions, tokens):
        """One decode step of this rank's sequences (sessions[i] fed tokens[i]): (logits [n, V], routes [n, L, k])."""
        c = self.model.cfg
        for s, tok in zip(sessions, tokens):
            s.step_begin(tok)
        routes = np.empty((len(sessions), c["layers"], c["k"]), np.int32)
        for l in range(c["layers"]):
            xs = [s.layer_attention(l) for s in sessions]
            y, ids = self.moe(l, xs)
            routes[:, l] = ids
            for i, s in enumerate(sessions):
                s.layer_moe(l, y[i])
        return np.stack([s.step_end() for s in sessions]), routes
