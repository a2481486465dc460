"""ORACLE (test infrastructure only): the MoE MLP of the MoE variant, in fp32.

The reference has no mixture of experts; these are the variant's semantics
(the CUDA path in chessdecoder_b200/csrc/moe.cu restates them):

* router Linear(E -> X, no bias); p = softmax(router(x)); the top-2 experts
  (e1, e2) by probability, weights w_k = p_ek / (p_e1 + p_e2);
* per forward call (one pass over T tokens) each expert has
  cap = ceil(capacity * 2 * T / X) slots, filled by the first choices in token
  order and then by the second choices in token order; a choice whose expert is
  full is dropped (contributes nothing; no auxiliary loss);
* each expert is a SwiGLU FFN with the dense layer's shapes: w13[x] = [gate; up]
  [2F, E], w2[x] = down [E, F];
* y = sum over kept choices of w_k * FFN_ek(x).

Construction order (so that torch.manual_seed gives the CUDA engine's initial
weights): router, then per expert gate (E->F), down (F->E), up (E->F) as
nn.Linear layers, stacked into w13 / w2.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


class _Router(nn.Module):
    def __init__(self, E, X):
        super().__init__()
        self.weight = nn.Linear(E, X, bias=False).weight


class _Experts(nn.Module):
    def __init__(self, E, Fd, X):
        super().__init__()
        w13, w2 = [], []
        for _ in range(X):
            gate = nn.Linear(E, Fd, bias=False).weight.data
            down = nn.Linear(Fd, E, bias=False).weight.data
            up = nn.Linear(E, Fd, bias=False).weight.data
            w13.append(torch.cat([gate, up], 0))
            w2.append(down)
        self.w13 = nn.Parameter(torch.stack(w13))  # [X, 2F, E]
        self.w2 = nn.Parameter(torch.stack(w2))    # [X, E, F]


class OracleMoE(nn.Module):
    """``forced``: optional list of (expert [T, 2], keep [T, 2] bool) decisions,
    one per forward call in call order, that replace the top-2 / capacity
    choices (the weights are still this module's renormalised probabilities
    of the given experts): a check of everything downstream of the discrete
    routing against another implementation's decisions.  ``record``: when a
    list, each call appends its own (expert, keep)."""

    def __init__(self, embed_dim, d_ff, n_experts=8, capacity=1.25):
        super().__init__()
        self.E, self.F, self.X, self.capacity = embed_dim, d_ff, n_experts, capacity
        self.router = _Router(embed_dim, n_experts)
        self.experts = _Experts(embed_dim, d_ff, n_experts)
        self.forced = None
        self.record = None

    def route(self, xt):
        """(idx [T,2], w [T,2], keep [T,2] bool, cap) for tokens xt [T, E]."""
        T, X = xt.shape[0], self.X
        p = torch.softmax(xt @ self.router.weight.t(), dim=-1)
        cap = math.ceil(self.capacity * 2 * T / X)
        if self.forced:
            idx, keep = self.forced.pop(0)
            idx, keep = idx.to(xt.device).long(), keep.to(xt.device).bool()
            v = p.gather(1, idx)
            return idx, v / v.sum(-1, keepdim=True), keep, cap
        v, idx = torch.topk(p, 2, dim=-1)
        w = v / v.sum(-1, keepdim=True)
        keep = torch.zeros(T, 2, dtype=torch.bool, device=xt.device)
        fill = torch.zeros(X, dtype=torch.long, device=xt.device)
        ar = torch.arange(T, device=xt.device)
        for k in range(2):
            e = idx[:, k]
            oh = F.one_hot(e, X)
            pos = (torch.cumsum(oh, 0) - 1)[ar, e] + fill[e]
            keep[:, k] = pos < cap
            fill = fill + oh.sum(0)
        if self.record is not None:
            self.record.append((idx.detach().clone(), keep.clone()))
        return idx, w, keep, cap

    def forward(self, x):
        shp = x.shape
        xt = x.reshape(-1, self.E)
        idx, w, keep, _ = self.route(xt)
        y = torch.zeros_like(xt)
        for e in range(self.X):
            w13, w2 = self.experts.w13[e], self.experts.w2[e]
            for k in range(2):
                rows = torch.nonzero((idx[:, k] == e) & keep[:, k]).flatten()
                if rows.numel() == 0:
                    continue
                z = xt[rows]
                h = z @ w13.t()
                out = (F.silu(h[:, : self.F]) * h[:, self.F:]) @ w2.t()
                y = y.index_add(0, rows, w[rows, k:k + 1] * out)
        return y.reshape(shp)
