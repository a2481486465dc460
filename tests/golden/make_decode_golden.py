"""Generates tests/golden/decode_reference.pt from the reference's exported
KV-cache module (chessdecoder/export/backbone_causal.py, ``BackboneCausal``,
which imports only torch).  Run where the ChessDecoder repository is mounted
(its root given by the REFERENCE_ROOT environment variable, required):

    REFERENCE_ROOT=<ChessDecoder checkout> python tests/golden/make_decode_golden.py

The C++ ``BatchedBackbone`` (chessdecoder/cpp/decoder/batched_backbone.cpp)
that drives the module cannot run here (it needs libtorch and a TorchScript
export); its cache and mask bookkeeping is restated below, line for line in
behaviour, around the reference module's own ``forward``.  The module runs in
fp32 on the CPU.  Weights come from ``numpy.random.RandomState(seed)`` (a
frozen stream), so the fixture stores only the seed, the call inputs and the
hidden states.
"""
from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np
import torch



def reference_root() -> Path:
    """The ChessDecoder checkout named by REFERENCE_ROOT (required)."""
    if not os.environ.get("REFERENCE_ROOT"):
        raise SystemExit("set REFERENCE_ROOT to the root of the ChessDecoder repository")
    return Path(os.environ["REFERENCE_ROOT"])


CONFIG = dict(num_layers=2, num_heads=2, head_dim=64, embed_dim=128, d_ff=256, vocab_size=64, max_seq_len=64,
              num_fourier_freq=16)
SEED = 11


def module_weights(cfg, seed):
    """Random weights in BackboneCausal's parameter names (fp32 numpy)."""
    rs = np.random.RandomState(seed)
    L, E, F, V, nf = (cfg["num_layers"], cfg["embed_dim"], cfg["d_ff"], cfg["vocab_size"], cfg["num_fourier_freq"])
    w = {"tok_embedding.weight": rs.randn(V, E) * 0.5,
         "fourier_frequencies": rs.randn(1, nf),
         "fourier_proj.weight": rs.randn(E, 2 * nf) / math.sqrt(2 * nf),
         "fourier_proj.bias": rs.randn(E) * 0.1}
    for i in range(L):
        for n in ("q_projs", "k_projs", "v_projs", "o_projs"):
            w[f"{n}.{i}.weight"] = rs.randn(E, E) / math.sqrt(E)
        w[f"sa_norm_weights.{i}"] = 1.0 + 0.1 * rs.randn(E)
        w[f"mlp_norm_weights.{i}"] = 1.0 + 0.1 * rs.randn(E)
        w[f"gate_projs.{i}.weight"] = rs.randn(F, E) / math.sqrt(E)
        w[f"up_projs.{i}.weight"] = rs.randn(F, E) / math.sqrt(E)
        w[f"down_projs.{i}.weight"] = rs.randn(E, F) / math.sqrt(F)
    w["final_norm_weight"] = 1.0 + 0.1 * rs.randn(E)
    return {k: np.asarray(v, dtype=np.float32) for k, v in w.items()}


def rope_cache(max_seq_len, head_dim, base=10000.0):
    theta = 1.0 / (base ** (torch.arange(0, head_dim, 2)[: head_dim // 2].float() / head_dim))
    ang = torch.outer(torch.arange(max_seq_len).float(), theta)
    return torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1)


class Batched:
    """batched_backbone.cpp's bookkeeping around the module (fp32, CPU)."""

    def __init__(self, model, B, cfg):
        self.m, self.B = model, B
        L, H, HD = cfg["num_layers"], cfg["num_heads"], cfg["head_dim"]
        self.empty = torch.zeros(L, B, H, 0, HD)
        self.max_len = cfg["max_seq_len"]
        self.ck = self.cv = self.pk = self.pv = self.empty
        self.cbuf = torch.full((B, 1, 1, self.max_len), -1e9)
        self.pbuf = torch.full((B, 1, 1, self.max_len), -1e9)

    def run(self, ids, pos, mask, k, v, ov, om):
        with torch.no_grad():
            return self.m(ids, pos, mask, k, v, ov, om)

    def causal_forward(self, ids, pos, ov, om, active, num_real):
        B, S = ids.shape
        old = self.ck.shape[3]
        mask = torch.full((B, 1, S, old + S), -1e9)
        if old:
            mask[..., :old] = self.cbuf[..., :old].expand(B, 1, S, old)
        j = torch.arange(S)
        new_valid = j[None, :] < num_real[:, None]
        att = new_valid[:, None, :] & (j[None, :] <= j[:, None])[None]
        mask[..., old:] = torch.where(att, 0.0, -1e9)[:, None]
        h, self.ck, self.cv = self.run(ids, pos, mask, self.ck, self.cv, ov, om)
        self.cbuf[:, 0, 0, old:old + S].masked_fill_(new_valid, 0.0)
        return h

    def _incremental(self, buf, k, v, ids, pos, ov, om, active):
        new = k.shape[3]
        buf[:, 0, 0, new].masked_fill_(active, 0.0)
        mask = buf[..., :new + 1].clone()
        return self.run(ids, pos, mask, k, v, ov, om)

    def causal_incremental(self, ids, pos, ov, om, active):
        h, self.ck, self.cv = self._incremental(self.cbuf, self.ck, self.cv, ids, pos, ov, om, active)
        return h

    def prefix_forward(self, ids, pos, mask, ov, om, active):
        S = ids.shape[1]
        h, self.pk, self.pv = self.run(ids, pos, mask, self.pk, self.pv, ov, om)
        self.pbuf[:, 0, 0, :S].masked_fill_(active[:, None], 0.0)
        return h

    def prefix_incremental(self, ids, pos, ov, om, active):
        h, self.pk, self.pv = self._incremental(self.pbuf, self.pk, self.pv, ids, pos, ov, om, active)
        return h

    def prefix_block_forward(self, ids, pos, ov, om, active):
        B, S = ids.shape
        old = self.pk.shape[3]
        mask = torch.full((B, 1, S, old + S), -1e9)
        if old:
            mask[..., :old] = self.pbuf[..., :old].expand(B, 1, S, old)
        mask[..., old:] = torch.where(active.view(B, 1, 1, 1), 0.0, -1e9).expand(B, 1, S, S)
        h, self.pk, self.pv = self.run(ids, pos, mask, self.pk, self.pv, ov, om)
        self.pbuf[:, 0, 0, old:old + S].masked_fill_(active[:, None], 0.0)
        return h

    def _probe(self, buf, k, v, ids, pos, ov, om):
        B, S = ids.shape
        old = k.shape[3]
        mask = torch.full((B, 1, S, old + S), -1e9)
        if old:
            mask[..., :old] = buf[..., :old].expand(B, 1, S, old)
        mask[..., old:] = 0.0
        return self.run(ids, pos, mask, k, v, ov, om)[0]

    def causal_probe(self, ids, pos, ov, om):
        return self._probe(self.cbuf, self.ck, self.cv, ids, pos, ov, om)

    def prefix_probe(self, ids, pos, ov, om):
        return self._probe(self.pbuf, self.pk, self.pv, ids, pos, ov, om)


def scenario(B, V, seed):
    """The call list: (method, kwargs) in order, inputs as tensors."""
    g = torch.Generator().manual_seed(seed)
    ids = lambda S: torch.randint(0, V, (B, S), generator=g)  # noqa: E731
    t = lambda *x: torch.tensor(x)  # noqa: E731
    calls = []
    S0 = 8
    om = torch.zeros(B, S0, dtype=torch.bool)
    om[0, 3] = om[2, 5] = True
    ov = torch.zeros(B, S0)
    ov[0, 3], ov[2, 5] = 0.37, -0.52
    num_real = t(8, 6, 7)
    calls.append(("causal_forward", dict(ids=ids(S0), pos=torch.arange(S0).repeat(B, 1), ov=ov, om=om,
                                         active=t(True, True, True), num_real=num_real)))
    seq_pos = num_real.clone()
    for k, act in enumerate(((True, True, True), (True, False, True), (True, True, True))):
        om1 = torch.zeros(B, 1, dtype=torch.bool)
        ov1 = torch.zeros(B, 1)
        if k == 1:
            om1[0, 0], ov1[0, 0] = True, 0.81
        calls.append(("causal_incremental", dict(ids=ids(1), pos=seq_pos[:, None].clone(), ov=ov1, om=om1,
                                                 active=t(*act))))
        seq_pos += t(*act).long()
    calls.append(("causal_probe", dict(ids=ids(2), pos=torch.stack([seq_pos, seq_pos + 1], 1), ov=torch.zeros(B, 2),
                                       om=torch.zeros(B, 2, dtype=torch.bool))))
    S1 = 10
    block = torch.tensor([0, 0, 1, 1, 1, 1, 2, 3, 4, 5])
    allowed = (block[None, :] <= block[:, None]) | (block[None, :] == block[:, None])
    causal = torch.arange(S1)[None, :] <= torch.arange(S1)[:, None]
    m = torch.where(allowed | causal, 0.0, -1e9).expand(B, 1, S1, S1).clone()
    omp = torch.zeros(B, S1, dtype=torch.bool)
    omp[1, 7] = True
    ovp = torch.zeros(B, S1)
    ovp[1, 7] = 0.25
    calls.append(("prefix_forward", dict(ids=ids(S1), pos=torch.arange(S1).repeat(B, 1), mask=m, ov=ovp, om=omp,
                                         active=t(True, True, True))))
    calls.append(("prefix_block_forward", dict(ids=ids(4), pos=torch.arange(S1, S1 + 4).repeat(B, 1),
                                               ov=torch.zeros(B, 4), om=torch.zeros(B, 4, dtype=torch.bool),
                                               active=t(True, False, True))))
    calls.append(("prefix_incremental", dict(ids=ids(1), pos=torch.full((B, 1), S1 + 4), ov=torch.zeros(B, 1),
                                             om=torch.zeros(B, 1, dtype=torch.bool), active=t(True, True, False))))
    calls.append(("prefix_probe", dict(ids=ids(3), pos=torch.arange(S1 + 5, S1 + 8).repeat(B, 1),
                                       ov=torch.zeros(B, 3), om=torch.zeros(B, 3, dtype=torch.bool))))
    return calls


def main():
    sys.path.insert(0, str(reference_root()))
    from chessdecoder.export.backbone_causal import BackboneCausal
    cfg = CONFIG
    model = BackboneCausal(cfg["num_layers"], cfg["num_heads"], cfg["head_dim"], cfg["embed_dim"], cfg["d_ff"],
                           cfg["vocab_size"], cfg["max_seq_len"], cfg["num_fourier_freq"])
    w = module_weights(cfg, SEED)
    sd = {k: torch.from_numpy(v) for k, v in w.items()}
    sd["rope_cache"] = rope_cache(cfg["max_seq_len"], cfg["head_dim"])
    model.load_state_dict(sd)
    model.eval()
    B = 3
    runner = Batched(model, B, cfg)
    calls = scenario(B, cfg["vocab_size"], SEED)
    out = []
    for name, kw in calls:
        h = getattr(runner, name)(**kw)
        out.append({"method": name, "inputs": kw, "hidden": h.detach().clone()})
    torch.save({"config": cfg, "seed": SEED, "batch": B, "calls": out},
               Path(__file__).with_name("decode_reference.pt"))
    print("wrote decode_reference.pt:", [c["method"] for c in out])


if __name__ == "__main__":
    main()
