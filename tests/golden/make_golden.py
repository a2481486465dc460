"""Generates the golden fixtures in this directory from the reference code.

Run where the ChessDecoder repository is mounted, its root given by the
REFERENCE_ROOT environment variable (required):

    REFERENCE_ROOT=<ChessDecoder checkout> python tests/golden/make_golden.py

Only reference modules that import without torchtune / python-chess are
executed:
  * chessdecoder/models/vocab.py                 -> vocab_reference.json
  * chessdecoder/export/backbone_causal.py        -> backbone_reference.pt
    (the reference's own torchtune-free restatement of the backbone, run on
    seeded weights, with the causal and the block-prefix additive masks and
    Fourier value injection)
  * chessdecoder/utils/training.py                -> utils_reference.pt
    (soft_bucket_loss value and gradient, prepare_fourier_inputs)
  * from chessdecoder/models/model.py, the pure-torch definitions
    make_wl_buckets, make_d_buckets, FourierEncoder, ValueHead and
    ChessDecoder.discretize_to_bucket are extracted with ast and executed on
    their own (the module's top-level imports of torchtune / chess are not).

The RoPE cache that BackboneCausal receives comes from torchtune in the
reference (export/backbone_causal.py:170); here it is filled with the
published torchtune formula, so the fixture pins everything downstream of the
cache but not the cache values themselves.
"""
from __future__ import annotations

import ast
import json
import math
import os
import sys
import types
from pathlib import Path

import torch



def reference_root() -> Path:
    """The ChessDecoder checkout named by REFERENCE_ROOT (required)."""
    if not os.environ.get("REFERENCE_ROOT"):
        raise SystemExit("set REFERENCE_ROOT to the root of the ChessDecoder repository")
    return Path(os.environ["REFERENCE_ROOT"])

OUT = Path(__file__).resolve().parent


def _extract_model_defs():
    src = (reference_root() / "chessdecoder/models/model.py").read_text()
    tree = ast.parse(src)
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in ("make_wl_buckets", "make_d_buckets"):
            keep.append(node)
        if isinstance(node, ast.ClassDef) and node.name in ("FourierEncoder", "ValueHead"):
            keep.append(node)
        if isinstance(node, ast.ClassDef) and node.name == "ChessDecoder":
            for item in node.body:
                if isinstance(item, ast.FunctionDef) and item.name == "discretize_to_bucket":
                    keep.append(item)
    mod = ast.Module(body=keep, type_ignores=[])
    ns = {"torch": torch, "nn": torch.nn, "math": math}
    exec(compile(mod, str(reference_root() / "chessdecoder/models/model.py"), "exec"), ns)
    return ns


def rope_cache_torchtune(max_seq_len, dim, base=10000.0):
    theta = 1.0 / (base ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
    ang = torch.einsum("i,j->ij", torch.arange(max_seq_len, dtype=theta.dtype), theta).float()
    return torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1)


def main():
    sys.path.insert(0, str(reference_root()))
    from chessdecoder.models import vocab as V
    from chessdecoder.export.backbone_causal import BackboneCausal
    from chessdecoder.utils import training as T

    # ---- vocabulary --------------------------------------------------------
    (OUT / "vocab_reference.json").write_text(json.dumps({
        "vocab": V.vocab, "board_vocab": V.board_vocab, "move_vocab": V.move_vocab,
        "POSITION_TOKEN_LENGTH": V.POSITION_TOKEN_LENGTH}))

    ns = _extract_model_defs()

    # ---- backbone ----------------------------------------------------------
    torch.manual_seed(7)
    L, H, hd, E, F, Vs, Smax, nf = 2, 2, 64, 128, 256, V.vocab_size, 80, 16
    bb = BackboneCausal(L, H, hd, E, F, Vs, Smax, nf)
    with torch.no_grad():
        bb.rope_cache.copy_(rope_cache_torchtune(Smax, hd))
        for i in range(L):  # non-trivial norm scales
            bb.sa_norm_weights[i].uniform_(0.5, 1.5)
            bb.mlp_norm_weights[i].uniform_(0.5, 1.5)
        bb.final_norm_weight.uniform_(0.5, 1.5)
    B, S = 3, 72
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, Vs, (B, S), generator=g)
    pos = torch.arange(S).unsqueeze(0).expand(B, S).contiguous()
    override_mask = torch.zeros(B, S, dtype=torch.bool)
    override_mask[:, 5::9] = True
    # values on WL bucket centres, so that bucket snapping (utils/training.py:114-133) is the identity
    override_values = ns["make_wl_buckets"](100, 0.4)[torch.randint(0, 100, (B, S), generator=g)]
    block_id = torch.arange(S).unsqueeze(0).repeat(B, 1) + 1000
    block_id[0, 2:70] = 0
    block_id[1, 0:20] = 0
    block_id[1, 30:50] = 1
    causal = torch.tril(torch.ones(S, S, dtype=torch.bool))
    prefix = causal.unsqueeze(0) | (block_id.unsqueeze(-1) == block_id.unsqueeze(-2))

    def additive(mask):
        return torch.where(mask, 0.0, -1e9).float().unsqueeze(1)

    empty = torch.zeros(L, B, H, 0, hd)
    with torch.no_grad():
        h_causal, _, _ = bb(ids, pos, additive(causal.unsqueeze(0).expand(B, S, S)), empty, empty,
                            override_values, override_mask)
        h_prefix, _, _ = bb(ids, pos, additive(prefix), empty, empty, override_values, override_mask)
    torch.save({
        "config": dict(num_layers=L, num_heads=H, head_dim=hd, embed_dim=E, d_ff=F, vocab_size=Vs, max_seq_len=Smax,
                       num_fourier_freq=nf),
        "state_dict": {k: v.clone() for k, v in bb.state_dict().items()},
        "input_ids": ids, "override_values": override_values, "override_mask": override_mask,
        "block_id": block_id, "h_causal": h_causal, "h_prefix": h_prefix,
    }, OUT / "backbone_reference.pt")

    # ---- utils: soft_bucket_loss, prepare_fourier_inputs, buckets, heads ------
    wl_c = ns["make_wl_buckets"](100, 0.4)
    d_c = ns["make_d_buckets"](100)
    g = torch.Generator().manual_seed(5)
    N = 41
    logits = torch.randn(N, 100, generator=g, requires_grad=True)
    targets = torch.rand(N, generator=g) * 2.2 - 1.1   # includes values outside the centre range
    targets[0] = float(wl_c[0])
    targets[1] = float(wl_c[57])
    targets[2] = -1.0
    targets[3] = 1.0
    valid = torch.rand(N, generator=g) > 0.2
    loss = T.soft_bucket_loss(logits, targets, wl_c, valid)
    loss.backward()
    loss_none = T.soft_bucket_loss(logits.detach(), targets, wl_c, torch.zeros(N, dtype=torch.bool))

    fake_model = types.SimpleNamespace(wl_bucket_centers=wl_c, d_bucket_centers=d_c,
                                       discretize_to_bucket=lambda v, c: ns["discretize_to_bucket"](None, v, c))
    Bq, Sq = 2, 50
    wl_t = torch.rand(Bq, Sq, generator=g) * 2 - 1
    d_t = torch.rand(Bq, Sq, generator=g)
    wl_pos = torch.rand(Bq, Sq, generator=g) > 0.8
    d_pos = torch.roll(wl_pos, 1, dims=1)
    wl_in, d_in = T.prepare_fourier_inputs(fake_model, wl_t, d_t, wl_pos, d_pos)

    torch.manual_seed(3)
    fe = ns["FourierEncoder"](32, 8)
    vh = ns["ValueHead"](32, 100, 16)
    xs = torch.rand(13, generator=g) * 2 - 1
    hs = torch.randn(9, 32, generator=g)
    with torch.no_grad():
        fe_out = fe(xs)
        vh_out = vh(hs)
    torch.save({
        "wl_centers": wl_c, "d_centers": d_c,
        "sbl_logits": logits.detach(), "sbl_targets": targets, "sbl_valid": valid, "sbl_loss": loss.detach(),
        "sbl_grad": logits.grad.clone(), "sbl_loss_no_valid": loss_none,
        "pf_wl_t": wl_t, "pf_d_t": d_t, "pf_wl_pos": wl_pos, "pf_d_pos": d_pos, "pf_wl_in": wl_in, "pf_d_in": d_in,
        "fe_state": fe.state_dict(), "fe_x": xs, "fe_out": fe_out,
        "vh_state": vh.state_dict(), "vh_x": hs, "vh_out": vh_out,
    }, OUT / "utils_reference.pt")
    print("wrote", sorted(p.name for p in OUT.iterdir() if p.suffix in (".pt", ".json")))


if __name__ == "__main__":
    main()
