"""The KV-cache oracle (oracle/decode.py) against the reference's exported
module (chessdecoder/export/backbone_causal.py, via
tests/golden/decode_reference.pt): every causal / prefix / probe call of a
scenario with padding, inactive sequences, per-sequence positions and Fourier
overrides, plus the host-side argument checks of the product class."""
import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import decode as OD

GOLD = Path(__file__).parent / "golden"
G = torch.load(GOLD / "decode_reference.pt")


def _golden_module():
    spec = importlib.util.spec_from_file_location("make_decode_golden", GOLD / "make_decode_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def golden_weights():
    """ChessDecoder-named fp32 weights of the golden config."""
    mod = _golden_module()
    cfg = G["config"]
    return OD.module_to_chess_decoder(mod.module_weights(cfg, G["seed"]), cfg["num_layers"]), cfg


def _np(kw):
    return {k: (v.numpy() if isinstance(v, torch.Tensor) else v) for k, v in kw.items()}


def test_oracle_matches_reference_module():
    w, cfg = golden_weights()
    ob = OD.Batched(w, cfg, G["batch"], cfg["max_seq_len"])
    for call in G["calls"]:
        h = getattr(ob, call["method"])(**_np(call["inputs"]))
        ref = call["hidden"].numpy()
        err = np.abs(h - ref).max()
        assert err < 2e-4, (call["method"], err)


def test_golden_rope_table_is_the_oracles():
    mod = _golden_module()
    cfg = G["config"]
    assert np.allclose(mod.rope_cache(cfg["max_seq_len"], cfg["head_dim"]).numpy(),
                       OD.rope_table(cfg["max_seq_len"], cfg["head_dim"]), atol=1e-5)


def test_scenario_covers_every_mode():
    names = {c["method"] for c in G["calls"]}
    assert names == {"causal_forward", "causal_incremental", "causal_probe", "prefix_forward",
                     "prefix_block_forward", "prefix_incremental", "prefix_probe"}


def test_product_rejects_bad_shapes_without_gpu():
    from chessdecoder_b200 import decode as D
    from chessdecoder_b200.engine import ModelConfig
    with pytest.raises(ValueError):
        D.BatchedBackbone(ModelConfig(moe_experts=4), batch_size=2, device="cpu")
    with pytest.raises(ValueError):
        D.BatchedBackbone(ModelConfig(embed_dim=256, num_heads=2), batch_size=2, device="cpu")
