"""Golden fixtures made from the reference code itself (tests/golden/make_golden.py):
they pin the oracle (CPU) and the CUDA path (GPU) to the reference's own
arithmetic.

* vocab_reference.json    <- chessdecoder/models/vocab.py
* backbone_reference.pt   <- chessdecoder/export/backbone_causal.py (the
  reference's torchtune-free backbone) on seeded weights, causal and
  block-prefix masks, Fourier injection
* utils_reference.pt      <- chessdecoder/utils/training.py (soft_bucket_loss
  value + gradient, prepare_fourier_inputs) and the pure-torch definitions of
  chessdecoder/models/model.py (bucket centres, FourierEncoder, ValueHead,
  discretize_to_bucket)
"""
import json
import types
from pathlib import Path

import pytest
import torch

GOLD = Path(__file__).resolve().parent / "golden"


def _bb():
    return torch.load(GOLD / "backbone_reference.pt", weights_only=False)


def _utils():
    return torch.load(GOLD / "utils_reference.pt", weights_only=False)


def to_model_state_dict(bsd, num_layers):
    """BackboneCausal names -> ChessDecoder (torchtune) names, the inverse of
    chessdecoder/export/backbone_causal.py:174-187."""
    sd = {"tok_embedding.weight": bsd["tok_embedding.weight"],
          "fourier_encoder.frequencies": bsd["fourier_frequencies"],
          "fourier_encoder.proj.weight": bsd["fourier_proj.weight"],
          "fourier_encoder.proj.bias": bsd["fourier_proj.bias"],
          "norm.scale": bsd["final_norm_weight"]}
    for i in range(num_layers):
        p = f"layers.{i}."
        sd[p + "attn.q_proj.weight"] = bsd[f"q_projs.{i}.weight"]
        sd[p + "attn.k_proj.weight"] = bsd[f"k_projs.{i}.weight"]
        sd[p + "attn.v_proj.weight"] = bsd[f"v_projs.{i}.weight"]
        sd[p + "attn.output_proj.weight"] = bsd[f"o_projs.{i}.weight"]
        sd[p + "mlp.w1.weight"] = bsd[f"gate_projs.{i}.weight"]
        sd[p + "mlp.w3.weight"] = bsd[f"up_projs.{i}.weight"]
        sd[p + "mlp.w2.weight"] = bsd[f"down_projs.{i}.weight"]
        sd[p + "sa_norm.scale"] = bsd[f"sa_norm_weights.{i}"]
        sd[p + "mlp_norm.scale"] = bsd[f"mlp_norm_weights.{i}"]
    return sd


# ---------------------------------------------------------------------------
# CPU: product vocabulary and bucket centres, oracle arithmetic
# ---------------------------------------------------------------------------
def test_vocab_matches_reference_table():
    from chessdecoder_b200 import vocab as V
    ref = json.loads((GOLD / "vocab_reference.json").read_text())
    assert V.vocab == ref["vocab"]
    assert V.board_vocab == ref["board_vocab"]
    assert V.move_vocab == ref["move_vocab"]
    assert V.POSITION_TOKEN_LENGTH == ref["POSITION_TOKEN_LENGTH"]


def test_bucket_centres_match_reference():
    from chessdecoder_b200 import engine
    from oracle import model as om
    u = _utils()
    for mk in (engine, om):
        assert torch.equal(mk.make_wl_buckets(100, 0.4), u["wl_centers"])
        assert torch.equal(mk.make_d_buckets(100), u["d_centers"])


def test_oracle_backbone_matches_reference_backbone():
    from oracle.model import OracleChessDecoder
    g = _bb()
    c = g["config"]
    m = OracleChessDecoder(c["vocab_size"], embed_dim=c["embed_dim"], num_heads=c["num_heads"],
                           num_layers=c["num_layers"], max_seq_len=c["max_seq_len"], d_ff=c["d_ff"],
                           num_fourier_freq=c["num_fourier_freq"])
    missing, unexpected = m.load_state_dict(to_model_state_dict(g["state_dict"], c["num_layers"]), strict=False)
    assert not unexpected
    assert all(k.startswith(("board_head", "policy_head", "thinking_policy_head", "wl_head", "d_head", "wl_bucket", "d_bucket"))
               for k in missing), missing
    with torch.no_grad():
        h1 = m(g["input_ids"], mask_type="causal", wl_values=g["override_values"], wl_positions=g["override_mask"])
        h2 = m(g["input_ids"], mask_type="prefix", block_id=g["block_id"], wl_values=g["override_values"],
               wl_positions=g["override_mask"])
    torch.testing.assert_close(h1, g["h_causal"], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(h2, g["h_prefix"], rtol=1e-4, atol=1e-4)


def test_oracle_soft_bucket_loss_value_and_grad():
    from oracle.step import soft_bucket_loss
    u = _utils()
    logits = u["sbl_logits"].clone().requires_grad_(True)
    loss = soft_bucket_loss(logits, u["sbl_targets"], u["wl_centers"], u["sbl_valid"])
    loss.backward()
    torch.testing.assert_close(loss.detach(), u["sbl_loss"], rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(logits.grad, u["sbl_grad"], rtol=1e-5, atol=1e-7)
    z = soft_bucket_loss(logits.detach(), u["sbl_targets"], u["wl_centers"],
                         torch.zeros_like(u["sbl_valid"]))
    assert float(z) == float(u["sbl_loss_no_valid"]) == 0.0


def test_oracle_prepare_fourier_inputs():
    from oracle.model import OracleChessDecoder
    from oracle.step import prepare_fourier_inputs
    u = _utils()
    m = types.SimpleNamespace(wl_bucket_centers=u["wl_centers"], d_bucket_centers=u["d_centers"],
                              discretize_to_bucket=lambda v, c: OracleChessDecoder.discretize_to_bucket(None, v, c))
    wl_in, d_in = prepare_fourier_inputs(m, u["pf_wl_t"], u["pf_d_t"], u["pf_wl_pos"], u["pf_d_pos"])
    assert torch.equal(wl_in, u["pf_wl_in"])
    assert torch.equal(d_in, u["pf_d_in"])


def test_oracle_fourier_encoder_and_value_head():
    from oracle.model import FourierEncoder, ValueHead
    u = _utils()
    fe = FourierEncoder(32, 8)
    fe.load_state_dict(u["fe_state"])
    vh = ValueHead(32, 100, 16)
    vh.load_state_dict(u["vh_state"])
    with torch.no_grad():
        torch.testing.assert_close(fe(u["fe_x"]), u["fe_out"], rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(vh(u["vh_x"]), u["vh_out"], rtol=1e-6, atol=1e-6)


# ---------------------------------------------------------------------------
# GPU: the CUDA backbone (both passes in one merged batch) vs BackboneCausal
# ---------------------------------------------------------------------------
@pytest.mark.gpu
def test_cuda_backbone_matches_reference_backbone():
    """bf16 kernels against the reference's fp32 backbone: relative Frobenius
    error <= 2e-2 and cosine >= 0.999 for each pass."""
    from chessdecoder_b200 import kernels as K
    from chessdecoder_b200.engine import ModelConfig, TrainStep, prepare_batch, init_reference_weights
    g = _bb()
    c = g["config"]
    cfg = ModelConfig(vocab_size=c["vocab_size"], embed_dim=c["embed_dim"], num_heads=c["num_heads"],
                      num_layers=c["num_layers"], max_seq_len=c["max_seq_len"], d_ff=c["d_ff"],
                      num_fourier_freq=c["num_fourier_freq"])
    sd = init_reference_weights(cfg, seed=0)  # heads (unused here)
    sd.update(to_model_state_dict(g["state_dict"], c["num_layers"]))
    step = TrainStep(cfg, device="cuda", state_dict=sd)
    B, S = g["input_ids"].shape
    batch = {"input_ids": g["input_ids"], "board_target_ids": torch.full((B, S), -100),
             "move_target_ids": torch.full((B, S), -100), "move_mask": torch.zeros(B, S, dtype=torch.bool),
             "wl_positions": g["override_mask"], "d_positions": torch.zeros(B, S, dtype=torch.bool),
             "wl_targets": g["override_values"], "d_targets": torch.zeros(B, S),
             "wdl_valid": torch.zeros(B, S, dtype=torch.bool), "block_id": g["block_id"]}
    db = prepare_batch(batch, "cuda", require_pairing=False)
    meta = K.attn_meta(db.bid, S)
    h0, _ = step.front.forward(db, n_copies=2)
    _, h32, _ = step.backbone.forward(h0, 2 * B, B, S, db.bid, meta, want_f32=True)
    torch.cuda.synchronize()
    got = h32.view(2, B, S, -1).cpu()
    for half, ref in ((0, g["h_causal"]), (1, g["h_prefix"])):
        a, b = got[half].flatten(), ref.flatten()
        rel = ((a - b).norm() / b.norm()).item()
        cos = (a @ b / (a.norm() * b.norm())).item()
        assert rel <= 2e-2 and cos >= 0.999, (half, rel, cos)
