"""Checkpoint layout of the fused step (CPU): the parameter order used for
optimizer state indices is the reference model's ``parameters()`` order, and
the AdamW state exported from the flat store loads into
``torch.optim.AdamW(model.parameters())`` and back
(chessdecoder/utils/training.py:136-157, chessdecoder/train/train.py:81-104)."""
import pytest
import torch

from chessdecoder_b200.engine import ModelConfig, ParamStore, reference_param_names

SMALL = dict(embed_dim=64, num_heads=2, num_layers=2, max_seq_len=64, d_ff=96)


@pytest.mark.parametrize("moe", [0, 4])
def test_reference_param_order(moe):
    from oracle.model import OracleChessDecoder
    kw = dict(SMALL, moe_experts=moe)
    cfg = ModelConfig(**kw)
    names = [n for n, _ in OracleChessDecoder(cfg.vocab_size, **kw).named_parameters()]
    assert reference_param_names(cfg) == names


def test_dropin_module_param_order():
    from chessdecoder_b200.model import ChessDecoder
    cfg = ModelConfig(**SMALL)
    with torch.device("meta"):
        m = ChessDecoder(cfg.vocab_size, **SMALL)
    assert [n for n, _ in m.named_parameters()] == reference_param_names(cfg)


def test_optimizer_state_round_trips_through_torch_adamw():
    from oracle.model import OracleChessDecoder
    cfg = ModelConfig(**SMALL)
    st = ParamStore(cfg, "cpu")
    g = torch.Generator().manual_seed(0)
    st.exp_avg.copy_(torch.randn(st.numel, generator=g))
    st.exp_avg_sq.copy_(torch.rand(st.numel, generator=g))
    st.step = 7
    sd = st.optimizer_state_dict(3e-4, (0.9, 0.999), 1e-8, 0.1)
    # loads into the reference-shaped model's AdamW (shapes and indices checked there)
    model = OracleChessDecoder(cfg.vocab_size, **SMALL)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, weight_decay=0.1)
    opt.load_state_dict(sd)
    named = dict(model.named_parameters())
    assert named["thinking_policy_head.weight"] not in opt.state  # never stepped in pretraining
    for name in st.names():
        s = opt.state[named[name]]
        assert torch.equal(s["exp_avg"], st._view(st.exp_avg, name))
        assert float(s["step"]) == 7.0
    # ... and back from the torch optimizer's own state_dict
    st2 = ParamStore(cfg, "cpu")
    grp = st2.load_optimizer_state_dict(opt.state_dict())
    assert st2.step == 7 and grp["weight_decay"] == 0.1
    for name in st.names():
        assert torch.equal(st2._view(st2.exp_avg, name), st._view(st.exp_avg, name))
        assert torch.equal(st2._view(st2.exp_avg_sq, name), st._view(st.exp_avg_sq, name))


def test_mismatched_optimizer_state_is_rejected():
    cfg = ModelConfig(**SMALL)
    st = ParamStore(cfg, "cpu")
    sd = st.optimizer_state_dict(1e-3, (0.9, 0.999), 1e-8, 0.0)
    sd["param_groups"][0]["params"] = sd["param_groups"][0]["params"][:-1]
    with pytest.raises(ValueError):
        st.load_optimizer_state_dict(sd)
