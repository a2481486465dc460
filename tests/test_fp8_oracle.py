"""The fp8-recipe oracle (oracle/fp8.py) on the CPU: the quantiser is the
saturating round-to-nearest-even float8 conversion of the scaled tensor, the
simulated linear's forward and gradients equal the hand-written products of
the 8-bit values, and the fp8 model keeps the base model's weights and stays
close to it."""
import torch

from oracle.fp8 import E4M3_MAX, E5M2_MAX, Fp8OracleChessDecoder, fp8_linear, quantize


def test_quantize_is_saturating_rne_of_scaled_tensor():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 96, generator=g) * 3
    q, s = quantize(x, torch.float8_e4m3fn, E4M3_MAX)
    assert torch.allclose(s, E4M3_MAX / x.abs().max())
    assert torch.equal(q, (x * s).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).float())
    assert q.abs().max() == E4M3_MAX
    q5, s5 = quantize(x, torch.float8_e5m2, E5M2_MAX)
    assert torch.equal(q5, (x * s5).clamp(-E5M2_MAX, E5M2_MAX).to(torch.float8_e5m2).float())
    z, sz = quantize(torch.zeros(4, 4), torch.float8_e4m3fn, E4M3_MAX)
    assert float(sz) == 1.0 and not z.any()


def test_fp8_linear_forward_and_gradients():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 5, 32, generator=g).requires_grad_(True)
    w = torch.randn(24, 32, generator=g).requires_grad_(True)
    y = fp8_linear(x, w)
    x8, sx = quantize(x.reshape(-1, 32), torch.float8_e4m3fn, E4M3_MAX)
    w8, sw = quantize(w, torch.float8_e4m3fn, E4M3_MAX)
    assert torch.allclose(y.reshape(-1, 24), (x8 @ w8.t()) / (sx * sw), rtol=1e-6, atol=1e-6)
    dy = torch.randn(2, 5, 24, generator=g)
    y.backward(dy)
    g8, sg = quantize(dy.reshape(-1, 24), torch.float8_e5m2, E5M2_MAX)
    assert torch.allclose(x.grad.reshape(-1, 32), (g8 @ w8) / (sg * sw), rtol=1e-6, atol=1e-6)
    assert torch.allclose(w.grad, (g8.t() @ x8) / (sg * sx), rtol=1e-6, atol=1e-6)
    # the quantised product stays close to the exact one
    rel = ((y - x @ w.t()).norm() / (x @ w.t()).norm()).item()
    assert rel < 0.05, rel


def test_fp8_model_keeps_weights_and_tracks_fp32_model():
    from chessdecoder_b200 import data
    from oracle.model import OracleChessDecoder
    from oracle.step import step_losses
    kw = dict(embed_dim=128, num_heads=2, num_layers=2, max_seq_len=128, d_ff=192)
    torch.manual_seed(0)
    base = OracleChessDecoder(1968, **kw)
    torch.manual_seed(0)
    f8 = Fp8OracleChessDecoder(1968, **kw)
    sb, s8 = base.state_dict(), f8.state_dict()
    assert sb.keys() == s8.keys() and all(torch.equal(sb[k], s8[k]) for k in sb)
    batch = data.synthetic_batches(1, 2, 128, seed=4)[0]
    lb = step_losses(base, batch)
    l8 = step_losses(f8, batch)
    for n in ("move", "board", "wl", "d"):
        assert abs(float(l8[n]) - float(lb[n])) <= 3e-2 * abs(float(lb[n])), n


def test_fp8_model_heads_follow_the_recipe():
    from oracle.model import OracleChessDecoder  # noqa: F401
    torch.manual_seed(0)
    f8 = Fp8OracleChessDecoder(1968, embed_dim=64, num_heads=2, num_layers=1, max_seq_len=32, d_ff=96)
    x = torch.randn(2, 7, 64)
    for lin in (f8.board_head, f8.policy_head, f8.thinking_policy_head, f8.wl_head.mlp[0], f8.d_head.mlp[0]):
        assert torch.equal(lin(x), fp8_linear(x, lin.weight) + lin.bias)
    # the value head's second Linear stays fp32
    h = f8.wl_head.mlp[1](f8.wl_head.mlp[0](x))
    assert torch.allclose(f8.wl_head(x), f8.wl_head.mlp[2](h))
