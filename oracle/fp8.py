"""ORACLE (test infrastructure only): the fp8 variant's recipe simulated in fp32.

The reference has no fp8 path (its linears run in fp16 under torch.autocast,
chessdecoder/train/train.py:168).  The fp8 variant's recipe, restated here
with PyTorch's float8 conversions so that the CUDA path can be checked against
the recipe itself rather than only against the fp32 step:

* every backbone linear -- the fused q|k|v projection, the output projection,
  the fused gate|up (w1|w3) projection and the down projection (w2) -- is one
  site with three quantised tensors: its input X and weight W in e4m3 (fmax
  448), the gradient of its output dY in e5m2 (fmax 57344);
* per-tensor scaling; in the first step of a run each tensor is scaled by its
  own amax: scale = fmax / amax(|t|) (1 if the tensor is all zero); the cast
  is saturating round-to-nearest-even (clamp to +-fmax, then the float8
  conversion);
* Y = (X8 W8^T) / (sX sW); dX = (dY8 W8) / (sdY sW); dW = (dY8^T X8) / (sdY sX),
  products of the 8-bit values accumulated in fp32;
* the head linears follow the same recipe: the board head on the pass-1 rows,
  the policy / thinking heads on all pass-2 rows (as the step applies them;
  the CUDA step evaluates only the rows the loss reads, whose products are the
  same, with the input scale taken over all pass-2 rows), the first Linear of
  each value head on its gathered rows; biases are added in fp32;
* the value heads' second Linear, norms, attention, softmax, the Fourier
  encoder and the embedding stay in fp32 here (the CUDA step runs them in
  bf16 / fp32).

``Fp8OracleChessDecoder`` is ``OracleChessDecoder`` with these linears; its
construction order, weights and state-dict keys are the base model's.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .model import OracleChessDecoder, apply_rope

E4M3_MAX = 448.0
E5M2_MAX = 57344.0


def quantize(t: torch.Tensor, dtype, fmax: float):
    """(fp32 values of the 8-bit tensor, scale): saturating RNE cast of t * scale."""
    amax = t.detach().abs().max()
    scale = (fmax / amax) if float(amax) > 0 else torch.ones((), device=t.device)
    q = (t.detach().float() * scale).clamp(-fmax, fmax).to(dtype).float()
    return q, scale


class _Fp8Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        x8, sx = quantize(x, torch.float8_e4m3fn, E4M3_MAX)
        w8, sw = quantize(w, torch.float8_e4m3fn, E4M3_MAX)
        ctx.save_for_backward(x8, w8, sx, sw)
        return (x8 @ w8.t()) / (sx * sw)

    @staticmethod
    def backward(ctx, g):
        x8, w8, sx, sw = ctx.saved_tensors
        g8, sg = quantize(g, torch.float8_e5m2, E5M2_MAX)
        dx = (g8 @ w8) / (sg * sw)
        dw = (g8.t() @ x8) / (sg * sx)
        return dx, dw


def fp8_linear(x, w):
    """y = x W^T with the recipe's quantisation; x [..., K], w [N, K]."""
    shp = x.shape
    y = _Fp8Linear.apply(x.reshape(-1, shp[-1]), w)
    return y.reshape(*shp[:-1], w.shape[0])


def _fp8_head(lin):
    def forward(x):
        return fp8_linear(x, lin.weight) + lin.bias
    return forward


class Fp8OracleChessDecoder(OracleChessDecoder):
    """OracleChessDecoder whose four backbone linears per layer and whose head
    linears follow the fp8 recipe."""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        for lin in (self.board_head, self.policy_head, self.thinking_policy_head, self.wl_head.mlp[0],
                    self.d_head.mlp[0]):
            lin.forward = _fp8_head(lin)  # an instance attribute: parameters and state-dict keys unchanged

    def _layer(self, layer, x, mask, input_pos):
        B, S, E = x.shape
        h = layer.sa_norm(x)
        a = layer.attn
        wqkv = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0)
        qkv = fp8_linear(h, wqkv)
        q, k, v = qkv.split(E, dim=-1)
        q = apply_rope(q.reshape(B, S, a.num_heads, a.head_dim), self.rope, input_pos).transpose(1, 2)
        k = apply_rope(k.reshape(B, S, a.num_heads, a.head_dim), self.rope, input_pos).transpose(1, 2)
        v = v.reshape(B, S, a.num_heads, a.head_dim).transpose(1, 2)
        if mask is None:
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        else:
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask[:, None])
        x = x + fp8_linear(o.transpose(1, 2).reshape(B, S, E), a.output_proj.weight)
        m = layer.mlp
        n2 = layer.mlp_norm(x)
        gu = fp8_linear(n2, torch.cat([m.w1.weight, m.w3.weight], 0))
        g, u = gu.split(m.w1.weight.shape[0], dim=-1)
        return x + fp8_linear(F.silu(g) * u, m.w2.weight)
